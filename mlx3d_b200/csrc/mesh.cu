// Hard z-buffer mesh rasterizer: the nearest triangle per pixel over the
// triangles binned to the pixel's 16x16 tile (src/mlx3d/renderer/
// rasterizer.py:29-79, the mesh_rasterize_hard_tiled Metal kernel, and its
// caller rasterize_meshes, :120-162, which bins the triangles with the
// Gaussian tiler by their bounding circles).
//
// One 256-thread CTA per tile, one thread per pixel; the tile's triangles
// (screen-space corners and camera depths) are staged 256 at a time in
// shared memory and scanned in the binned order.  Per pixel, per triangle:
// barycentrics l0, l1 by the edge-function formula of the reference,
// l2 = 1 - l0 - l1; skip when |denom| < 1e-12 or any l < -1e-5; depth
// z = l0 z0 + l1 z1 + l2 z2; skip z <= znear; keep the strictly smallest z
// (the first in binned order on ties).  Every operation is an exactly
// rounded gs_math.h primitive in the reference's order, so the result is
// bit-identical to the CPU oracle's.
#include "gs_common.cuh"

namespace gs {

constexpr int kMeshThreads = GS_TILE * GS_TILE;
constexpr int kMeshBatch = 256;

struct MeshArgs {
  const float *tri_xy, *tri_z;
  const int32_t *ids, *ranges;
  int64_t n_faces;
  int width, height, tiles_x;
  float znear;
  int32_t* pix_to_face;
  float* zbuf;
};

__global__ void __launch_bounds__(kMeshThreads) k_mesh_raster(const MeshArgs a) {
  __shared__ float s_xy[6][kMeshBatch];
  __shared__ float s_z[3][kMeshBatch];
  __shared__ int s_f[kMeshBatch];
  const int tile = blockIdx.x;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  const int px = tx * GS_TILE + (int)(threadIdx.x % GS_TILE);
  const int py = ty * GS_TILE + (int)(threadIdx.x / GS_TILE);
  const float cx = gs_add((float)px, 0.5f), cy = gs_add((float)py, 0.5f);
  const int start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  int best_f = -1;
  float best_z = 1e30f;
  for (int b0 = start; b0 < end; b0 += kMeshBatch) {
    __syncthreads();  // the previous batch is no longer read
    const int li = b0 + (int)threadIdx.x;
    if (li < end) {
      const int f = a.ids[li];
      const bool ok = f >= 0 && (int64_t)f < a.n_faces;
      s_f[threadIdx.x] = ok ? f : -1;
#pragma unroll
      for (int k = 0; k < 6; ++k) s_xy[k][threadIdx.x] = ok ? a.tri_xy[(int64_t)f * 6 + k] : 0.0f;
#pragma unroll
      for (int k = 0; k < 3; ++k) s_z[k][threadIdx.x] = ok ? a.tri_z[(int64_t)f * 3 + k] : 0.0f;
    }
    __syncthreads();
    const int bs = min(kMeshBatch, end - b0);
    for (int j = 0; j < bs; ++j) {
      const int f = s_f[j];
      if (f < 0) continue;
      const float ax = s_xy[0][j], ay = s_xy[1][j], bx = s_xy[2][j], by = s_xy[3][j];
      const float ccx = s_xy[4][j], ccy = s_xy[5][j];
      const float denom =
          gs_add(gs_mul(gs_sub(by, ccy), gs_sub(ax, ccx)), gs_mul(gs_sub(ccx, bx), gs_sub(ay, ccy)));
      if (fabsf(denom) < 1e-12f) continue;
      const float dx = gs_sub(cx, ccx), dy = gs_sub(cy, ccy);
      const float l0 = gs_div(gs_add(gs_mul(gs_sub(by, ccy), dx), gs_mul(gs_sub(ccx, bx), dy)), denom);
      const float l1 = gs_div(gs_add(gs_mul(gs_sub(ccy, ay), dx), gs_mul(gs_sub(ax, ccx), dy)), denom);
      const float l2 = gs_sub(gs_sub(1.0f, l0), l1);
      if (l0 < -1e-5f || l1 < -1e-5f || l2 < -1e-5f) continue;
      const float z = gs_add(gs_add(gs_mul(l0, s_z[0][j]), gs_mul(l1, s_z[1][j])), gs_mul(l2, s_z[2][j]));
      if (z <= a.znear) continue;
      if (z < best_z) {
        best_z = z;
        best_f = f;
      }
    }
  }
  if (px < a.width && py < a.height) {
    const int64_t idx = (int64_t)py * a.width + px;
    a.pix_to_face[idx] = best_f;
    a.zbuf[idx] = best_f >= 0 ? best_z : 0.0f;
  }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_mesh_rasterize(const float* tri_xy, const float* tri_z, int64_t n_faces, const int32_t* sorted_ids,
                                 const int32_t* tile_ranges, int width, int height, float znear,
                                 int32_t* pix_to_face, float* zbuf, void* stream) {
  clear_error();
  if (width <= 0 || height <= 0) return set_error(GS_ERR_INVALID_ARG, "image size must be positive");
  if (n_faces < 0) return set_error(GS_ERR_INVALID_ARG, "n_faces must be >= 0");
  if (!tile_ranges || !pix_to_face || !zbuf) return set_error(GS_ERR_INVALID_ARG, "gs_mesh_rasterize: NULL pointer");
  // sorted_ids is read only inside non-empty tile ranges (it may be NULL when D = 0)
  if (n_faces > 0 && (!tri_xy || !tri_z))
    return set_error(GS_ERR_INVALID_ARG, "gs_mesh_rasterize: NULL pointer");
  MeshArgs a{};
  a.tri_xy = tri_xy;
  a.tri_z = tri_z;
  a.ids = sorted_ids;
  a.ranges = tile_ranges;
  a.n_faces = n_faces;
  a.width = width;
  a.height = height;
  a.tiles_x = (int)ceil_div(width, GS_TILE);
  a.znear = znear;
  a.pix_to_face = pix_to_face;
  a.zbuf = zbuf;
  const int tiles_y = (int)ceil_div(height, GS_TILE);
  k_mesh_raster<<<(unsigned)(a.tiles_x * tiles_y), kMeshThreads, 0, as_stream(stream)>>>(a);
  return check_launch("k_mesh_raster");
}
