// 16x16-tile compositors: forward (front-to-back alpha blending with
// optional expected depth and any number of channels) and backward
// (back-to-front replay with gradient reduction before global atomics).
//
// Reference: the gs_rasterize_forward / gs_rasterize_backward /
// gs_rasterize_depth Metal kernels, src/mlx3d/splatting/rasterize.py:28-290.
// One CTA per tile, one thread per pixel, Gaussians staged 256 at a time in
// shared memory.  Per-pixel arithmetic uses gs_math.h's exactly rounded
// operations in the reference's order, so image / final_T / n_contrib / depth
// are bit-identical to the CPU oracle's.
#include "gs_common.cuh"

namespace gs {

struct RasterArgs {
  const float *means2d, *conics, *colors, *opac, *depths;
  const int32_t *ids, *ranges;
  const float* bg;
  int c_total, c0, cc;  // channel count, first channel of this launch, channels in it
  int width, height, tiles_x, tiles_y;
  float *image, *final_T, *depth;
  int32_t* n_contrib;
  int write_aux;  // final_T / n_contrib / depth written by this launch
};

// Opacity-aware early reject: alpha = min(0.99, o*e^p) < 1/255 is certain
// when p < ln(1/(255 o)) - margin.  The margin (1e-3) is far above the error
// of gs_expf (< 2 ulp), so the skip never changes a decision of the exact
// test; it only avoids evaluating the exponential.
__device__ __forceinline__ float power_floor(float o) {
  return o > 0.0f ? -logf(255.0f * o) - 1e-3f : INFINITY;
}

template <int CMAX, bool DEPTH>
__global__ void __launch_bounds__(GS_BLOCK) k_raster_fwd(const RasterArgs a) {
  __shared__ float2 s_xy[GS_BLOCK];
  __shared__ float4 s_co[GS_BLOCK];  // conic a, b, c, opacity
  __shared__ float s_pf[GS_BLOCK];   // power floor
  __shared__ float s_col[CMAX > 0 ? CMAX : 1][GS_BLOCK];
  __shared__ float s_z[DEPTH ? GS_BLOCK : 1];

  const int tile = blockIdx.x;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  const int px = tx * GS_TILE + (threadIdx.x & 15);
  const int py = ty * GS_TILE + (threadIdx.x >> 4);
  const bool inside = px < a.width && py < a.height;
  const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
  const int start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  const int num = end - start;

  float T = 1.0f;
  float acc[CMAX > 0 ? CMAX : 1];
#pragma unroll
  for (int ch = 0; ch < (CMAX > 0 ? CMAX : 1); ++ch) acc[ch] = 0.0f;
  float dacc = 0.0f;
  int last = 0;
  bool done = !inside;

  for (int b0 = 0; b0 < num; b0 += GS_BLOCK) {
    // Barrier before the batch overwrites shared memory; also ends the tile
    // once every pixel has terminated.
    if (__syncthreads_count(done) == GS_BLOCK) break;
    const int li = start + b0 + threadIdx.x;
    if (li < end) {
      const int g = __ldg(a.ids + li);
      s_xy[threadIdx.x] = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
      const float o = __ldg(a.opac + g);
      s_co[threadIdx.x] = make_float4(__ldg(a.conics + 3 * g), __ldg(a.conics + 3 * g + 1),
                                      __ldg(a.conics + 3 * g + 2), o);
      s_pf[threadIdx.x] = power_floor(o);
#pragma unroll
      for (int ch = 0; ch < CMAX; ++ch)
        if (ch < a.cc) s_col[ch][threadIdx.x] = __ldg(a.colors + (int64_t)g * a.c_total + a.c0 + ch);
      if (DEPTH) s_z[threadIdx.x] = __ldg(a.depths + g);
    }
    __syncthreads();
    if (done) continue;
    const int bs = min(GS_BLOCK, num - b0);
    for (int j = 0; j < bs; ++j) {
      const float2 m = s_xy[j];
      const float4 co = s_co[j];
      const float dx = gs_sub(m.x, pxf), dy = gs_sub(m.y, pyf);
      const float power = gs_sub(
          gs_mul(-0.5f, gs_add(gs_mul(gs_mul(co.x, dx), dx), gs_mul(gs_mul(co.z, dy), dy))),
          gs_mul(gs_mul(co.y, dx), dy));
      if (power > 0.0f || power < s_pf[j]) continue;
      const float alpha = gs_minf(GS_ALPHA_MAX, gs_mul(co.w, gs_expf(power)));
      if (alpha < GS_ALPHA_MIN) continue;
      const float next_T = gs_mul(T, gs_sub(1.0f, alpha));
      if (next_T < GS_T_MIN) {
        done = true;
        break;
      }
      const float w = gs_mul(alpha, T);
#pragma unroll
      for (int ch = 0; ch < CMAX; ++ch) acc[ch] = gs_add(acc[ch], gs_mul(s_col[ch][j], w));
      if (DEPTH) dacc = gs_add(dacc, gs_mul(s_z[j], w));
      T = next_T;
      last = b0 + j + 1;
    }
  }
  if (!inside) return;
  const int64_t pid = (int64_t)py * a.width + px;
  if (a.image) {
#pragma unroll
    for (int ch = 0; ch < CMAX; ++ch) {
      if (ch < a.cc) {
        const float bgv = a.bg ? a.bg[a.c0 + ch] : 0.0f;
        a.image[pid * a.c_total + a.c0 + ch] = gs_add(acc[ch], gs_mul(T, bgv));
      }
    }
  }
  if (a.write_aux) {
    if (a.final_T) a.final_T[pid] = T;
    if (a.n_contrib) a.n_contrib[pid] = last;
    if (DEPTH && a.depth) {
      const float al = gs_sub(1.0f, T);
      a.depth[pid] = al > 1e-6f ? gs_div(dacc, al) : 0.0f;
    }
  }
}

struct RasterBwdArgs {
  RasterArgs f;
  const float *grad_image, *grad_final_T;
  int use_grad_final_T;
  float *g_means2d, *g_conics, *g_colors, *g_opac;
};

// Gradient slots per staged Gaussian: 0-1 means2d, 2-4 conic, 5 opacity,
// 6.. colour channels.
template <int CMAX>
__global__ void __launch_bounds__(GS_BLOCK) k_raster_bwd(const RasterBwdArgs g) {
  const RasterArgs& a = g.f;
  constexpr int NG = 6 + CMAX;
  __shared__ int s_id[GS_BLOCK];
  __shared__ float2 s_xy[GS_BLOCK];
  __shared__ float4 s_co[GS_BLOCK];
  __shared__ float s_col[CMAX][GS_BLOCK];
  __shared__ float s_g[NG][GS_BLOCK];
  __shared__ int s_hit[GS_BLOCK];
  __shared__ int s_max_last;

  const int tile = blockIdx.x;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  const int px = tx * GS_TILE + (threadIdx.x & 15);
  const int py = ty * GS_TILE + (threadIdx.x >> 4);
  const bool inside = px < a.width && py < a.height;
  const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
  const int64_t pid = (int64_t)py * a.width + px;
  const int start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  const int num = end - start;
  const int lane = threadIdx.x & 31;

  const float T_final = inside ? a.final_T[pid] : 1.0f;
  float T = T_final;
  const int last = inside ? a.n_contrib[pid] : 0;
  float dpix[CMAX];
  float bg_dot = 0.0f;
#pragma unroll
  for (int ch = 0; ch < CMAX; ++ch) {
    dpix[ch] = 0.0f;
    if (inside && ch < a.cc) {
      dpix[ch] = g.grad_image[pid * a.c_total + a.c0 + ch];
      if (a.bg) bg_dot += a.bg[a.c0 + ch] * dpix[ch];
    }
  }
  if (inside && g.use_grad_final_T && g.grad_final_T) bg_dot += g.grad_final_T[pid];
  float accum[CMAX], last_color[CMAX];
#pragma unroll
  for (int ch = 0; ch < CMAX; ++ch) accum[ch] = last_color[ch] = 0.0f;
  float last_alpha = 0.0f;

  // Nothing at or beyond the largest n_contrib of this warp (block) matters.
  int wmax = last;
  for (int o = 16; o > 0; o >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  if (threadIdx.x == 0) s_max_last = 0;
  __syncthreads();
  if (lane == 0) atomicMax(&s_max_last, wmax);
  __syncthreads();
  const int block_last = s_max_last;
  const int nbat = (block_last + GS_BLOCK - 1) / GS_BLOCK;

  for (int b = nbat - 1; b >= 0; --b) {
    const int b0 = b * GS_BLOCK;
    __syncthreads();
    const int li = start + b0 + threadIdx.x;
    if (li < end) {
      const int gid = __ldg(a.ids + li);
      s_id[threadIdx.x] = gid;
      s_xy[threadIdx.x] = __ldg(reinterpret_cast<const float2*>(a.means2d) + gid);
      s_co[threadIdx.x] = make_float4(__ldg(a.conics + 3 * gid), __ldg(a.conics + 3 * gid + 1),
                                      __ldg(a.conics + 3 * gid + 2), __ldg(a.opac + gid));
#pragma unroll
      for (int ch = 0; ch < CMAX; ++ch)
        s_col[ch][threadIdx.x] =
            ch < a.cc ? __ldg(a.colors + (int64_t)gid * a.c_total + a.c0 + ch) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < NG; ++k) s_g[k][threadIdx.x] = 0.0f;
    s_hit[threadIdx.x] = 0;
    __syncthreads();
    const int bs = min(GS_BLOCK, num - b0);
    const int jtop = min(bs, wmax - b0) - 1;
    for (int j = jtop; j >= 0; --j) {
      bool contrib = inside && (b0 + j < last);
      float G = 0.0f, alpha = 0.0f, dx = 0.0f, dy = 0.0f;
      const float4 co = s_co[j];
      if (contrib) {
        const float2 m = s_xy[j];
        dx = gs_sub(m.x, pxf);
        dy = gs_sub(m.y, pyf);
        const float power = gs_sub(
            gs_mul(-0.5f, gs_add(gs_mul(gs_mul(co.x, dx), dx), gs_mul(gs_mul(co.z, dy), dy))),
            gs_mul(gs_mul(co.y, dx), dy));
        if (power > 0.0f) {
          contrib = false;
        } else {
          G = gs_expf(power);
          alpha = gs_minf(GS_ALPHA_MAX, gs_mul(co.w, G));
          if (alpha < GS_ALPHA_MIN) contrib = false;
        }
      }
      float gv[NG];
#pragma unroll
      for (int k = 0; k < NG; ++k) gv[k] = 0.0f;
      if (contrib) {
        T = T / (1.0f - alpha);
        const float aT = alpha * T;
        float dL_dalpha = 0.0f;
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch) {
          const float c = s_col[ch][j];
          accum[ch] = last_alpha * last_color[ch] + (1.0f - last_alpha) * accum[ch];
          last_color[ch] = c;
          dL_dalpha += (c - accum[ch]) * dpix[ch];
          gv[6 + ch] = aT * dpix[ch];
        }
        last_alpha = alpha;
        dL_dalpha *= T;
        dL_dalpha += (-T_final / (1.0f - alpha)) * bg_dot;
        const float dL_dG = co.w * dL_dalpha;
        const float gdx = G * dx, gdy = G * dy;
        gv[0] = -(gdx * co.x + gdy * co.y) * dL_dG;
        gv[1] = -(gdy * co.z + gdx * co.y) * dL_dG;
        gv[2] = -0.5f * gdx * dx * dL_dG;
        gv[3] = -gdx * dy * dL_dG;
        gv[4] = -0.5f * gdy * dy * dL_dG;
        gv[5] = G * dL_dalpha;
      }
      if (__any_sync(0xffffffffu, contrib)) {
#pragma unroll
        for (int k = 0; k < NG; ++k) {
          if (k >= 6 + a.cc) break;
          float v = gv[k];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          gv[k] = v;
        }
        if (lane == 0) {
          for (int k = 0; k < 6 + a.cc; ++k) atomicAdd(&s_g[k][j], gv[k]);
          s_hit[j] = 1;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x < bs && s_hit[threadIdx.x]) {
      const int gid = s_id[threadIdx.x];
      atomicAdd(g.g_means2d + 2 * gid, s_g[0][threadIdx.x]);
      atomicAdd(g.g_means2d + 2 * gid + 1, s_g[1][threadIdx.x]);
      atomicAdd(g.g_conics + 3 * gid, s_g[2][threadIdx.x]);
      atomicAdd(g.g_conics + 3 * gid + 1, s_g[3][threadIdx.x]);
      atomicAdd(g.g_conics + 3 * gid + 2, s_g[4][threadIdx.x]);
      atomicAdd(g.g_opac + gid, s_g[5][threadIdx.x]);
      for (int ch = 0; ch < a.cc; ++ch)
        atomicAdd(g.g_colors + (int64_t)gid * a.c_total + a.c0 + ch, s_g[6 + ch][threadIdx.x]);
    }
  }
}

// Channel chunk widths the kernels are instantiated for.
static int pick_cmax(int c) {
  if (c <= 1) return 1;
  if (c <= 2) return 2;
  if (c <= 3) return 3;
  if (c <= 4) return 4;
  if (c <= 8) return 8;
  return 16;
}
constexpr int kMaxChunk = 16;

template <int CMAX>
static void launch_fwd(const RasterArgs& a, bool depth, int grid, cudaStream_t s) {
  if (depth)
    k_raster_fwd<CMAX, true><<<grid, GS_BLOCK, 0, s>>>(a);
  else
    k_raster_fwd<CMAX, false><<<grid, GS_BLOCK, 0, s>>>(a);
}

static void dispatch_fwd(const RasterArgs& a, bool depth, int grid, cudaStream_t s) {
  switch (a.cc == 0 ? 0 : pick_cmax(a.cc)) {
    case 0: launch_fwd<0>(a, depth, grid, s); break;
    case 1: launch_fwd<1>(a, depth, grid, s); break;
    case 2: launch_fwd<2>(a, depth, grid, s); break;
    case 3: launch_fwd<3>(a, depth, grid, s); break;
    case 4: launch_fwd<4>(a, depth, grid, s); break;
    case 8: launch_fwd<8>(a, depth, grid, s); break;
    default: launch_fwd<16>(a, depth, grid, s); break;
  }
}

static void dispatch_bwd(const RasterBwdArgs& g, int grid, cudaStream_t s) {
  switch (pick_cmax(g.f.cc)) {
    case 1: k_raster_bwd<1><<<grid, GS_BLOCK, 0, s>>>(g); break;
    case 2: k_raster_bwd<2><<<grid, GS_BLOCK, 0, s>>>(g); break;
    case 3: k_raster_bwd<3><<<grid, GS_BLOCK, 0, s>>>(g); break;
    case 4: k_raster_bwd<4><<<grid, GS_BLOCK, 0, s>>>(g); break;
    case 8: k_raster_bwd<8><<<grid, GS_BLOCK, 0, s>>>(g); break;
    default: k_raster_bwd<16><<<grid, GS_BLOCK, 0, s>>>(g); break;
  }
}

static int check_raster_args(int channels, int width, int height, int tiles_x, int tiles_y) {
  if (channels < 0 || channels > 1024)
    return set_error(GS_ERR_INVALID_ARG, "channels must be in [0, 1024] (got %d)", channels);
  if (width <= 0 || height <= 0) return set_error(GS_ERR_INVALID_ARG, "image size must be positive");
  if (tiles_x != (int)ceil_div(width, GS_TILE) || tiles_y != (int)ceil_div(height, GS_TILE))
    return set_error(GS_ERR_INVALID_ARG, "tiles_x/tiles_y (%d, %d) do not match a %dx%d image",
                     tiles_x, tiles_y, width, height);
  return GS_OK;
}

}  // namespace gs

using namespace gs;

extern "C" {

int gs_rasterize_forward(const float* means2d, const float* conics, const float* colors,
                         int channels, const float* opacities, const float* depths,
                         const int32_t* sorted_ids, const int32_t* tile_ranges,
                         const float* background, int width, int height, int tiles_x,
                         int tiles_y, float* image, float* final_T, int32_t* n_contrib,
                         float* depth, void* stream) {
  clear_error();
  if (int e = check_raster_args(channels, width, height, tiles_x, tiles_y)) return e;
  if (!means2d || !conics || !opacities || !sorted_ids || !tile_ranges || !final_T)
    return set_error(GS_ERR_INVALID_ARG, "gs_rasterize_forward: NULL pointer");
  if (channels > 0 && (!colors || !image))
    return set_error(GS_ERR_INVALID_ARG, "colors / image must be given when channels > 0");
  if (depth && !depths) return set_error(GS_ERR_INVALID_ARG, "depth output needs depths");
  if (!aligned(means2d, 8)) return set_error(GS_ERR_INVALID_ARG, "means2d must be 8-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int grid = tiles_x * tiles_y;
  RasterArgs a{};
  a.means2d = means2d; a.conics = conics; a.colors = colors; a.opac = opacities; a.depths = depths;
  a.ids = sorted_ids; a.ranges = tile_ranges; a.bg = background;
  a.c_total = channels;
  a.width = width; a.height = height; a.tiles_x = tiles_x; a.tiles_y = tiles_y;
  a.image = image; a.final_T = final_T; a.depth = depth; a.n_contrib = n_contrib;
  if (channels == 0) {
    a.c0 = 0; a.cc = 0; a.write_aux = 1;
    dispatch_fwd(a, depth != nullptr, grid, s);
    return check_launch("k_raster_fwd");
  }
  for (int c0 = 0; c0 < channels; c0 += kMaxChunk) {
    a.c0 = c0;
    a.cc = channels - c0 < kMaxChunk ? channels - c0 : kMaxChunk;
    a.write_aux = c0 == 0;
    dispatch_fwd(a, c0 == 0 && depth != nullptr, grid, s);
    if (int e = check_launch("k_raster_fwd")) return e;
  }
  return GS_OK;
}

int gs_rasterize_backward(const float* means2d, const float* conics, const float* colors,
                          int channels, const float* opacities, int64_t n,
                          const int32_t* sorted_ids, const int32_t* tile_ranges,
                          const float* background, int width, int height, int tiles_x,
                          int tiles_y, const float* final_T, const int32_t* n_contrib,
                          const float* grad_image, const float* grad_final_T,
                          float* grad_means2d, float* grad_conics, float* grad_colors,
                          float* grad_opacities, void* stream) {
  clear_error();
  if (int e = check_raster_args(channels, width, height, tiles_x, tiles_y)) return e;
  if (channels < 1) return set_error(GS_ERR_INVALID_ARG, "backward needs channels >= 1");
  if (!means2d || !conics || !colors || !opacities || !sorted_ids || !tile_ranges || !final_T ||
      !n_contrib || !grad_image || !grad_means2d || !grad_conics || !grad_colors || !grad_opacities)
    return set_error(GS_ERR_INVALID_ARG, "gs_rasterize_backward: NULL pointer");
  if (!aligned(means2d, 8)) return set_error(GS_ERR_INVALID_ARG, "means2d must be 8-byte aligned");
  cudaStream_t s = as_stream(stream);
  if (n > 0) {
    bool ok = cudaMemsetAsync(grad_means2d, 0, sizeof(float) * 2 * n, s) == cudaSuccess &&
              cudaMemsetAsync(grad_conics, 0, sizeof(float) * 3 * n, s) == cudaSuccess &&
              cudaMemsetAsync(grad_colors, 0, sizeof(float) * channels * n, s) == cudaSuccess &&
              cudaMemsetAsync(grad_opacities, 0, sizeof(float) * n, s) == cudaSuccess;
    if (!ok) return set_error(GS_ERR_CUDA, "cudaMemsetAsync failed");
  }
  const int grid = tiles_x * tiles_y;
  RasterBwdArgs g{};
  RasterArgs& a = g.f;
  a.means2d = means2d; a.conics = conics; a.colors = colors; a.opac = opacities;
  a.ids = sorted_ids; a.ranges = tile_ranges; a.bg = background;
  a.c_total = channels;
  a.width = width; a.height = height; a.tiles_x = tiles_x; a.tiles_y = tiles_y;
  a.final_T = const_cast<float*>(final_T); a.n_contrib = const_cast<int32_t*>(n_contrib);
  g.grad_image = grad_image; g.grad_final_T = grad_final_T;
  g.g_means2d = grad_means2d; g.g_conics = grad_conics; g.g_colors = grad_colors;
  g.g_opac = grad_opacities;
  for (int c0 = 0; c0 < channels; c0 += kMaxChunk) {
    a.c0 = c0;
    a.cc = channels - c0 < kMaxChunk ? channels - c0 : kMaxChunk;
    g.use_grad_final_T = c0 == 0;
    dispatch_bwd(g, grid, s);
    if (int e = check_launch("k_raster_bwd")) return e;
  }
  return GS_OK;
}

}  // extern "C"
