// CPU ORACLE — TEST INFRASTRUCTURE ONLY.
//
// A plain C++ restatement of mlx3D's Gaussian-splatting path, used by tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference arm
// as the checker and CPU baseline.  Product code never calls it.
//
// Each function follows the reference file:line named in its comment, in the
// reference's order of float32 operations.  Exactly rounded float32 primitives
// and the exponential come from mlx3d_b200/csrc/gs_math.h (the reference's
// MLX / Metal exp is not reproducible off Apple hardware; both this oracle and
// the CUDA kernels use the same published-method exp so cut-off decisions
// agree bit for bit).  Build: oracle/Makefile (-O2 -ffp-contract=off, OpenMP).
//
// Parity pinning: MLX cannot run in this environment (macOS arm64 wheels
// only), so the oracle is pinned by the known-answer tests of the reference's
// own test suite (tests/test_splatting.py:57-72, 114-195, 198-211) and by the
// naive O(N*H*W) renderer of src/mlx3d/splatting/reference.py restated in
// oracle/torch_ref.py; see tests/test_oracle.py.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/gsplat_b200.h"
#include "../mlx3d_b200/csrc/gs_math.h"

namespace {

constexpr int TILE = 16;
constexpr int BLOCK = 256;

// projection.py:56-138, one Gaussian.
void project_one(const gs_camera& cam, const float* m, const float* qr, const float* s, float blur,
                 bool aa, float* out_uv, float* out_conic, float* out_z, float* out_r,
                 float* out_comp) {
  const float* R = cam.R;
  const float x = gs_add(gs_add(gs_add(gs_mul(m[0], R[0]), gs_mul(m[1], R[1])), gs_mul(m[2], R[2])), cam.t[0]);
  const float y = gs_add(gs_add(gs_add(gs_mul(m[0], R[3]), gs_mul(m[1], R[4])), gs_mul(m[2], R[5])), cam.t[1]);
  const float z = gs_add(gs_add(gs_add(gs_mul(m[0], R[6]), gs_mul(m[1], R[7])), gs_mul(m[2], R[8])), cam.t[2]);
  const float z_safe = gs_maxf(z, 1e-6f);  // :61
  out_uv[0] = gs_add(gs_div(gs_mul(cam.fx, x), z_safe), cam.cx);  // :64
  out_uv[1] = gs_add(gs_div(gs_mul(cam.fy, y), z_safe), cam.cy);  // :65
  // clip(v, lo, hi) = minimum(maximum(v, lo), hi)  (:72-73)
  const float tx = gs_mul(gs_minf(gs_maxf(gs_div(x, z_safe), -cam.clip_x), cam.clip_x), z_safe);
  const float ty = gs_mul(gs_minf(gs_maxf(gs_div(y, z_safe), -cam.clip_y), cam.clip_y), z_safe);
  const float inv_z = gs_div(1.0f, z_safe);
  const float inv_z2 = gs_mul(inv_z, inv_z);
  const float j00 = gs_mul(cam.fx, inv_z);
  const float j02 = gs_mul(gs_mul(cam.neg_fx, tx), inv_z2);
  const float j11 = gs_mul(cam.fy, inv_z);
  const float j12 = gs_mul(gs_mul(cam.neg_fy, ty), inv_z2);
  float T[2][3];
  for (int k = 0; k < 3; ++k) {  // :87-92
    T[0][k] = gs_add(gs_mul(j00, R[k]), gs_mul(j02, R[6 + k]));
    T[1][k] = gs_add(gs_mul(j11, R[3 + k]), gs_mul(j12, R[6 + k]));
  }
  const float nrm = gs_sqrt(gs_add(gs_add(gs_add(gs_mul(qr[0], qr[0]), gs_mul(qr[1], qr[1])), gs_mul(qr[2], qr[2])), gs_mul(qr[3], qr[3])));
  const float qw = gs_div(qr[0], nrm), qx = gs_div(qr[1], nrm), qy = gs_div(qr[2], nrm), qz = gs_div(qr[3], nrm);
  float Q[3][3];  // :97-105
  Q[0][0] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(qy, qy), gs_mul(qz, qz))));
  Q[0][1] = gs_mul(2.0f, gs_sub(gs_mul(qx, qy), gs_mul(qw, qz)));
  Q[0][2] = gs_mul(2.0f, gs_add(gs_mul(qx, qz), gs_mul(qw, qy)));
  Q[1][0] = gs_mul(2.0f, gs_add(gs_mul(qx, qy), gs_mul(qw, qz)));
  Q[1][1] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(qx, qx), gs_mul(qz, qz))));
  Q[1][2] = gs_mul(2.0f, gs_sub(gs_mul(qy, qz), gs_mul(qw, qx)));
  Q[2][0] = gs_mul(2.0f, gs_sub(gs_mul(qx, qz), gs_mul(qw, qy)));
  Q[2][1] = gs_mul(2.0f, gs_add(gs_mul(qy, qz), gs_mul(qw, qx)));
  Q[2][2] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(qx, qx), gs_mul(qy, qy))));
  float M[2][3];  // :108-113
  for (int r = 0; r < 2; ++r)
    for (int k = 0; k < 3; ++k)
      M[r][k] = gs_mul(gs_add(gs_add(gs_mul(T[r][0], Q[0][k]), gs_mul(T[r][1], Q[1][k])), gs_mul(T[r][2], Q[2][k])), s[k]);
  const float a0 = gs_add(gs_add(gs_mul(M[0][0], M[0][0]), gs_mul(M[0][1], M[0][1])), gs_mul(M[0][2], M[0][2]));
  const float b = gs_add(gs_add(gs_mul(M[0][0], M[1][0]), gs_mul(M[0][1], M[1][1])), gs_mul(M[0][2], M[1][2]));
  const float c0 = gs_add(gs_add(gs_mul(M[1][0], M[1][0]), gs_mul(M[1][1], M[1][1])), gs_mul(M[1][2], M[1][2]));
  const float a = gs_add(a0, blur), c = gs_add(c0, blur);  // :119-120
  const float det = gs_sub(gs_mul(a, c), gs_mul(b, b));
  const float det_safe = gs_maxf(det, 1e-12f);
  out_conic[0] = gs_div(c, det_safe);
  out_conic[1] = gs_div(-b, det_safe);
  out_conic[2] = gs_div(a, det_safe);
  float comp = 1.0f;
  if (aa && blur > 0.0f) comp = gs_sqrt(gs_div(gs_maxf(gs_sub(gs_mul(a0, c0), gs_mul(b, b)), 0.0f), det_safe));
  const float mid = gs_mul(0.5f, gs_add(a, c));  // :132-134
  const float lam1 = gs_add(mid, gs_sqrt(gs_maxf(gs_sub(gs_mul(mid, mid), det), 0.01f)));
  const float radius = std::ceil(gs_mul(3.0f, gs_sqrt(gs_maxf(lam1, 0.0f))));
  const bool valid = (z > cam.znear) && (det > 0.0f);  // :136-138
  *out_z = z;
  *out_r = valid ? radius : 0.0f;
  *out_comp = valid ? comp : 0.0f;
}

const float kC0 = (float)0.28209479177387814, kC1 = (float)0.4886025119029199;
const float kC2[5] = {(float)1.0925484305920792, (float)-1.0925484305920792, (float)0.31539156525252005,
                      (float)-1.0925484305920792, (float)0.5462742152960396};
const float kC3[7] = {(float)-0.5900435899266435, (float)2.890611442640554, (float)-0.4570457994644658,
                      (float)0.3731763325901154, (float)-0.4570457994644658, (float)1.445305721320277,
                      (float)-0.5900435899266435};

// sh.py:57-78, one (Gaussian, channel); sh[k * stride] is coefficient k.
float eval_sh_one(int degree, const float* sh, int stride, float x, float y, float z) {
  float r = gs_mul(kC0, sh[0]);
  if (degree > 0) {
    r = gs_sub(r, gs_mul(gs_mul(kC1, y), sh[1 * stride]));
    r = gs_add(r, gs_mul(gs_mul(kC1, z), sh[2 * stride]));
    r = gs_sub(r, gs_mul(gs_mul(kC1, x), sh[3 * stride]));
    if (degree > 1) {
      const float xx = gs_mul(x, x), yy = gs_mul(y, y), zz = gs_mul(z, z);
      const float xy = gs_mul(x, y), yz = gs_mul(y, z), xz = gs_mul(x, z);
      r = gs_add(r, gs_mul(gs_mul(kC2[0], xy), sh[4 * stride]));
      r = gs_add(r, gs_mul(gs_mul(kC2[1], yz), sh[5 * stride]));
      r = gs_add(r, gs_mul(gs_mul(kC2[2], gs_sub(gs_sub(gs_mul(2.0f, zz), xx), yy)), sh[6 * stride]));
      r = gs_add(r, gs_mul(gs_mul(kC2[3], xz), sh[7 * stride]));
      r = gs_add(r, gs_mul(gs_mul(kC2[4], gs_sub(xx, yy)), sh[8 * stride]));
      if (degree > 2) {
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[0], y), gs_sub(gs_mul(3.0f, xx), yy)), sh[9 * stride]));
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[1], xy), z), sh[10 * stride]));
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[2], y), gs_sub(gs_sub(gs_mul(4.0f, zz), xx), yy)), sh[11 * stride]));
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[3], z), gs_sub(gs_sub(gs_mul(2.0f, zz), gs_mul(3.0f, xx)), gs_mul(3.0f, yy))), sh[12 * stride]));
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[4], x), gs_sub(gs_sub(gs_mul(4.0f, zz), xx), yy)), sh[13 * stride]));
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[5], z), gs_sub(xx, yy)), sh[14 * stride]));
        r = gs_add(r, gs_mul(gs_mul(gs_mul(kC3[6], x), gs_sub(xx, gs_mul(3.0f, yy))), sh[15 * stride]));
      }
    }
  }
  return gs_add(r, 0.5f);
}

// tiles.py:54-65: inclusive tile bbox and count of one Gaussian.
int tile_bbox(float x, float y, float r, int W, int H, int tx, int ty, int* bb) {
  auto cl = [](float v, float hi) { return (int)gs_minf(gs_maxf(v, 0.0f), hi); };
  bb[0] = cl(std::floor(gs_div(gs_sub(x, r), (float)TILE)), (float)(tx - 1));
  bb[1] = cl(std::floor(gs_div(gs_add(x, r), (float)TILE)), (float)(tx - 1));
  bb[2] = cl(std::floor(gs_div(gs_sub(y, r), (float)TILE)), (float)(ty - 1));
  bb[3] = cl(std::floor(gs_div(gs_add(y, r), (float)TILE)), (float)(ty - 1));
  const bool on = (r > 0.0f) && (gs_add(x, r) >= 0.0f) && (gs_sub(x, r) < (float)W) &&
                  (gs_add(y, r) >= 0.0f) && (gs_sub(y, r) < (float)H);
  return on ? (bb[1] - bb[0] + 1) * (bb[3] - bb[2] + 1) : 0;
}

// tiles.py:96-141 for one duplicate: minimum of the conic form over the tile
// rectangle (corners, four clipped edge minimisers, 0 inside); keep if <= 12.
bool refine_keep(const float* co, float gx, float gy, int tile_x, int tile_y, int W, int H) {
  const float x0 = (float)(tile_x * TILE), y0 = (float)(tile_y * TILE);
  const float x1 = (float)std::min((tile_x + 1) * TILE, W), y1 = (float)std::min((tile_y + 1) * TILE, H);
  const float dx_min = gs_sub(x0, gx), dx_max = gs_sub(x1, gx);
  const float dy_min = gs_sub(y0, gy), dy_max = gs_sub(y1, gy);
  const float a = co[0], b = co[1], c = co[2];
  auto q = [&](float dx, float dy) {
    return gs_add(gs_add(gs_mul(gs_mul(a, dx), dx), gs_mul(gs_mul(gs_mul(2.0f, b), dx), dy)),
                  gs_mul(gs_mul(c, dy), dy));
  };
  auto clip = [](float v, float lo, float hi) { return gs_minf(gs_maxf(v, lo), hi); };
  const bool inside = dx_min <= 0 && dx_max >= 0 && dy_min <= 0 && dy_max >= 0;
  const float dy_at_left = clip(gs_mul(-gs_div(b, c), dx_min), dy_min, dy_max);
  const float dy_at_right = clip(gs_mul(-gs_div(b, c), dx_max), dy_min, dy_max);
  const float dx_at_bottom = clip(gs_mul(-gs_div(b, a), dy_min), dx_min, dx_max);
  const float dx_at_top = clip(gs_mul(-gs_div(b, a), dy_max), dx_min, dx_max);
  float qmin = q(dx_min, dy_min);
  qmin = gs_minf(qmin, q(dx_min, dy_max));
  qmin = gs_minf(qmin, q(dx_max, dy_min));
  qmin = gs_minf(qmin, q(dx_max, dy_max));
  qmin = gs_minf(qmin, q(dx_min, dy_at_left));
  qmin = gs_minf(qmin, q(dx_max, dy_at_right));
  qmin = gs_minf(qmin, q(dx_at_bottom, dy_min));
  qmin = gs_minf(qmin, q(dx_at_top, dy_max));
  return (inside ? 0.0f : qmin) <= 12.0f;
}

int n_threads(int requested) {
#ifdef _OPENMP
  return requested > 0 ? requested : omp_get_max_threads();
#else
  (void)requested;
  return 1;
#endif
}

}  // namespace

extern "C" {

// project_gaussians (projection.py:24-146).
void or_project(const gs_camera* cam, const float* means, const float* quats, const float* scales,
                int64_t n, float blur, int aa, float* means2d, float* conics, float* depths,
                float* radii, float* comp, int threads) {
#pragma omp parallel for schedule(static) num_threads(n_threads(threads))
  for (int64_t i = 0; i < n; ++i)
    project_one(*cam, means + 3 * i, quats + 4 * i, scales + 3 * i, blur, aa != 0, means2d + 2 * i,
                conics + 3 * i, depths + i, radii + i, comp + i);
}

// eval_sh (sh.py:41-78) for sh (N, K, C) and dirs (N, 3).
void or_eval_sh(int degree, const float* sh, int64_t n, int K, int C, const float* dirs, float* out) {
  for (int64_t i = 0; i < n; ++i)
    for (int ch = 0; ch < C; ++ch)
      out[i * C + ch] = eval_sh_one(degree, sh + i * K * C + ch, C, dirs[3 * i], dirs[3 * i + 1], dirs[3 * i + 2]);
}

// The SH colour step of render_gaussians (render.py:77-80): normalised view
// directions and max(eval_sh(...), 0) for sh (N, K, 3).
void or_sh_colors(const gs_camera* cam, int degree, const float* means, const float* sh, int64_t n,
                  int K, float* colors, int threads) {
#pragma omp parallel for schedule(static) num_threads(n_threads(threads))
  for (int64_t i = 0; i < n; ++i) {
    const float dx = gs_sub(means[3 * i], cam->center[0]);
    const float dy = gs_sub(means[3 * i + 1], cam->center[1]);
    const float dz = gs_sub(means[3 * i + 2], cam->center[2]);
    const float nr = gs_maxf(gs_sqrt(gs_add(gs_add(gs_mul(dx, dx), gs_mul(dy, dy)), gs_mul(dz, dz))), 1e-8f);
    const float x = gs_div(dx, nr), y = gs_div(dy, nr), z = gs_div(dz, nr);
    for (int ch = 0; ch < 3; ++ch)
      colors[3 * i + ch] = gs_maxf(eval_sh_one(degree, sh + i * K * 3 + ch, 3, x, y, z), 0.0f);
  }
}

// Activations of GaussianModel (model.py:116-122) with the shared exp.
void or_activate(const float* log_scales, const float* logits, int64_t n, float* scales, float* opac) {
  for (int64_t i = 0; i < 3 * n; ++i) scales[i] = gs_expf(log_scales[i]);
  for (int64_t i = 0; i < n; ++i) opac[i] = gs_sigmoidf(logits[i]);
}

// tiles.py:49-68 (and, with conics, the refinement's kept count
// tiles.py:141-143): tiles per Gaussian; returns the duplicate total D.
int64_t or_bin_count(const float* means2d, const float* radii, const float* conics, int64_t n, int W, int H,
                     int32_t* counts) {
  const int tx = (W + TILE - 1) / TILE, ty = (H + TILE - 1) / TILE;
  int64_t total = 0;
  int bb[4];
  for (int64_t i = 0; i < n; ++i) {
    const int c = tile_bbox(means2d[2 * i], means2d[2 * i + 1], radii[i], W, H, tx, ty, bb);
    int kept = c;
    if (conics && c) {
      kept = 0;
      for (int y = bb[2]; y <= bb[3]; ++y)
        for (int x = bb[0]; x <= bb[1]; ++x)
          kept += refine_keep(conics + 3 * i, means2d[2 * i], means2d[2 * i + 1], x, y, W, H);
    }
    counts[i] = kept;
    total += kept;
  }
  return total;
}

// tiles.py:77-182: duplicates in Gaussian order, key = tile * N + rank(depth)
// with rank from a stable argsort of all depths, stable argsort of the keys,
// per-tile [start, end) ranges with empty tiles at [0, 0).
void or_bin_fill(const float* means2d, const float* radii, const float* depths, const float* conics,
                 int64_t n, int W, int H, int64_t D, int32_t* sorted_ids, int32_t* ranges) {
  const int tx = (W + TILE - 1) / TILE, ty = (H + TILE - 1) / TILE;
  const int64_t num_tiles = (int64_t)tx * ty;
  std::vector<int32_t> gid, tid;
  gid.reserve(D);
  tid.reserve(D);
  int bb[4];
  for (int64_t i = 0; i < n; ++i) {
    const int c = tile_bbox(means2d[2 * i], means2d[2 * i + 1], radii[i], W, H, tx, ty, bb);
    if (!c) continue;
    const int w = bb[1] - bb[0] + 1;
    for (int l = 0; l < c; ++l) {  // :85-89, then the refinement's compaction :152-163
      const int x = bb[0] + l % w, y = bb[2] + l / w;
      if (conics && !refine_keep(conics + 3 * i, means2d[2 * i], means2d[2 * i + 1], x, y, W, H)) continue;
      gid.push_back((int32_t)i);
      tid.push_back(y * tx + x);
    }
  }
  std::vector<int64_t> order(n);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int64_t p, int64_t q) { return depths[p] < depths[q]; });
  std::vector<int64_t> rank(n);
  for (int64_t r = 0; r < n; ++r) rank[order[r]] = r;
  std::vector<int64_t> key(D);
  for (int64_t j = 0; j < D; ++j) key[j] = (int64_t)tid[j] * n + rank[gid[j]];
  std::vector<int64_t> idx(D);
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int64_t p, int64_t q) { return key[p] < key[q]; });
  std::vector<int32_t> starts(num_tiles, (int32_t)D), ends(num_tiles, 0);
  for (int64_t p = 0; p < D; ++p) {
    sorted_ids[p] = gid[idx[p]];
    const int32_t t = tid[idx[p]];
    starts[t] = std::min(starts[t], (int32_t)p);
    ends[t] = std::max(ends[t], (int32_t)(p + 1));
  }
  for (int64_t t = 0; t < num_tiles; ++t) {
    ranges[2 * t] = std::min(starts[t], ends[t]);
    ranges[2 * t + 1] = ends[t];
  }
}

// gs_rasterize_forward + gs_rasterize_depth (rasterize.py:28-98, 223-290) for
// C channels (C == 0: depth only); colors (N, C).
void or_rasterize_fwd(const float* means2d, const float* conics, const float* colors, int C,
                      const float* opac, const float* depths, const int32_t* ids,
                      const int32_t* ranges, const float* bg, int W, int H, float* image,
                      float* final_T, int32_t* n_contrib, float* depth, int threads, int64_t* stats) {
  // stats (optional): [0] pixel-Gaussian pairs evaluated (loop iterations up
  // to termination), [1] pairs composited.
  const int tx = (W + TILE - 1) / TILE, ty = (H + TILE - 1) / TILE;
  int64_t n_eval = 0, n_comp = 0;
#pragma omp parallel for schedule(dynamic, 4) num_threads(n_threads(threads)) reduction(+ : n_eval, n_comp)
  for (int tile = 0; tile < tx * ty; ++tile) {
    const int start = ranges[2 * tile], end = ranges[2 * tile + 1];
    std::vector<float> acc(C > 0 ? C : 1);
    for (int ly = 0; ly < TILE; ++ly)
      for (int lx = 0; lx < TILE; ++lx) {
        const int px = (tile % tx) * TILE + lx, py = (tile / tx) * TILE + ly;
        if (px >= W || py >= H) continue;
        const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
        float T = 1.0f, dacc = 0.0f;
        std::fill(acc.begin(), acc.end(), 0.0f);
        int last = 0;
        for (int k = start; k < end; ++k) {
          ++n_eval;
          const int g = ids[k];
          const float dx = gs_sub(means2d[2 * g], pxf), dy = gs_sub(means2d[2 * g + 1], pyf);
          const float* co = conics + 3 * g;
          const float power = gs_sub(gs_mul(-0.5f, gs_add(gs_mul(gs_mul(co[0], dx), dx), gs_mul(gs_mul(co[2], dy), dy))),
                                     gs_mul(gs_mul(co[1], dx), dy));
          if (power > 0.0f) continue;
          const float alpha = gs_minf(0.99f, gs_mul(opac[g], gs_expf(power)));
          if (alpha < 1.0f / 255.0f) continue;
          const float next_T = gs_mul(T, gs_sub(1.0f, alpha));
          if (next_T < 1e-4f) break;
          ++n_comp;
          const float w = gs_mul(alpha, T);
          for (int ch = 0; ch < C; ++ch) acc[ch] = gs_add(acc[ch], gs_mul(colors[(int64_t)g * C + ch], w));
          if (depth) dacc = gs_add(dacc, gs_mul(depths[g], w));
          T = next_T;
          last = k - start + 1;
        }
        const int64_t pid = (int64_t)py * W + px;
        for (int ch = 0; ch < C; ++ch) image[pid * C + ch] = gs_add(acc[ch], gs_mul(T, bg ? bg[ch] : 0.0f));
        final_T[pid] = T;
        if (n_contrib) n_contrib[pid] = last;
        if (depth) {
          const float al = gs_sub(1.0f, T);
          depth[pid] = al > 1e-6f ? gs_div(dacc, al) : 0.0f;
        }
      }
  }
  if (stats) {
    stats[0] = n_eval;
    stats[1] = n_comp;
  }
}

// gs_rasterize_backward (rasterize.py:100-221) for C channels; sequential
// per-pixel back-to-front replay, gradients summed per thread then reduced in
// thread order (deterministic for a fixed thread count).  Outputs are
// overwritten.
void or_rasterize_bwd(const float* means2d, const float* conics, const float* colors, int C,
                      const float* opac, int64_t n, const int32_t* ids, const int32_t* ranges,
                      const float* bg, int W, int H, const float* final_T, const int32_t* n_contrib,
                      const float* grad_image, const float* grad_final_T, float* g_means2d,
                      float* g_conics, float* g_colors, float* g_opac, int threads) {
  const int tx = (W + TILE - 1) / TILE, ty = (H + TILE - 1) / TILE;
  const int nt = n_threads(threads);
  const int64_t stride = 6 + C;
  std::vector<std::vector<float>> part(nt);
#pragma omp parallel num_threads(nt)
  {
#ifdef _OPENMP
    const int me = omp_get_thread_num();
#else
    const int me = 0;
#endif
    std::vector<float>& gp = part[me];
    gp.assign(n * stride, 0.0f);
    std::vector<float> dpix(C), accum(C), last_color(C);
#pragma omp for schedule(static)
    for (int tile = 0; tile < tx * ty; ++tile) {
      const int start = ranges[2 * tile], end = ranges[2 * tile + 1];
      for (int ly = 0; ly < TILE; ++ly)
        for (int lx = 0; lx < TILE; ++lx) {
          const int px = (tile % tx) * TILE + lx, py = (tile / tx) * TILE + ly;
          if (px >= W || py >= H) continue;
          const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
          const int64_t pid = (int64_t)py * W + px;
          const float T_final = final_T[pid];
          float T = T_final;
          const int last = n_contrib[pid];
          float bg_dot = 0.0f;
          for (int ch = 0; ch < C; ++ch) {
            dpix[ch] = grad_image[pid * C + ch];
            bg_dot += (bg ? bg[ch] : 0.0f) * dpix[ch];
          }
          if (grad_final_T) bg_dot += grad_final_T[pid];
          std::fill(accum.begin(), accum.end(), 0.0f);
          std::fill(last_color.begin(), last_color.end(), 0.0f);
          float last_alpha = 0.0f;
          for (int k = start + last - 1; k >= start; --k) {
            const int g = ids[k];
            const float dx = gs_sub(means2d[2 * g], pxf), dy = gs_sub(means2d[2 * g + 1], pyf);
            const float* co = conics + 3 * g;
            const float power = gs_sub(gs_mul(-0.5f, gs_add(gs_mul(gs_mul(co[0], dx), dx), gs_mul(gs_mul(co[2], dy), dy))),
                                       gs_mul(gs_mul(co[1], dx), dy));
            if (power > 0.0f) continue;
            const float G = gs_expf(power);
            const float alpha = gs_minf(0.99f, gs_mul(opac[g], G));
            if (alpha < 1.0f / 255.0f) continue;
            T = T / (1.0f - alpha);
            const float aT = alpha * T;
            float dL_dalpha = 0.0f;
            for (int ch = 0; ch < C; ++ch) {
              const float c = colors[(int64_t)g * C + ch];
              accum[ch] = last_alpha * last_color[ch] + (1.0f - last_alpha) * accum[ch];
              last_color[ch] = c;
              dL_dalpha += (c - accum[ch]) * dpix[ch];
            }
            last_alpha = alpha;
            dL_dalpha *= T;
            dL_dalpha += (-T_final / (1.0f - alpha)) * bg_dot;
            const float dL_dG = opac[g] * dL_dalpha;
            const float gdx = G * dx, gdy = G * dy;
            float* o = gp.data() + (int64_t)g * stride;
            o[0] += -(gdx * co[0] + gdy * co[1]) * dL_dG;
            o[1] += -(gdy * co[2] + gdx * co[1]) * dL_dG;
            o[2] += -0.5f * gdx * dx * dL_dG;
            o[3] += -gdx * dy * dL_dG;
            o[4] += -0.5f * gdy * dy * dL_dG;
            o[5] += G * dL_dalpha;
            for (int ch = 0; ch < C; ++ch) o[6 + ch] += aT * dpix[ch];
          }
        }
    }
  }
  for (int64_t g = 0; g < n; ++g) {
    float s[6] = {0, 0, 0, 0, 0, 0};
    for (int t = 0; t < nt; ++t)
      for (int k = 0; k < 6; ++k) s[k] += part[t][g * stride + k];
    g_means2d[2 * g] = s[0];
    g_means2d[2 * g + 1] = s[1];
    g_conics[3 * g] = s[2];
    g_conics[3 * g + 1] = s[3];
    g_conics[3 * g + 2] = s[4];
    g_opac[g] = s[5];
    for (int ch = 0; ch < C; ++ch) {
      float v = 0.0f;
      for (int t = 0; t < nt; ++t) v += part[t][g * stride + 6 + ch];
      g_colors[g * C + ch] = v;
    }
  }
}

// project_gaussians_ut (projection.py:149-205) with Camera.project_points
// (cameras.py:290-317; distortion :42-50, :68-76).  `lens` = {orthographic,
// fisheye, n_dist, dist[5]} as gs_lens.
static void ut_project_point(const gs_camera& c, const gs_lens& L, const float* P, float* uv) {
  float pc[3];
  for (int i = 0; i < 3; ++i)
    pc[i] = gs_add(gs_add(gs_add(gs_mul(P[0], c.R[3 * i]), gs_mul(P[1], c.R[3 * i + 1])), gs_mul(P[2], c.R[3 * i + 2])), c.t[i]);
  if (L.orthographic) {
    uv[0] = gs_add(gs_mul(c.fx, pc[0]), c.cx);
    uv[1] = gs_add(gs_mul(c.fy, pc[1]), c.cy);
    return;
  }
  const float inv = gs_div(1.0f, std::fabs(pc[2]) < 1e-8f ? 1e-8f : pc[2]);
  float x = gs_mul(pc[0], inv), y = gs_mul(pc[1], inv);
  if (L.n_dist > 0 && !L.fisheye) {
    const float k1 = L.dist[0], k2 = L.dist[1], p1 = L.dist[2], p2 = L.dist[3], k3 = L.dist[4];
    const float r2 = gs_add(gs_mul(x, x), gs_mul(y, y));
    const float radial = gs_add(1.0f, gs_mul(r2, gs_add(k1, gs_mul(r2, gs_add(k2, gs_mul(r2, k3))))));
    const float xd = gs_add(gs_add(gs_mul(x, radial), gs_mul(gs_mul(2.0f * p1, x), y)),
                            gs_mul(p2, gs_add(r2, gs_mul(gs_mul(2.0f, x), x))));
    const float yd = gs_add(gs_add(gs_mul(y, radial), gs_mul(p1, gs_add(r2, gs_mul(gs_mul(2.0f, y), y)))),
                            gs_mul(gs_mul(2.0f * p2, x), y));
    x = xd;
    y = yd;
  } else if (L.n_dist > 0) {
    const float k1 = L.dist[0], k2 = L.dist[1], k3 = L.dist[2], k4 = L.dist[3];
    const float r = gs_sqrt(gs_add(gs_mul(x, x), gs_mul(y, y)));
    const float th = std::atan(r), t2 = gs_mul(th, th);
    const float thd = gs_mul(th, gs_add(1.0f, gs_mul(t2, gs_add(k1, gs_mul(t2, gs_add(k2, gs_mul(t2, gs_add(k3, gs_mul(t2, k4)))))))));
    const float sc = gs_div(thd, gs_maxf(r, 1e-9f));
    x = gs_mul(x, sc);
    y = gs_mul(y, sc);
  }
  uv[0] = gs_add(gs_mul(c.fx, x), c.cx);
  uv[1] = gs_add(gs_mul(c.fy, y), c.cy);
}

void or_project_ut(const gs_camera* cam, const gs_lens* lens, const float* means, const float* quats,
                   const float* scales, int64_t n, float blur, int aa, float* means2d, float* conics,
                   float* depths, float* radii, float* comp) {
  const gs_camera& c = *cam;
  const float sq3 = gs_sqrt(3.0f), sixth = 1.0f / 6.0f;
  for (int64_t i = 0; i < n; ++i) {
    const float* q = quats + 4 * i;
    const float* m = means + 3 * i;
    const float nrm = gs_sqrt(gs_add(gs_add(gs_add(gs_mul(q[0], q[0]), gs_mul(q[1], q[1])), gs_mul(q[2], q[2])), gs_mul(q[3], q[3])));
    const float w = gs_div(q[0], nrm), x = gs_div(q[1], nrm), y = gs_div(q[2], nrm), z = gs_div(q[3], nrm);
    float R[3][3];  // transforms/rotations.py:30-49
    R[0][0] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(y, y), gs_mul(z, z))));
    R[0][1] = gs_mul(2.0f, gs_sub(gs_mul(x, y), gs_mul(w, z)));
    R[0][2] = gs_mul(2.0f, gs_add(gs_mul(x, z), gs_mul(w, y)));
    R[1][0] = gs_mul(2.0f, gs_add(gs_mul(x, y), gs_mul(w, z)));
    R[1][1] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(x, x), gs_mul(z, z))));
    R[1][2] = gs_mul(2.0f, gs_sub(gs_mul(y, z), gs_mul(w, x)));
    R[2][0] = gs_mul(2.0f, gs_sub(gs_mul(x, z), gs_mul(w, y)));
    R[2][1] = gs_mul(2.0f, gs_add(gs_mul(y, z), gs_mul(w, x)));
    R[2][2] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(x, x), gs_mul(y, y))));
    float uv[6][2];
    for (int j = 0; j < 6; ++j) {  // offsets: columns of R diag(s), then their negatives
      const int k = j % 3;
      float P[3];
      for (int r = 0; r < 3; ++r) {
        float off = gs_mul(R[r][k], scales[3 * i + k]);
        if (j >= 3) off = -off;
        P[r] = gs_add(m[r], gs_mul(sq3, off));
      }
      ut_project_point(c, *lens, P, uv[j]);
    }
    float su = uv[0][0], sv = uv[0][1];
    for (int j = 1; j < 6; ++j) { su = gs_add(su, uv[j][0]); sv = gs_add(sv, uv[j][1]); }
    const float mu = gs_mul(su, sixth), mv = gs_mul(sv, sixth);
    float sa = 0, sb = 0, sc = 0;
    for (int j = 0; j < 6; ++j) {
      const float dx = gs_sub(uv[j][0], mu), dy = gs_sub(uv[j][1], mv);
      sa = j ? gs_add(sa, gs_mul(dx, dx)) : gs_mul(dx, dx);
      sb = j ? gs_add(sb, gs_mul(dx, dy)) : gs_mul(dx, dy);
      sc = j ? gs_add(sc, gs_mul(dy, dy)) : gs_mul(dy, dy);
    }
    const float a0 = gs_mul(sa, sixth), b = gs_mul(sb, sixth), c0 = gs_mul(sc, sixth);
    const float a = gs_add(a0, blur), cc = gs_add(c0, blur);
    const float det = gs_sub(gs_mul(a, cc), gs_mul(b, b));
    const float ds = gs_maxf(det, 1e-12f);
    conics[3 * i] = gs_div(cc, ds);
    conics[3 * i + 1] = gs_div(-b, ds);
    conics[3 * i + 2] = gs_div(a, ds);
    float cp = 1.0f;
    if (aa && blur > 0.0f) cp = gs_sqrt(gs_div(gs_maxf(gs_sub(gs_mul(a0, c0), gs_mul(b, b)), 0.0f), ds));
    const float mid = gs_mul(0.5f, gs_add(a, cc));
    const float lam1 = gs_add(mid, gs_sqrt(gs_maxf(gs_sub(gs_mul(mid, mid), det), 0.01f)));
    const float rad = std::ceil(gs_mul(3.0f, gs_sqrt(gs_maxf(lam1, 0.0f))));
    const float zc = gs_add(gs_add(gs_add(gs_mul(m[0], c.R[6]), gs_mul(m[1], c.R[7])), gs_mul(m[2], c.R[8])), c.t[2]);
    const bool valid = zc > c.znear && det > 0.0f;
    means2d[2 * i] = mu;
    means2d[2 * i + 1] = mv;
    depths[i] = zc;
    radii[i] = valid ? rad : 0.0f;
    comp[i] = valid ? cp : 0.0f;
  }
}

// Hard z-buffer mesh rasterizer (src/mlx3d/renderer/rasterizer.py:29-79):
// per pixel of each tile, the tile's binned triangles in order; barycentrics
// by the reference's edge-function formula, skip |denom| < 1e-12, any
// l < -1e-5 or z <= znear; keep the strictly nearest (first on ties).
void or_mesh_rasterize(const float* tri_xy, const float* tri_z, const int32_t* ids, const int32_t* ranges,
                       int width, int height, float znear, int32_t* pix_to_face, float* zbuf) {
  const int tiles_x = (width + GS_TILE - 1) / GS_TILE, tiles_y = (height + GS_TILE - 1) / GS_TILE;
#pragma omp parallel for schedule(dynamic, 4)
  for (int tile = 0; tile < tiles_x * tiles_y; ++tile) {
    const int tx = tile % tiles_x, ty = tile / tiles_x;
    for (int ly = 0; ly < GS_TILE; ++ly)
      for (int lx = 0; lx < GS_TILE; ++lx) {
        const int px = tx * GS_TILE + lx, py = ty * GS_TILE + ly;
        if (px >= width || py >= height) continue;
        const float cx = (float)px + 0.5f, cy = (float)py + 0.5f;
        int best_f = -1;
        float best_z = 1e30f;
        for (int k = ranges[2 * tile]; k < ranges[2 * tile + 1]; ++k) {
          const int f = ids[k];
          const float* t = tri_xy + (int64_t)f * 6;
          const float ax = t[0], ay = t[1], bx = t[2], by = t[3], ccx = t[4], ccy = t[5];
          const float denom = (by - ccy) * (ax - ccx) + (ccx - bx) * (ay - ccy);
          if (fabsf(denom) < 1e-12f) continue;
          const float l0 = ((by - ccy) * (cx - ccx) + (ccx - bx) * (cy - ccy)) / denom;
          const float l1 = ((ccy - ay) * (cx - ccx) + (ax - ccx) * (cy - ccy)) / denom;
          const float l2 = 1.0f - l0 - l1;
          if (l0 < -1e-5f || l1 < -1e-5f || l2 < -1e-5f) continue;
          const float* z3 = tri_z + (int64_t)f * 3;
          const float z = l0 * z3[0] + l1 * z3[1] + l2 * z3[2];
          if (z <= znear) continue;
          if (z < best_z) {
            best_z = z;
            best_f = f;
          }
        }
        pix_to_face[(int64_t)py * width + px] = best_f;
        zbuf[(int64_t)py * width + px] = best_f >= 0 ? best_z : 0.0f;
      }
  }
}

// The shared exponential, exported so tests can check it against libm.
float or_expf(float x) { return gs_expf(x); }

// Number of floats x in [-87, 0] (and -0) where gs_expf_nonpos(x) differs
// bitwise from gs_expf(x): an exhaustive check of the compositors' exponential.
int64_t or_expf_nonpos_mismatches(void) {
  const int64_t lo = 0x80000000LL, hi = (int64_t)gs_float_to_bits(-87.0f);
  int64_t bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static)
  for (int64_t b = lo; b <= hi; ++b) {
    const float x = gs_bits_to_float((uint32_t)b);
    bad += gs_float_to_bits(gs_expf_nonpos(x)) != gs_float_to_bits(gs_expf(x));
  }
  // +0 as well
  bad += gs_float_to_bits(gs_expf_nonpos(0.0f)) != gs_float_to_bits(gs_expf(0.0f));
  return bad;
}

}  // extern "C"
