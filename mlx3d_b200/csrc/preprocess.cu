// Per-Gaussian kernels of the splatting path: EWA projection, SH colour,
// opacity compensation and tile counts (forward), and their vector-Jacobian
// products (backward).
//
// One thread per Gaussian; the wide per-Gaussian rows (SH coefficients,
// 12..192 B) are staged through shared memory with coalesced loads/stores.
// Everything a cut-off depends on (radii, tile bounds, counts) is evaluated
// with gs_math.h's exactly rounded primitives in the reference's operation
// order, so the result is bit-identical to the CPU oracle.
#include "gs_common.cuh"

namespace gs {

// Real SH constants (src/mlx3d/splatting/sh.py:7-25), rounded to float32 as
// MLX does when a Python float meets a float32 array.
#define SH_C0 ((float)0.28209479177387814)
#define SH_C1 ((float)0.4886025119029199)
#define SH_C2_0 ((float)1.0925484305920792)
#define SH_C2_1 ((float)-1.0925484305920792)
#define SH_C2_2 ((float)0.31539156525252005)
#define SH_C2_3 ((float)-1.0925484305920792)
#define SH_C2_4 ((float)0.5462742152960396)
#define SH_C3_0 ((float)-0.5900435899266435)
#define SH_C3_1 ((float)2.890611442640554)
#define SH_C3_2 ((float)-0.4570457994644658)
#define SH_C3_3 ((float)0.3731763325901154)
#define SH_C3_4 ((float)-0.4570457994644658)
#define SH_C3_5 ((float)1.445305721320277)
#define SH_C3_6 ((float)-0.5900435899266435)

// Basis values b_k with eval_sh(...) = sum_k b_k * sh_k + 0.5, each rounded
// exactly like the reference's sub-expression (sh.py:57-77); terms 1 and 3
// carry their minus sign (a - p*q == a + (-p)*q in IEEE arithmetic).
__device__ __forceinline__ int sh_basis(int degree, float x, float y, float z, float* b) {
  b[0] = SH_C0;
  if (degree < 1) return 1;
  b[1] = -gs_mul(SH_C1, y);
  b[2] = gs_mul(SH_C1, z);
  b[3] = -gs_mul(SH_C1, x);
  if (degree < 2) return 4;
  const float xx = gs_mul(x, x), yy = gs_mul(y, y), zz = gs_mul(z, z);
  const float xy = gs_mul(x, y), yz = gs_mul(y, z), xz = gs_mul(x, z);
  b[4] = gs_mul(SH_C2_0, xy);
  b[5] = gs_mul(SH_C2_1, yz);
  b[6] = gs_mul(SH_C2_2, gs_sub(gs_sub(gs_mul(2.0f, zz), xx), yy));
  b[7] = gs_mul(SH_C2_3, xz);
  b[8] = gs_mul(SH_C2_4, gs_sub(xx, yy));
  if (degree < 3) return 9;
  b[9] = gs_mul(gs_mul(SH_C3_0, y), gs_sub(gs_mul(3.0f, xx), yy));
  b[10] = gs_mul(gs_mul(SH_C3_1, xy), z);
  b[11] = gs_mul(gs_mul(SH_C3_2, y), gs_sub(gs_sub(gs_mul(4.0f, zz), xx), yy));
  b[12] = gs_mul(gs_mul(SH_C3_3, z), gs_sub(gs_sub(gs_mul(2.0f, zz), gs_mul(3.0f, xx)), gs_mul(3.0f, yy)));
  b[13] = gs_mul(gs_mul(SH_C3_4, x), gs_sub(gs_sub(gs_mul(4.0f, zz), xx), yy));
  b[14] = gs_mul(gs_mul(SH_C3_5, z), gs_sub(xx, yy));
  b[15] = gs_mul(gs_mul(SH_C3_6, x), gs_sub(xx, gs_mul(3.0f, yy)));
  return 16;
}

// d b_k / d(x, y, z) for the standalone eval_sh backward (dirs gradient).
__device__ __forceinline__ void sh_basis_grad(int degree, float x, float y, float z,
                                              float (*db)[3]) {
  for (int k = 0; k < 16; ++k) db[k][0] = db[k][1] = db[k][2] = 0.f;
  if (degree < 1) return;
  db[1][1] = -SH_C1;
  db[2][2] = SH_C1;
  db[3][0] = -SH_C1;
  if (degree < 2) return;
  const float xx = x * x, yy = y * y, zz = z * z;
  db[4][0] = SH_C2_0 * y;  db[4][1] = SH_C2_0 * x;
  db[5][1] = SH_C2_1 * z;  db[5][2] = SH_C2_1 * y;
  db[6][0] = -2.f * SH_C2_2 * x;  db[6][1] = -2.f * SH_C2_2 * y;  db[6][2] = 4.f * SH_C2_2 * z;
  db[7][0] = SH_C2_3 * z;  db[7][2] = SH_C2_3 * x;
  db[8][0] = 2.f * SH_C2_4 * x;  db[8][1] = -2.f * SH_C2_4 * y;
  if (degree < 3) return;
  db[9][0] = 6.f * SH_C3_0 * x * y;  db[9][1] = SH_C3_0 * (3.f * xx - 3.f * yy);
  db[10][0] = SH_C3_1 * y * z;  db[10][1] = SH_C3_1 * x * z;  db[10][2] = SH_C3_1 * x * y;
  db[11][0] = -2.f * SH_C3_2 * x * y;
  db[11][1] = SH_C3_2 * (4.f * zz - xx - 3.f * yy);
  db[11][2] = 8.f * SH_C3_2 * y * z;
  db[12][0] = -6.f * SH_C3_3 * x * z;
  db[12][1] = -6.f * SH_C3_3 * y * z;
  db[12][2] = SH_C3_3 * (6.f * zz - 3.f * xx - 3.f * yy);
  db[13][0] = SH_C3_4 * (4.f * zz - 3.f * xx - yy);
  db[13][1] = -2.f * SH_C3_4 * x * y;
  db[13][2] = 8.f * SH_C3_4 * x * z;
  db[14][0] = 2.f * SH_C3_5 * x * z;  db[14][1] = -2.f * SH_C3_5 * y * z;
  db[14][2] = SH_C3_5 * (xx - yy);
  db[15][0] = SH_C3_6 * (3.f * xx - 3.f * yy);  db[15][1] = -6.f * SH_C3_6 * x * y;
}

// View direction (means - camera_center) / max(|.|, 1e-8)  (render.py:77-78).
__device__ __forceinline__ void view_dir(const gs_camera& cam, float m0, float m1, float m2,
                                         float& x, float& y, float& z) {
  const float dx = gs_sub(m0, cam.center[0]);
  const float dy = gs_sub(m1, cam.center[1]);
  const float dz = gs_sub(m2, cam.center[2]);
  const float nrm = gs_sqrt(gs_add(gs_add(gs_mul(dx, dx), gs_mul(dy, dy)), gs_mul(dz, dz)));
  const float d = gs_maxf(nrm, 1e-8f);
  x = gs_div(dx, d);
  y = gs_div(dy, d);
  z = gs_div(dz, d);
}

// ---------------------------------------------------------------- projection
struct Proj {
  float u, v;           // means2d
  float ca, cb, cc;     // conic
  float z;              // depth
  float radius;
  float comp;
};

// Forward EWA projection of one Gaussian, operation by operation as
// src/mlx3d/splatting/projection.py:56-138 evaluates it.
__device__ __forceinline__ void project_one(const gs_camera& cam, float m0, float m1, float m2,
                                            float qw, float qx, float qy, float qz, float sx,
                                            float sy, float sz, float blur, bool aa, Proj& o) {
  const float* R = cam.R;
  const float x = gs_add(gs_add(gs_add(gs_mul(m0, R[0]), gs_mul(m1, R[1])), gs_mul(m2, R[2])), cam.t[0]);
  const float y = gs_add(gs_add(gs_add(gs_mul(m0, R[3]), gs_mul(m1, R[4])), gs_mul(m2, R[5])), cam.t[1]);
  const float z = gs_add(gs_add(gs_add(gs_mul(m0, R[6]), gs_mul(m1, R[7])), gs_mul(m2, R[8])), cam.t[2]);
  const float zs = gs_maxf(z, 1e-6f);
  o.u = gs_add(gs_div(gs_mul(cam.fx, x), zs), cam.cx);
  o.v = gs_add(gs_div(gs_mul(cam.fy, y), zs), cam.cy);
  const float tx = gs_mul(gs_minf(gs_maxf(gs_div(x, zs), -cam.clip_x), cam.clip_x), zs);
  const float ty = gs_mul(gs_minf(gs_maxf(gs_div(y, zs), -cam.clip_y), cam.clip_y), zs);
  const float iz = gs_div(1.0f, zs);
  const float iz2 = gs_mul(iz, iz);
  const float j00 = gs_mul(cam.fx, iz);
  const float j02 = gs_mul(gs_mul(cam.neg_fx, tx), iz2);
  const float j11 = gs_mul(cam.fy, iz);
  const float j12 = gs_mul(gs_mul(cam.neg_fy, ty), iz2);
  const float t00 = gs_add(gs_mul(j00, R[0]), gs_mul(j02, R[6]));
  const float t01 = gs_add(gs_mul(j00, R[1]), gs_mul(j02, R[7]));
  const float t02 = gs_add(gs_mul(j00, R[2]), gs_mul(j02, R[8]));
  const float t10 = gs_add(gs_mul(j11, R[3]), gs_mul(j12, R[6]));
  const float t11 = gs_add(gs_mul(j11, R[4]), gs_mul(j12, R[7]));
  const float t12 = gs_add(gs_mul(j11, R[5]), gs_mul(j12, R[8]));
  // q / |q|  (projection.py:94)
  const float qn = gs_sqrt(gs_add(gs_add(gs_add(gs_mul(qw, qw), gs_mul(qx, qx)), gs_mul(qy, qy)), gs_mul(qz, qz)));
  const float w = gs_div(qw, qn), a = gs_div(qx, qn), b = gs_div(qy, qn), c = gs_div(qz, qn);
  const float r00 = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(b, b), gs_mul(c, c))));
  const float r01 = gs_mul(2.0f, gs_sub(gs_mul(a, b), gs_mul(w, c)));
  const float r02 = gs_mul(2.0f, gs_add(gs_mul(a, c), gs_mul(w, b)));
  const float r10 = gs_mul(2.0f, gs_add(gs_mul(a, b), gs_mul(w, c)));
  const float r11 = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(a, a), gs_mul(c, c))));
  const float r12 = gs_mul(2.0f, gs_sub(gs_mul(b, c), gs_mul(w, a)));
  const float r20 = gs_mul(2.0f, gs_sub(gs_mul(a, c), gs_mul(w, b)));
  const float r21 = gs_mul(2.0f, gs_add(gs_mul(b, c), gs_mul(w, a)));
  const float r22 = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(a, a), gs_mul(b, b))));
  const float m00 = gs_mul(gs_add(gs_add(gs_mul(t00, r00), gs_mul(t01, r10)), gs_mul(t02, r20)), sx);
  const float m01 = gs_mul(gs_add(gs_add(gs_mul(t00, r01), gs_mul(t01, r11)), gs_mul(t02, r21)), sy);
  const float m02 = gs_mul(gs_add(gs_add(gs_mul(t00, r02), gs_mul(t01, r12)), gs_mul(t02, r22)), sz);
  const float m10 = gs_mul(gs_add(gs_add(gs_mul(t10, r00), gs_mul(t11, r10)), gs_mul(t12, r20)), sx);
  const float m11 = gs_mul(gs_add(gs_add(gs_mul(t10, r01), gs_mul(t11, r11)), gs_mul(t12, r21)), sy);
  const float m12 = gs_mul(gs_add(gs_add(gs_mul(t10, r02), gs_mul(t11, r12)), gs_mul(t12, r22)), sz);
  const float a0 = gs_add(gs_add(gs_mul(m00, m00), gs_mul(m01, m01)), gs_mul(m02, m02));
  const float bb = gs_add(gs_add(gs_mul(m00, m10), gs_mul(m01, m11)), gs_mul(m02, m12));
  const float c0 = gs_add(gs_add(gs_mul(m10, m10), gs_mul(m11, m11)), gs_mul(m12, m12));
  const float ca = gs_add(a0, blur);
  const float cc = gs_add(c0, blur);
  const float det = gs_sub(gs_mul(ca, cc), gs_mul(bb, bb));
  const float ds = gs_maxf(det, 1e-12f);
  o.ca = gs_div(cc, ds);
  o.cb = gs_div(-bb, ds);
  o.cc = gs_div(ca, ds);
  float comp = 1.0f;
  if (aa) {
    const float det0 = gs_maxf(gs_sub(gs_mul(a0, c0), gs_mul(bb, bb)), 0.0f);
    comp = gs_sqrt(gs_div(det0, ds));
  }
  const float mid = gs_mul(0.5f, gs_add(ca, cc));
  const float lam1 = gs_add(mid, gs_sqrt(gs_maxf(gs_sub(gs_mul(mid, mid), det), 0.01f)));
  const float radius = ceilf(gs_mul(3.0f, gs_sqrt(gs_maxf(lam1, 0.0f))));
  const bool valid = (z > cam.znear) && (det > 0.0f);
  o.z = z;
  o.radius = valid ? radius : 0.0f;
  o.comp = valid ? comp : 0.0f;
}

// Inclusive tile rectangle and count of one Gaussian (tiles.py:54-65).
__device__ __forceinline__ int tile_rect(float u, float v, float r, int width, int height,
                                         int tiles_x, int tiles_y, int& x0, int& y0, int& x1,
                                         int& y1) {
  const float fx1 = (float)(tiles_x - 1), fy1 = (float)(tiles_y - 1);
  const float T = (float)GS_TILE;
  x0 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_sub(u, r), T)), 0.0f), fx1);
  x1 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_add(u, r), T)), 0.0f), fx1);
  y0 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_sub(v, r), T)), 0.0f), fy1);
  y1 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_add(v, r), T)), 0.0f), fy1);
  const bool on = (r > 0.0f) && (gs_add(u, r) >= 0.0f) && (gs_sub(u, r) < (float)width) &&
                  (gs_add(v, r) >= 0.0f) && (gs_sub(v, r) < (float)height);
  return on ? (x1 - x0 + 1) * (y1 - y0 + 1) : 0;
}

// ------------------------------------------------------------ forward kernel
struct PreFwdArgs {
  gs_camera cam;
  const float *means, *quats, *scales, *opac;
  const float *sh_dc, *sh_rest;
  int64_t dc_stride, rest_stride;
  int sh_degree;  // -1: no colour
  int64_t n;
  float blur;
  int aa;
  int flags;
  int fused;  // 1: opacity, colour and tile counts too
  float *means2d, *conics, *depths, *radii, *comp, *colors, *opac_out;
  int32_t* tiles_touched;
  int tiles_x, tiles_y;
};

constexpr int kPreBlock = 128;

__device__ unsigned long long g_wait_failures;

// Staging of one block's parameter rows (means, scales, and the SH rows when
// given).  Every row block that is contiguous, 16-byte aligned and a whole
// number of 16-byte units is fetched with one bulk copy (cp.async.bulk,
// issued by thread 0, completion on a shared-memory mbarrier); the others
// with 16-byte cp.async or scalar loads by all threads (stage_rows).  The
// decisions are block-uniform.  wait() completes both and synchronises the
// block; false (for every thread) if the bulk copies did not complete within
// the bounded wait, which is counted in g_wait_failures.
struct StagePlan {
  bool b_means, b_scales, b_dc, b_rest, want_dc, want_rest;
  unsigned tx;
  __device__ StagePlan(const float* g_means, const float* g_scales, const float* g_dc, int64_t dc_stride,
                       const float* g_rest, int64_t rest_stride, int rest_len, int rows) {
    want_dc = g_dc != nullptr;
    want_rest = g_rest != nullptr && rest_len > 0;
    b_means = rows_bulk(g_means, 3, 3, rows);
    b_scales = rows_bulk(g_scales, 3, 3, rows);
    b_dc = want_dc && rows_bulk(g_dc, dc_stride, 3, rows);
    b_rest = want_rest && rows_bulk(g_rest, rest_stride, rest_len, rows);
    tx = (b_means ? rows * 12u : 0u) + (b_scales ? rows * 12u : 0u) + (b_dc ? rows * 12u : 0u) +
         (b_rest ? (unsigned)rows * (unsigned)rest_len * 4u : 0u);
  }
  __device__ void issue(unsigned long long* bar, float* s_means, const float* g_means, float* s_scales,
                        const float* g_scales, float* s_dc, const float* g_dc, int64_t dc_stride, float* s_rest,
                        const float* g_rest, int64_t rest_stride, int rest_len, int rows) const {
    if (tx) {
      if (threadIdx.x == 0) mbar_init(bar, 1);
      __syncthreads();
      if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar, tx);
        if (b_means) bulk_g2s(s_means, g_means, rows * 12u, bar);
        if (b_scales) bulk_g2s(s_scales, g_scales, rows * 12u, bar);
        if (b_dc) bulk_g2s(s_dc, g_dc, rows * 12u, bar);
        if (b_rest) bulk_g2s(s_rest, g_rest, (unsigned)rows * (unsigned)rest_len * 4u, bar);
      }
    }
    if (!b_means) stage_rows<kPreBlock>(s_means, g_means, 3, 3, rows);
    if (!b_scales) stage_rows<kPreBlock>(s_scales, g_scales, 3, 3, rows);
    if (want_dc && !b_dc) stage_rows<kPreBlock>(s_dc, g_dc, dc_stride, 3, rows);
    if (want_rest && !b_rest) stage_rows<kPreBlock>(s_rest, g_rest, rest_stride, rest_len, rows);
  }
  // Failure path: a CTA must not exit while a bulk copy still writes into
  // its shared memory (what happens then is undefined).  So after the
  // bounded wait gives up, thread 0 waits once more (bounded again) before
  // the block leaves; if even that wait runs out, the block still leaves
  // (there is no safe alternative that keeps the wait bounded) and the
  // failure is counted, so the host can treat the launch's outputs as
  // invalid.  The barrier is single-use and dies with the CTA.
  __device__ bool wait(unsigned long long* bar) const {
    cp_async_wait_all();
    const bool ok = tx == 0 || mbar_wait(bar, 0);
    if (__syncthreads_and(ok)) return true;
    if (threadIdx.x == 0) {
      atomicAdd(&g_wait_failures, 1ull);
      (void)mbar_wait(bar, 0);
    }
    __syncthreads();
    return false;
  }
};


__global__ void __launch_bounds__(kPreBlock) k_preprocess_fwd(const PreFwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int64_t base = (int64_t)blockIdx.x * kPreBlock;
  const int rows = (int)min((int64_t)kPreBlock, a.n - base);
  const int nb = a.sh_degree >= 0 ? (a.sh_degree + 1) * (a.sh_degree + 1) : 0;
  const int rest_len = nb > 1 ? (nb - 1) * 3 : 0;
  const float* g_means = a.means + base * 3;
  const float* g_scales = a.scales + base * 3;
  const float* g_dc = a.sh_dc ? a.sh_dc + base * a.dc_stride : nullptr;
  const float* g_rest = a.sh_rest ? a.sh_rest + base * a.rest_stride : nullptr;
  const int mld = stage_pitch(g_means, 3, 3), sld = stage_pitch(g_scales, 3, 3);
  const int dld = g_dc ? stage_pitch(g_dc, a.dc_stride, 3) : 3;
  const int rest_ld = rest_len ? stage_pitch(g_rest, a.rest_stride, rest_len) : 1;
  float* s_means = smem;                       // pitch <= 4
  float* s_scales = s_means + kPreBlock * 4;   // pitch <= 4
  float* s_dc = s_scales + kPreBlock * 4;      // pitch <= 4
  float* s_rest = s_dc + kPreBlock * 4;        // pitch <= rest_len | 1
  __shared__ unsigned long long s_bar;
  const bool want_sh = a.fused && nb > 0;
  const StagePlan plan(g_means, g_scales, want_sh ? g_dc : nullptr, a.dc_stride,
                       want_sh && rest_len > 0 ? g_rest : nullptr, a.rest_stride, rest_len, rows);
  plan.issue(&s_bar, s_means, g_means, s_scales, g_scales, s_dc, g_dc, a.dc_stride, s_rest, g_rest, a.rest_stride,
             rest_len, rows);
  // This thread's own rows (quaternion, opacity) load while the staged
  // block lands.
  const int li = threadIdx.x;
  const int64_t i = base + li;
  float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
  float o_raw = 0.0f;
  if (li < rows) {
    q = __ldg(reinterpret_cast<const float4*>(a.quats) + i);
    if (a.fused) o_raw = __ldg(a.opac + i);
  }
  if (!plan.wait(&s_bar)) return;
  if (li >= rows) return;
  float s0 = s_scales[li * sld + 0], s1 = s_scales[li * sld + 1], s2 = s_scales[li * sld + 2];
  if (a.flags & GS_ACT_EXP_SCALES) {
    s0 = gs_expf(s0);
    s1 = gs_expf(s1);
    s2 = gs_expf(s2);
  }
  const float m0 = s_means[li * mld + 0], m1 = s_means[li * mld + 1], m2 = s_means[li * mld + 2];
  Proj p;
  project_one(a.cam, m0, m1, m2, q.x, q.y, q.z, q.w, s0, s1, s2, a.blur, a.aa != 0, p);
  reinterpret_cast<float2*>(a.means2d)[i] = make_float2(p.u, p.v);
  a.conics[i * 3 + 0] = p.ca;
  a.conics[i * 3 + 1] = p.cb;
  a.conics[i * 3 + 2] = p.cc;
  a.depths[i] = p.z;
  a.radii[i] = p.radius;
  a.comp[i] = p.comp;
  if (!a.fused) return;
  float o = o_raw;
  if (a.flags & GS_ACT_SIGMOID_OPACITY) o = gs_sigmoidf(o);
  a.opac_out[i] = gs_mul(o, p.comp);
  int x0, y0, x1, y1;
  a.tiles_touched[i] = tile_rect(p.u, p.v, p.radius, a.cam.width, a.cam.height, a.tiles_x,
                                 a.tiles_y, x0, y0, x1, y1);
  if (nb > 0) {
    float dx, dy, dz;
    view_dir(a.cam, m0, m1, m2, dx, dy, dz);
    float bs[16];
    sh_basis(a.sh_degree, dx, dy, dz, bs);
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      float r = gs_mul(bs[0], s_dc[li * dld + ch]);
      for (int k = 1; k < nb; ++k) r = gs_add(r, gs_mul(bs[k], s_rest[li * rest_ld + (k - 1) * 3 + ch]));
      r = gs_add(r, 0.5f);
      a.colors[i * 3 + ch] = gs_maxf(r, 0.0f);
    }
  }
}

// ----------------------------------------------------------- backward kernel
struct PreBwdArgs {
  PreFwdArgs f;
  const float *g_means2d, *g_conics, *g_colors, *g_opac_out, *g_depths, *g_comp;
  float *g_means, *g_quats, *g_scales, *g_opac, *g_sh_dc, *g_sh_rest;
};

// VJP of project_one (MLX autodiff conventions: maximum/minimum pass the
// gradient to the first argument only where it is strictly larger/smaller,
// so clip() passes it strictly inside the bounds; where() masks it).
__device__ __forceinline__ void project_vjp(const gs_camera& cam, float m0, float m1, float m2,
                                            float qw_, float qx_, float qy_, float qz_, float sx,
                                            float sy, float sz, float blur, bool aa, float gu,
                                            float gv, float gA, float gB, float gC, float gz_out,
                                            float gcomp, float* gm, float* gq, float* gs) {
  const float* R = cam.R;
  const float x = m0 * R[0] + m1 * R[1] + m2 * R[2] + cam.t[0];
  const float y = m0 * R[3] + m1 * R[4] + m2 * R[5] + cam.t[1];
  const float z = gs_add(gs_add(gs_add(gs_mul(m0, R[6]), gs_mul(m1, R[7])), gs_mul(m2, R[8])), cam.t[2]);
  const float zs = fmaxf(z, 1e-6f);
  const float iz = 1.0f / zs;
  const float iz2 = iz * iz;
  const float txr = x * iz, tyr = y * iz;
  const float txc = fminf(fmaxf(txr, -cam.clip_x), cam.clip_x);
  const float tyc = fminf(fmaxf(tyr, -cam.clip_y), cam.clip_y);
  const float tx = txc * zs, ty = tyc * zs;
  const float j00 = cam.fx * iz, j02 = cam.neg_fx * tx * iz2;
  const float j11 = cam.fy * iz, j12 = cam.neg_fy * ty * iz2;
  const float T0[3] = {j00 * R[0] + j02 * R[6], j00 * R[1] + j02 * R[7], j00 * R[2] + j02 * R[8]};
  const float T1[3] = {j11 * R[3] + j12 * R[6], j11 * R[4] + j12 * R[7], j11 * R[5] + j12 * R[8]};
  const float qn = sqrtf(qw_ * qw_ + qx_ * qx_ + qy_ * qy_ + qz_ * qz_);
  const float iqn = 1.0f / qn;
  const float w = qw_ * iqn, a = qx_ * iqn, b = qy_ * iqn, c = qz_ * iqn;
  float Rq[3][3] = {{1.f - 2.f * (b * b + c * c), 2.f * (a * b - w * c), 2.f * (a * c + w * b)},
                    {2.f * (a * b + w * c), 1.f - 2.f * (a * a + c * c), 2.f * (b * c - w * a)},
                    {2.f * (a * c - w * b), 2.f * (b * c + w * a), 1.f - 2.f * (a * a + b * b)}};
  const float s[3] = {sx, sy, sz};
  float d0[3], d1[3], M0[3], M1[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    d0[k] = T0[0] * Rq[0][k] + T0[1] * Rq[1][k] + T0[2] * Rq[2][k];
    d1[k] = T1[0] * Rq[0][k] + T1[1] * Rq[1][k] + T1[2] * Rq[2][k];
    M0[k] = d0[k] * s[k];
    M1[k] = d1[k] * s[k];
  }
  const float a0 = M0[0] * M0[0] + M0[1] * M0[1] + M0[2] * M0[2];
  const float bb = M0[0] * M1[0] + M0[1] * M1[1] + M0[2] * M1[2];
  const float c0 = M1[0] * M1[0] + M1[1] * M1[1] + M1[2] * M1[2];
  const float ca = a0 + blur, cc = c0 + blur;
  const float det = ca * cc - bb * bb;
  const float ds = fmaxf(det, 1e-12f);
  const float ids = 1.0f / ds;
  const bool valid = (z > cam.znear) && (det > 0.0f);

  // conic = (c, -b, a) / ds
  float g_ca = gC * ids, g_cc = gA * ids, g_b = -gB * ids;
  float g_ds = -(gA * cc - gB * bb + gC * ca) * ids * ids;
  float g_a0 = 0.f, g_c0 = 0.f;
  if (aa && valid && gcomp != 0.0f) {
    const float det0r = a0 * c0 - bb * bb;
    const float det0 = fmaxf(det0r, 0.0f);
    const float qv = det0 * ids;
    const float comp = sqrtf(qv);
    // sqrt'(0) is unbounded; the gradient is taken as 0 there.
    const float g_q = comp > 0.0f ? gcomp * 0.5f / comp : 0.0f;
    g_ds -= g_q * qv * ids;
    if (det0r > 0.0f) {
      const float g_det0 = g_q * ids;
      g_a0 += g_det0 * c0;
      g_c0 += g_det0 * a0;
      g_b -= 2.0f * bb * g_det0;
    }
  }
  const float g_det = det > 1e-12f ? g_ds : 0.0f;
  g_ca += g_det * cc;
  g_cc += g_det * ca;
  g_b -= 2.0f * bb * g_det;
  g_a0 += g_ca;
  g_c0 += g_cc;
  float gT0[3] = {0.f, 0.f, 0.f}, gT1[3] = {0.f, 0.f, 0.f};
  float gR[3][3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float gM0 = 2.0f * M0[k] * g_a0 + M1[k] * g_b;
    const float gM1 = 2.0f * M1[k] * g_c0 + M0[k] * g_b;
    gs[k] = gM0 * d0[k] + gM1 * d1[k];
    const float gd0 = gM0 * s[k], gd1 = gM1 * s[k];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      gT0[i] += gd0 * Rq[i][k];
      gT1[i] += gd1 * Rq[i][k];
      gR[i][k] = gd0 * T0[i] + gd1 * T1[i];
    }
  }
  const float g_j00 = gT0[0] * R[0] + gT0[1] * R[1] + gT0[2] * R[2];
  const float g_j02 = gT0[0] * R[6] + gT0[1] * R[7] + gT0[2] * R[8];
  const float g_j11 = gT1[0] * R[3] + gT1[1] * R[4] + gT1[2] * R[5];
  const float g_j12 = gT1[0] * R[6] + gT1[1] * R[7] + gT1[2] * R[8];
  float g_iz = cam.fx * g_j00 + cam.fy * g_j11;
  const float g_iz2 = cam.neg_fx * tx * g_j02 + cam.neg_fy * ty * g_j12;
  const float g_tx = cam.neg_fx * iz2 * g_j02;
  const float g_ty = cam.neg_fy * iz2 * g_j12;
  g_iz += 2.0f * iz * g_iz2;
  float g_zs = -iz * iz * g_iz;
  g_zs += g_tx * txc + g_ty * tyc;
  const float g_txr = (txr > -cam.clip_x && txr < cam.clip_x) ? g_tx * zs : 0.0f;
  const float g_tyr = (tyr > -cam.clip_y && tyr < cam.clip_y) ? g_ty * zs : 0.0f;
  float g_x = g_txr * iz + gu * cam.fx * iz;
  float g_y = g_tyr * iz + gv * cam.fy * iz;
  g_zs -= (g_txr * txr + g_tyr * tyr) * iz;
  g_zs -= (gu * cam.fx * x + gv * cam.fy * y) * iz * iz;
  const float g_z = (z > 1e-6f ? g_zs : 0.0f) + gz_out;
  gm[0] = g_x * R[0] + g_y * R[3] + g_z * R[6];
  gm[1] = g_x * R[1] + g_y * R[4] + g_z * R[7];
  gm[2] = g_x * R[2] + g_y * R[5] + g_z * R[8];
  // Rotation matrix of a unit quaternion -> gradient of (w, a, b, c).
  const float gw = 2.f * (-c * gR[0][1] + b * gR[0][2] + c * gR[1][0] - a * gR[1][2] - b * gR[2][0] + a * gR[2][1]);
  const float ga = 2.f * (b * gR[0][1] + c * gR[0][2] + b * gR[1][0] - 2.f * a * gR[1][1] - w * gR[1][2] +
                          c * gR[2][0] + w * gR[2][1] - 2.f * a * gR[2][2]);
  const float gb = 2.f * (-2.f * b * gR[0][0] + a * gR[0][1] + w * gR[0][2] + a * gR[1][0] + c * gR[1][2] -
                          w * gR[2][0] + c * gR[2][1] - 2.f * b * gR[2][2]);
  const float gc = 2.f * (-2.f * c * gR[0][0] - w * gR[0][1] + a * gR[0][2] + w * gR[1][0] - 2.f * c * gR[1][1] +
                          b * gR[1][2] + a * gR[2][0] + b * gR[2][1]);
  // Normalisation q / |q|.
  const float dot = w * gw + a * ga + b * gb + c * gc;
  gq[0] = (gw - w * dot) * iqn;
  gq[1] = (ga - a * dot) * iqn;
  gq[2] = (gb - b * dot) * iqn;
  gq[3] = (gc - c * dot) * iqn;
}

__global__ void __launch_bounds__(kPreBlock) k_preprocess_bwd(const PreBwdArgs g) {
  extern __shared__ __align__(16) float smem[];
  const PreFwdArgs& a = g.f;
  const int64_t base = (int64_t)blockIdx.x * kPreBlock;
  const int rows = (int)min((int64_t)kPreBlock, a.n - base);
  const int nb = a.sh_degree >= 0 ? (a.sh_degree + 1) * (a.sh_degree + 1) : 0;
  const int rest_len = nb > 1 ? (nb - 1) * 3 : 0;
  const bool sh = a.fused && nb > 0;
  const float* g_means = a.means + base * 3;
  const float* g_scales = a.scales + base * 3;
  const float* g_dc = sh ? a.sh_dc + base * a.dc_stride : nullptr;
  const float* g_rest = (sh && rest_len) ? a.sh_rest + base * a.rest_stride : nullptr;
  const int mld = stage_pitch(g_means, 3, 3), sld = stage_pitch(g_scales, 3, 3);
  const int dld = g_dc ? stage_pitch(g_dc, a.dc_stride, 3) : 3;
  const int rest_ld = g_rest ? stage_pitch(g_rest, a.rest_stride, rest_len) : 1;
  float* s_means = smem;
  float* s_scales = s_means + kPreBlock * 4;
  float* s_dc = s_scales + kPreBlock * 4;      // sh_dc rows, then their gradients
  float* s_rest = s_dc + kPreBlock * 4;        // sh_rest rows, then their gradients
  __shared__ unsigned long long s_bar;
  const StagePlan plan(g_means, g_scales, sh ? g_dc : nullptr, a.dc_stride, g_rest, a.rest_stride, rest_len, rows);
  plan.issue(&s_bar, s_means, g_means, s_scales, g_scales, s_dc, g_dc, a.dc_stride, s_rest, g_rest, a.rest_stride,
             rest_len, rows);
  // This thread's own rows (quaternion, cotangents, opacity) load while
  // the staged block lands.
  const int li = threadIdx.x;
  const int64_t i = base + li;
  float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
  float gu = 0.f, gv = 0.f, gA = 0.f, gB = 0.f, gC = 0.f, gz = 0.f, gcomp = 0.f, o_raw = 0.f, goo = 0.f;
  if (li < rows) {
    q = __ldg(reinterpret_cast<const float4*>(a.quats) + i);
    if (g.g_means2d) { gu = g.g_means2d[2 * i]; gv = g.g_means2d[2 * i + 1]; }
    if (g.g_conics) { gA = g.g_conics[3 * i]; gB = g.g_conics[3 * i + 1]; gC = g.g_conics[3 * i + 2]; }
    if (g.g_depths) gz = g.g_depths[i];
    if (g.g_comp) gcomp = g.g_comp[i];
    if (a.fused) {
      o_raw = __ldg(a.opac + i);
      if (g.g_opac_out) goo = g.g_opac_out[i];
    }
  }
  if (!plan.wait(&s_bar)) return;
  if (li < rows) {
    const float r0 = s_scales[li * sld + 0], r1 = s_scales[li * sld + 1], r2 = s_scales[li * sld + 2];
    float s0 = r0, s1 = r1, s2 = r2;
    if (a.flags & GS_ACT_EXP_SCALES) {
      s0 = gs_expf(r0);
      s1 = gs_expf(r1);
      s2 = gs_expf(r2);
    }
    const float m0 = s_means[li * mld + 0], m1 = s_means[li * mld + 1], m2 = s_means[li * mld + 2];
    if (a.fused) {
      // opacities_out = act(opacity) * compensation   (render.py:75)
      float o = o_raw;
      if (a.flags & GS_ACT_SIGMOID_OPACITY) o = gs_sigmoidf(o_raw);
      // Compensation of this Gaussian (forward value needed for d/d opacity).
      Proj p;
      project_one(a.cam, m0, m1, m2, q.x, q.y, q.z, q.w, s0, s1, s2, a.blur, a.aa != 0, p);
      float go = goo * p.comp;
      gcomp += goo * o;
      if (a.flags & GS_ACT_SIGMOID_OPACITY) go = go * o * (1.0f - o);
      g.g_opac[i] = go;
    }
    float gm[3], gq[4], gsc[3];
    project_vjp(a.cam, m0, m1, m2, q.x, q.y, q.z, q.w, s0, s1, s2, a.blur, a.aa != 0, gu, gv,
                gA, gB, gC, gz, gcomp, gm, gq, gsc);
    if (a.flags & GS_ACT_EXP_SCALES) {
      gsc[0] *= s0;
      gsc[1] *= s1;
      gsc[2] *= s2;
    }
    g.g_means[3 * i + 0] = gm[0];
    g.g_means[3 * i + 1] = gm[1];
    g.g_means[3 * i + 2] = gm[2];
    reinterpret_cast<float4*>(g.g_quats)[i] = make_float4(gq[0], gq[1], gq[2], gq[3]);
    g.g_scales[3 * i + 0] = gsc[0];
    g.g_scales[3 * i + 1] = gsc[1];
    g.g_scales[3 * i + 2] = gsc[2];
    if (sh) {
      // colors = max(eval_sh(...), 0): recompute the raw value to mask the
      // gradient, then overwrite the staged coefficients with their gradients
      // (each channel's coefficients are read before they are overwritten).
      float dx, dy, dz;
      view_dir(a.cam, m0, m1, m2, dx, dy, dz);
      float bs[16];
      sh_basis(a.sh_degree, dx, dy, dz, bs);
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        float r = gs_mul(bs[0], s_dc[li * dld + ch]);
        for (int k = 1; k < nb; ++k) r = gs_add(r, gs_mul(bs[k], s_rest[li * rest_ld + (k - 1) * 3 + ch]));
        r = gs_add(r, 0.5f);
        const float gcol = r > 0.0f ? g.g_colors[3 * i + ch] : 0.0f;
        s_dc[li * dld + ch] = bs[0] * gcol;
        for (int k = 1; k < nb; ++k) s_rest[li * rest_ld + (k - 1) * 3 + ch] = bs[k] * gcol;
      }
    }
  }
  if (sh) {
    __syncthreads();
    unstage_rows<kPreBlock>(g.g_sh_dc + base * a.dc_stride, a.dc_stride, s_dc, dld, 3, rows);
    if (rest_len > 0)
      unstage_rows<kPreBlock>(g.g_sh_rest + base * a.rest_stride, a.rest_stride, s_rest, rest_ld,
                              rest_len, rows);
  }
}

// ------------------------------------------------- view-batched backward
// The VJP of gs_preprocess_forward summed over several views of the same
// Gaussians: gradient = sum over views v of VJP_v(cotangents_v).  Used when
// the views' screen-space cotangents (9 floats per Gaussian and view:
// means2d 2, conic 3, colour 3, effective opacity 1) have been gathered on
// one device, e.g. a rank that owns a slice of the Gaussians after an
// all-to-all of every rank's cotangents for that slice.  One thread per
// Gaussian walks the views: the parameter rows are read once, each view's
// projection is recomputed (as the single-view backward does), and the SH
// coefficient gradients sum in shared memory (48 floats per row, odd pitch).
constexpr int kViewsGradPitch = 49;

struct PreBwdViewsArgs {
  PreFwdArgs f;                // cam unused
  const gs_camera* cams;       // device array of n_views cameras
  int n_views;
  const float* g_screen;       // packed: view v, Gaussian i at g_screen + v * view_stride + 9 i
  int64_t view_stride;
  const float* const* cot;     // or per view v: cot[4 v + 0..3] = dL/d means2d (2), conic (3),
                               // colour (3), effective opacity (1) arrays of Gaussian 0 of the slice
  float *g_means, *g_quats, *g_scales, *g_opac, *g_sh_dc, *g_sh_rest;
};

template <bool PTRS>
__global__ void __launch_bounds__(kPreBlock) k_preprocess_bwd_views(const PreBwdViewsArgs g) {
  extern __shared__ __align__(16) float smem[];
  const PreFwdArgs& a = g.f;
  const int64_t base = (int64_t)blockIdx.x * kPreBlock;
  const int rows = (int)min((int64_t)kPreBlock, a.n - base);
  const int nb = a.sh_degree >= 0 ? (a.sh_degree + 1) * (a.sh_degree + 1) : 0;
  const int rest_len = nb > 1 ? (nb - 1) * 3 : 0;
  const bool sh = nb > 0;
  const float* g_means = a.means + base * 3;
  const float* g_scales = a.scales + base * 3;
  const float* g_dc = sh ? a.sh_dc + base * a.dc_stride : nullptr;
  const float* g_rest = (sh && rest_len) ? a.sh_rest + base * a.rest_stride : nullptr;
  const int mld = stage_pitch(g_means, 3, 3), sld = stage_pitch(g_scales, 3, 3);
  const int dld = g_dc ? stage_pitch(g_dc, a.dc_stride, 3) : 3;
  const int rest_ld = g_rest ? stage_pitch(g_rest, a.rest_stride, rest_len) : 1;
  float* s_means = smem;
  float* s_scales = s_means + kPreBlock * 4;
  float* s_dc = s_scales + kPreBlock * 4;
  float* s_rest = s_dc + kPreBlock * 4;
  float* s_g = s_rest + kPreBlock * (rest_len | 1);  // SH gradient rows: dc 3, rest 45
  __shared__ unsigned long long s_bar;
  const StagePlan plan(g_means, g_scales, g_dc, a.dc_stride, g_rest, a.rest_stride, rest_len, rows);
  plan.issue(&s_bar, s_means, g_means, s_scales, g_scales, s_dc, g_dc, a.dc_stride, s_rest, g_rest, a.rest_stride,
             rest_len, rows);
  const int li = threadIdx.x;
  const int64_t i = base + li;
  float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
  float o_raw = 0.f;
  if (li < rows) {
    q = __ldg(reinterpret_cast<const float4*>(a.quats) + i);
    o_raw = __ldg(a.opac + i);
  }
  if (sh)
    for (int k = 0; k < kViewsGradPitch; ++k) s_g[li * kViewsGradPitch + k] = 0.0f;
  if (!plan.wait(&s_bar)) return;
  if (li < rows) {
    const float r0 = s_scales[li * sld + 0], r1 = s_scales[li * sld + 1], r2 = s_scales[li * sld + 2];
    float s0 = r0, s1 = r1, s2 = r2;
    if (a.flags & GS_ACT_EXP_SCALES) {
      s0 = gs_expf(r0);
      s1 = gs_expf(r1);
      s2 = gs_expf(r2);
    }
    const float m0 = s_means[li * mld + 0], m1 = s_means[li * mld + 1], m2 = s_means[li * mld + 2];
    float o = o_raw;
    if (a.flags & GS_ACT_SIGMOID_OPACITY) o = gs_sigmoidf(o_raw);
    float gm[3] = {0.f, 0.f, 0.f}, gq[4] = {0.f, 0.f, 0.f, 0.f}, gsc[3] = {0.f, 0.f, 0.f}, go = 0.f;
    for (int v = 0; v < g.n_views; ++v) {
      const gs_camera& cam = g.cams[v];
      float gu, gv, gA, gB, gC, gcv[3], goo;
      if (PTRS) {
        // cotangents of view v: possibly another GPU's memory (peer loads)
        const float* const* t = g.cot + 4 * v;
        const float* pm = t[0] + 2 * (int64_t)i;
        const float* pc = t[1] + 3 * (int64_t)i;
        const float* pk = t[2] + 3 * (int64_t)i;
        gu = pm[0]; gv = pm[1];
        gA = pc[0]; gB = pc[1]; gC = pc[2];
        gcv[0] = pk[0]; gcv[1] = pk[1]; gcv[2] = pk[2];
        goo = t[3][i];
      } else {
        const float* cot = g.g_screen + v * g.view_stride + 9 * (int64_t)i;
        gu = __ldg(cot + 0); gv = __ldg(cot + 1);
        gA = __ldg(cot + 2); gB = __ldg(cot + 3); gC = __ldg(cot + 4);
        gcv[0] = __ldg(cot + 5); gcv[1] = __ldg(cot + 6); gcv[2] = __ldg(cot + 7);
        goo = __ldg(cot + 8);
      }
      // opacities_out = act(opacity) * compensation   (render.py:75)
      Proj p;
      project_one(cam, m0, m1, m2, q.x, q.y, q.z, q.w, s0, s1, s2, a.blur, a.aa != 0, p);
      go += goo * p.comp;
      float gmv[3], gqv[4], gsv[3];
      project_vjp(cam, m0, m1, m2, q.x, q.y, q.z, q.w, s0, s1, s2, a.blur, a.aa != 0, gu, gv, gA, gB, gC, 0.0f,
                  goo * o, gmv, gqv, gsv);
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        gm[k] += gmv[k];
        gsc[k] += gsv[k];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) gq[k] += gqv[k];
      if (sh) {
        float dx, dy, dz;
        view_dir(cam, m0, m1, m2, dx, dy, dz);
        float bs[16];
        sh_basis(a.sh_degree, dx, dy, dz, bs);
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
          float r = gs_mul(bs[0], s_dc[li * dld + ch]);
          for (int k = 1; k < nb; ++k) r = gs_add(r, gs_mul(bs[k], s_rest[li * rest_ld + (k - 1) * 3 + ch]));
          r = gs_add(r, 0.5f);
          const float gcol = r > 0.0f ? gcv[ch] : 0.0f;
          s_g[li * kViewsGradPitch + ch] += bs[0] * gcol;
          for (int k = 1; k < nb; ++k) s_g[li * kViewsGradPitch + 3 + (k - 1) * 3 + ch] += bs[k] * gcol;
        }
      }
    }
    if (a.flags & GS_ACT_SIGMOID_OPACITY) go = go * o * (1.0f - o);
    if (a.flags & GS_ACT_EXP_SCALES) {
      gsc[0] *= s0;
      gsc[1] *= s1;
      gsc[2] *= s2;
    }
    g.g_opac[i] = go;
    g.g_means[3 * i + 0] = gm[0];
    g.g_means[3 * i + 1] = gm[1];
    g.g_means[3 * i + 2] = gm[2];
    reinterpret_cast<float4*>(g.g_quats)[i] = make_float4(gq[0], gq[1], gq[2], gq[3]);
    g.g_scales[3 * i + 0] = gsc[0];
    g.g_scales[3 * i + 1] = gsc[1];
    g.g_scales[3 * i + 2] = gsc[2];
  }
  if (sh) {
    __syncthreads();
    unstage_rows<kPreBlock>(g.g_sh_dc + base * a.dc_stride, a.dc_stride, s_g, kViewsGradPitch, 3, rows);
    if (rest_len > 0)
      unstage_rows<kPreBlock>(g.g_sh_rest + base * a.rest_stride, a.rest_stride, s_g + 3, kViewsGradPitch,
                              rest_len, rows);
  }
}

// ------------------------------------------------------------ eval_sh kernels
// Standalone eval_sh (N, K, C) with explicit directions; one thread per
// (Gaussian, channel) pair.
__global__ void k_eval_sh_fwd(int degree, const float* __restrict__ sh, int64_t n, int K, int C,
                              const float* __restrict__ dirs, float* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * C) return;
  const int64_t i = t / C;
  const int ch = (int)(t - i * C);
  float bs[16];
  const int nb = sh_basis(degree, dirs[3 * i], dirs[3 * i + 1], dirs[3 * i + 2], bs);
  const float* row = sh + i * K * C;
  float r = gs_mul(bs[0], row[ch]);
  for (int k = 1; k < nb; ++k) r = gs_add(r, gs_mul(bs[k], row[k * C + ch]));
  out[t] = gs_add(r, 0.5f);
}

__global__ void k_eval_sh_bwd(int degree, const float* __restrict__ sh, int64_t n, int K, int C,
                              const float* __restrict__ dirs, const float* __restrict__ g_out,
                              float* __restrict__ g_sh, float* __restrict__ g_dirs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = dirs[3 * i], y = dirs[3 * i + 1], z = dirs[3 * i + 2];
  float bs[16];
  const int nb = sh_basis(degree, x, y, z, bs);
  const float* row = sh + i * K * C;
  float* grow = g_sh + i * K * C;
  for (int k = 0; k < K; ++k)
    for (int ch = 0; ch < C; ++ch) grow[k * C + ch] = k < nb ? bs[k] * g_out[i * C + ch] : 0.0f;
  if (g_dirs) {
    float db[16][3];
    sh_basis_grad(degree, x, y, z, db);
    float gx = 0.f, gy = 0.f, gz = 0.f;
    for (int k = 1; k < nb; ++k) {
      float s = 0.f;
      for (int ch = 0; ch < C; ++ch) s += g_out[i * C + ch] * row[k * C + ch];
      gx += s * db[k][0];
      gy += s * db[k][1];
      gz += s * db[k][2];
    }
    g_dirs[3 * i] = gx;
    g_dirs[3 * i + 1] = gy;
    g_dirs[3 * i + 2] = gz;
  }
}

// Standalone tile counts (tiles.py:49-65) for bin_gaussians called with
// caller-provided means2d / radii.
__global__ void k_tile_counts(const float* __restrict__ means2d, const float* __restrict__ radii,
                              int64_t n, int width, int height, int tiles_x, int tiles_y,
                              int32_t* __restrict__ counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float2 m = reinterpret_cast<const float2*>(means2d)[i];
  int x0, y0, x1, y1;
  counts[i] = tile_rect(m.x, m.y, radii[i], width, height, tiles_x, tiles_y, x0, y0, x1, y1);
}

static size_t pre_smem_bytes(int sh_degree, bool fused) {
  const int nb = (fused && sh_degree >= 0) ? (sh_degree + 1) * (sh_degree + 1) : 0;
  const int rest_len = nb > 1 ? (nb - 1) * 3 : 0;
  return sizeof(float) * (size_t)kPreBlock * (4 + 4 + 4 + (rest_len | 1));
}

static int check_cam(const gs_camera* cam) {
  if (!cam) return set_error(GS_ERR_INVALID_ARG, "camera is NULL");
  if (cam->width <= 0 || cam->height <= 0)
    return set_error(GS_ERR_INVALID_ARG, "camera size must be positive (got %dx%d)", cam->width,
                     cam->height);
  return GS_OK;
}

int preprocess_wait_failures(unsigned long long* out, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_wait_failures, sizeof(*out));
  if (e == cudaSuccess && reset) {
    const unsigned long long z = 0;
    e = cudaMemcpyToSymbol(g_wait_failures, &z, sizeof(z));
  }
  return (int)e;
}

}  // namespace gs

using namespace gs;

extern "C" {

int gs_project_forward(const gs_camera* cam, const float* means, const float* quats,
                       const float* scales, int64_t n, float blur, int antialias, float* means2d,
                       float* conics, float* depths, float* radii, float* compensation,
                       void* stream) {
  clear_error();
  if (int e = check_cam(cam)) return e;
  if (n < 0) return set_error(GS_ERR_INVALID_ARG, "n must be >= 0");
  if (n == 0) return GS_OK;
  if (!means || !quats || !scales || !means2d || !conics || !depths || !radii || !compensation)
    return set_error(GS_ERR_INVALID_ARG, "gs_project_forward: NULL pointer");
  if (!aligned(quats, 16)) return set_error(GS_ERR_INVALID_ARG, "quats must be 16-byte aligned");
  PreFwdArgs a{};
  a.cam = *cam;
  a.means = means; a.quats = quats; a.scales = scales;
  a.sh_degree = -1; a.n = n; a.blur = blur; a.aa = antialias && blur > 0.0f; a.flags = 0; a.fused = 0;
  a.means2d = means2d; a.conics = conics; a.depths = depths; a.radii = radii; a.comp = compensation;
  const size_t sm = pre_smem_bytes(-1, false);
  k_preprocess_fwd<<<(unsigned)ceil_div(n, kPreBlock), kPreBlock, sm, as_stream(stream)>>>(a);
  return check_launch("k_preprocess_fwd");
}

int gs_project_backward(const gs_camera* cam, const float* means, const float* quats,
                        const float* scales, int64_t n, float blur, int antialias,
                        const float* g_means2d, const float* g_conics, const float* g_depths,
                        const float* g_compensation, float* g_means, float* g_quats,
                        float* g_scales, void* stream) {
  clear_error();
  if (int e = check_cam(cam)) return e;
  if (n < 0) return set_error(GS_ERR_INVALID_ARG, "n must be >= 0");
  if (n == 0) return GS_OK;
  if (!means || !quats || !scales || !g_means || !g_quats || !g_scales)
    return set_error(GS_ERR_INVALID_ARG, "gs_project_backward: NULL pointer");
  if (!aligned(quats, 16) || !aligned(g_quats, 16))
    return set_error(GS_ERR_INVALID_ARG, "quats / g_quats must be 16-byte aligned");
  PreBwdArgs g{};
  PreFwdArgs& a = g.f;
  a.cam = *cam;
  a.means = means; a.quats = quats; a.scales = scales;
  a.sh_degree = -1; a.n = n; a.blur = blur; a.aa = antialias && blur > 0.0f; a.flags = 0; a.fused = 0;
  g.g_means2d = g_means2d; g.g_conics = g_conics; g.g_depths = g_depths; g.g_comp = g_compensation;
  g.g_means = g_means; g.g_quats = g_quats; g.g_scales = g_scales;
  const size_t sm = pre_smem_bytes(-1, false);
  k_preprocess_bwd<<<(unsigned)ceil_div(n, kPreBlock), kPreBlock, sm, as_stream(stream)>>>(g);
  return check_launch("k_preprocess_bwd");
}

int gs_preprocess_forward(const gs_camera* cam, const float* means, const float* quats,
                          const float* scales, const float* opacities, const float* sh_dc,
                          int64_t sh_dc_stride, const float* sh_rest, int64_t sh_rest_stride,
                          int sh_degree, int64_t n, float blur, int antialias, int flags,
                          float* means2d, float* conics, float* depths, float* radii,
                          float* compensation, float* colors, float* opacities_out,
                          int32_t* tiles_touched, void* stream) {
  clear_error();
  if (int e = check_cam(cam)) return e;
  if (n < 0) return set_error(GS_ERR_INVALID_ARG, "n must be >= 0");
  if (n == 0) return GS_OK;
  if (!means || !quats || !scales || !opacities || !means2d || !conics || !depths || !radii ||
      !compensation || !opacities_out || !tiles_touched)
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_forward: NULL pointer");
  if (!aligned(quats, 16)) return set_error(GS_ERR_INVALID_ARG, "quats must be 16-byte aligned");
  const int deg = sh_dc ? sh_degree : -1;
  if (sh_dc && (sh_degree < 0 || sh_degree > 3))
    return set_error(GS_ERR_INVALID_ARG, "sh_degree must be in [0, 3] (got %d)", sh_degree);
  if (sh_dc && sh_degree > 0 && !sh_rest)
    return set_error(GS_ERR_INVALID_ARG, "sh_rest is NULL but sh_degree > 0");
  if (sh_dc && !colors) return set_error(GS_ERR_INVALID_ARG, "colors output is NULL");
  PreFwdArgs a{};
  a.cam = *cam;
  a.means = means; a.quats = quats; a.scales = scales; a.opac = opacities;
  a.sh_dc = sh_dc; a.sh_rest = sh_rest; a.dc_stride = sh_dc_stride; a.rest_stride = sh_rest_stride;
  a.sh_degree = deg; a.n = n; a.blur = blur; a.aa = antialias && blur > 0.0f; a.flags = flags; a.fused = 1;
  a.means2d = means2d; a.conics = conics; a.depths = depths; a.radii = radii; a.comp = compensation;
  a.colors = colors; a.opac_out = opacities_out; a.tiles_touched = tiles_touched;
  a.tiles_x = (int)ceil_div(cam->width, GS_TILE);
  a.tiles_y = (int)ceil_div(cam->height, GS_TILE);
  const size_t sm = pre_smem_bytes(deg, true);
  k_preprocess_fwd<<<(unsigned)ceil_div(n, kPreBlock), kPreBlock, sm, as_stream(stream)>>>(a);
  return check_launch("k_preprocess_fwd");
}

int gs_preprocess_backward(const gs_camera* cam, const float* means, const float* quats,
                           const float* scales, const float* opacities, const float* sh_dc,
                           int64_t sh_dc_stride, const float* sh_rest, int64_t sh_rest_stride,
                           int sh_degree, int64_t n, float blur, int antialias, int flags,
                           const float* g_means2d, const float* g_conics, const float* g_colors,
                           const float* g_opacities_out, const float* g_depths,
                           const float* g_compensation, float* g_means, float* g_quats,
                           float* g_scales, float* g_opacities, float* g_sh_dc,
                           float* g_sh_rest, void* stream) {
  clear_error();
  if (int e = check_cam(cam)) return e;
  if (n < 0) return set_error(GS_ERR_INVALID_ARG, "n must be >= 0");
  if (n == 0) return GS_OK;
  if (!means || !quats || !scales || !opacities || !g_means || !g_quats || !g_scales ||
      !g_opacities)
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_backward: NULL pointer");
  if (!aligned(quats, 16) || !aligned(g_quats, 16))
    return set_error(GS_ERR_INVALID_ARG, "quats / g_quats must be 16-byte aligned");
  const int deg = sh_dc ? sh_degree : -1;
  if (sh_dc && (sh_degree < 0 || sh_degree > 3))
    return set_error(GS_ERR_INVALID_ARG, "sh_degree must be in [0, 3] (got %d)", sh_degree);
  if (sh_dc && (!g_colors || !g_sh_dc || (sh_degree > 0 && (!sh_rest || !g_sh_rest))))
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_backward: NULL SH pointer");
  PreBwdArgs g{};
  PreFwdArgs& a = g.f;
  a.cam = *cam;
  a.means = means; a.quats = quats; a.scales = scales; a.opac = opacities;
  a.sh_dc = sh_dc; a.sh_rest = sh_rest; a.dc_stride = sh_dc_stride; a.rest_stride = sh_rest_stride;
  a.sh_degree = deg; a.n = n; a.blur = blur; a.aa = antialias && blur > 0.0f; a.flags = flags; a.fused = 1;
  g.g_means2d = g_means2d; g.g_conics = g_conics; g.g_colors = g_colors;
  g.g_opac_out = g_opacities_out; g.g_depths = g_depths; g.g_comp = g_compensation;
  g.g_means = g_means; g.g_quats = g_quats; g.g_scales = g_scales; g.g_opac = g_opacities;
  g.g_sh_dc = g_sh_dc; g.g_sh_rest = g_sh_rest;
  const size_t sm = pre_smem_bytes(deg, true);
  k_preprocess_bwd<<<(unsigned)ceil_div(n, kPreBlock), kPreBlock, sm, as_stream(stream)>>>(g);
  return check_launch("k_preprocess_bwd");
}

static int views_bwd_impl(const gs_camera* cams, int n_views, const float* means, const float* quats,
                          const float* scales, const float* opacities, const float* sh_dc, int64_t sh_dc_stride,
                          const float* sh_rest, int64_t sh_rest_stride, int sh_degree, int64_t n, float blur,
                          int antialias, int flags, const float* g_screen, int64_t view_stride,
                          const float* const* cot, float* g_means, float* g_quats, float* g_scales,
                          float* g_opacities, float* g_sh_dc, float* g_sh_rest, void* stream) {
  if (n < 0) return set_error(GS_ERR_INVALID_ARG, "n must be >= 0");
  if (n_views < 0) return set_error(GS_ERR_INVALID_ARG, "n_views must be >= 0");
  if (n == 0) return GS_OK;
  if (!cams && n_views > 0) return set_error(GS_ERR_INVALID_ARG, "cams is NULL");
  if (!means || !quats || !scales || !opacities || !g_means || !g_quats || !g_scales || !g_opacities ||
      (n_views > 0 && !g_screen && !cot))
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_backward_views: NULL pointer");
  if (!cot && view_stride < 9 * n && n_views > 1)
    return set_error(GS_ERR_INVALID_ARG, "view_stride %lld is below 9 n = %lld", (long long)view_stride,
                     (long long)(9 * n));
  if (!aligned(quats, 16) || !aligned(g_quats, 16))
    return set_error(GS_ERR_INVALID_ARG, "quats / g_quats must be 16-byte aligned");
  const int deg = sh_dc ? sh_degree : -1;
  if (sh_dc && (sh_degree < 0 || sh_degree > 3))
    return set_error(GS_ERR_INVALID_ARG, "sh_degree must be in [0, 3] (got %d)", sh_degree);
  if (sh_dc && (!g_sh_dc || (sh_degree > 0 && (!sh_rest || !g_sh_rest))))
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_backward_views: NULL SH pointer");
  PreBwdViewsArgs g{};
  PreFwdArgs& a = g.f;
  a.means = means; a.quats = quats; a.scales = scales; a.opac = opacities;
  a.sh_dc = sh_dc; a.sh_rest = sh_rest; a.dc_stride = sh_dc_stride; a.rest_stride = sh_rest_stride;
  a.sh_degree = deg; a.n = n; a.blur = blur; a.aa = antialias && blur > 0.0f; a.flags = flags; a.fused = 1;
  g.cams = cams; g.n_views = n_views; g.g_screen = g_screen; g.view_stride = view_stride; g.cot = cot;
  g.g_means = g_means; g.g_quats = g_quats; g.g_scales = g_scales; g.g_opac = g_opacities;
  g.g_sh_dc = g_sh_dc; g.g_sh_rest = g_sh_rest;
  const size_t sm = pre_smem_bytes(deg, true) + (deg >= 0 ? sizeof(float) * kPreBlock * kViewsGradPitch : 0);
  auto kern = cot ? k_preprocess_bwd_views<true> : k_preprocess_bwd_views<false>;
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return set_error(GS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  kern<<<(unsigned)ceil_div(n, kPreBlock), kPreBlock, sm, as_stream(stream)>>>(g);
  return check_launch("k_preprocess_bwd_views");
}

int gs_preprocess_backward_views(const gs_camera* cams, int n_views, const float* means,
                                 const float* quats, const float* scales, const float* opacities,
                                 const float* sh_dc, int64_t sh_dc_stride, const float* sh_rest,
                                 int64_t sh_rest_stride, int sh_degree, int64_t n, float blur, int antialias,
                                 int flags, const float* g_screen, int64_t view_stride, float* g_means,
                                 float* g_quats, float* g_scales, float* g_opacities, float* g_sh_dc,
                                 float* g_sh_rest, void* stream) {
  clear_error();
  if (!g_screen && n_views > 0 && n > 0)
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_backward_views: g_screen is NULL");
  return views_bwd_impl(cams, n_views, means, quats, scales, opacities, sh_dc, sh_dc_stride, sh_rest,
                        sh_rest_stride, sh_degree, n, blur, antialias, flags, g_screen, view_stride, nullptr,
                        g_means, g_quats, g_scales, g_opacities, g_sh_dc, g_sh_rest, stream);
}

int gs_preprocess_backward_views_peer(const gs_camera* cams, int n_views, const float* means,
                                      const float* quats, const float* scales, const float* opacities,
                                      const float* sh_dc, int64_t sh_dc_stride, const float* sh_rest,
                                      int64_t sh_rest_stride, int sh_degree, int64_t n, float blur,
                                      int antialias, int flags, const float* const* cotangents, float* g_means,
                                      float* g_quats, float* g_scales, float* g_opacities, float* g_sh_dc,
                                      float* g_sh_rest, void* stream) {
  clear_error();
  if (!cotangents && n_views > 0 && n > 0)
    return set_error(GS_ERR_INVALID_ARG, "gs_preprocess_backward_views_peer: cotangents is NULL");
  return views_bwd_impl(cams, n_views, means, quats, scales, opacities, sh_dc, sh_dc_stride, sh_rest,
                        sh_rest_stride, sh_degree, n, blur, antialias, flags, nullptr, 0, cotangents, g_means,
                        g_quats, g_scales, g_opacities, g_sh_dc, g_sh_rest, stream);
}

int gs_eval_sh_forward(int degree, const float* sh, int64_t n, int k, int channels,
                       const float* dirs, float* out, void* stream) {
  clear_error();
  if (degree < 0 || degree > 3) return set_error(GS_ERR_INVALID_ARG, "degree must be in [0, 3]");
  if (k < (degree + 1) * (degree + 1))
    return set_error(GS_ERR_INVALID_ARG, "sh has %d coefficients, degree %d needs %d", k, degree,
                     (degree + 1) * (degree + 1));
  if (channels <= 0) return set_error(GS_ERR_INVALID_ARG, "channels must be positive");
  if (n <= 0) return GS_OK;
  const int64_t total = n * channels;
  k_eval_sh_fwd<<<(unsigned)ceil_div(total, 256), 256, 0, as_stream(stream)>>>(degree, sh, n, k,
                                                                            channels, dirs, out);
  return check_launch("k_eval_sh_fwd");
}

int gs_eval_sh_backward(int degree, const float* sh, int64_t n, int k, int channels,
                        const float* dirs, const float* g_out, float* g_sh, float* g_dirs,
                        void* stream) {
  clear_error();
  if (degree < 0 || degree > 3) return set_error(GS_ERR_INVALID_ARG, "degree must be in [0, 3]");
  if (k < (degree + 1) * (degree + 1))
    return set_error(GS_ERR_INVALID_ARG, "sh has too few coefficients for degree %d", degree);
  if (channels <= 0) return set_error(GS_ERR_INVALID_ARG, "channels must be positive");
  if (n <= 0) return GS_OK;
  k_eval_sh_bwd<<<(unsigned)ceil_div(n, 128), 128, 0, as_stream(stream)>>>(
      degree, sh, n, k, channels, dirs, g_out, g_sh, g_dirs);
  return check_launch("k_eval_sh_bwd");
}

int gs_tile_counts(const float* means2d, const float* radii, int64_t n, int width, int height,
                   int32_t* tiles_touched, void* stream) {
  clear_error();
  if (width <= 0 || height <= 0) return set_error(GS_ERR_INVALID_ARG, "image size must be positive");
  if (n <= 0) return GS_OK;
  if (!aligned(means2d, 8)) return set_error(GS_ERR_INVALID_ARG, "means2d must be 8-byte aligned");
  const int tx = (int)ceil_div(width, GS_TILE), ty = (int)ceil_div(height, GS_TILE);
  k_tile_counts<<<(unsigned)ceil_div(n, 256), 256, 0, as_stream(stream)>>>(means2d, radii, n, width,
                                                                         height, tx, ty, tiles_touched);
  return check_launch("k_tile_counts");
}

}  // extern "C"
