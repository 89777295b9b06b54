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
// test; it only avoids evaluating the exponential.  The floor is at least
// -87 (o e^-87 < 1/255 for every o <= 1), which keeps the arguments that
// reach the exponential inside gs_expf_nonpos's domain.
__device__ __forceinline__ float power_floor(float o) {
  return o > 0.0f ? fmaxf(-logf(255.0f * o) - 1e-3f, -87.0f) : INFINITY;
}

// Conservative pixel-space box (xmin, xmax, ymin, ymax) around every pixel
// centre where power >= pf can hold, i.e. the ellipse
// A dx^2 + 2 B dx dy + C dy^2 <= 2 L with L = -pf: half extents
// sqrt(2 L C / det) and sqrt(2 L A / det).  The box is widened by 2 % + 1 px,
// far beyond the float32 evaluation error of power near the ellipse, so a
// warp whose pixels all lie outside it can skip the Gaussian: every one of
// its pixels would fail the exact power >= pf test anyway.  A Gaussian that
// can never reach alpha >= 1/255 gets an empty box; a degenerate conic an
// unbounded one.
__device__ __forceinline__ float4 cull_box(float2 m, float4 co, float pf) {
  const float L = -pf;
  if (!(L > 0.0f)) return make_float4(INFINITY, -INFINITY, INFINITY, -INFINITY);
  const float det = co.x * co.z - co.y * co.y;
  if (!(det > 0.0f) || !(co.x > 0.0f) || !(co.z > 0.0f))
    return make_float4(-INFINITY, INFINITY, -INFINITY, INFINITY);
  const float hx = sqrtf(2.0f * L * co.z / det) * 1.02f + 1.0f;
  const float hy = sqrtf(2.0f * L * co.x / det) * 1.02f + 1.0f;
  return make_float4(m.x - hx, m.x + hx, m.y - hy, m.y + hy);
}

// Pixel layout shared by both compositors: 128 threads per 16x16 tile, warp
// w owns the 8x8 quadrant (w & 1, w >> 1), lane l the two vertically
// adjacent pixels (l & 7, 2 (l >> 3) + {0, 1}) of it.
struct TilePixels {
  int px, py0;
  __device__ TilePixels(int tile, int tiles_x) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int qx = (tile % tiles_x) * GS_TILE + (warp & 1) * 8;
    const int qy = (tile / tiles_x) * GS_TILE + (warp >> 1) * 8;
    px = qx + (lane & 7);
    py0 = qy + 2 * (lane >> 3);
  }
};

// Minimum over the rectangle [x0,x1] x [y0,y1] of the positive-definite
// form A dx^2 + 2 B dx dy + C dy^2: 0 if the rectangle contains the origin,
// else the smallest of the four edge minima, each at the edge's clipped 1-D
// minimiser (the corner-and-edge evaluation of the reference's tile
// refinement, tiles.py:113-139).
__device__ __forceinline__ float rect_qmin(float A, float B, float C, float rbc, float rba, float x0,
                                           float x1, float y0, float y1) {
  if (x0 <= 0.0f && x1 >= 0.0f && y0 <= 0.0f && y1 >= 0.0f) return 0.0f;
  auto q = [&](float dx, float dy) { return A * dx * dx + 2.0f * B * dx * dy + C * dy * dy; };
  const float m0 = q(x0, fminf(fmaxf(-rbc * x0, y0), y1));
  const float m1 = q(x1, fminf(fmaxf(-rbc * x1, y0), y1));
  const float m2 = q(fminf(fmaxf(-rba * y0, x0), x1), y0);
  const float m3 = q(fminf(fmaxf(-rba * y1, x0), x1), y1);
  return fminf(fminf(m0, m1), fminf(m2, m3));
}

// Bit w set: warp w's 8x8 quadrant of tile `tile` may hold a pixel with
// power >= pf.  A quadrant is dropped only when its pixel-centre rectangle,
// widened by 1 px, lies outside the ellipse q <= 2 (1.05 L + 0.05),
// L = -pf — margins far above the float32 error of power near the ellipse
// (the same safety argument as cull_box, which it refines).
__device__ __forceinline__ int quad_mask(float2 m, float4 co, float pf, float4 bb, int tile,
                                         int tiles_x) {
  const float L = -pf;
  if (!(L > 0.0f)) return 0;
  const float det = co.x * co.z - co.y * co.y;
  if (!(det > 0.0f) || !(co.x > 0.0f) || !(co.z > 0.0f)) return 0xF;
  const float lim = 2.0f * (1.05f * L + 0.05f);
  const float rbc = __fdividef(co.y, co.z), rba = __fdividef(co.y, co.x);
  const float tx0 = (float)((tile % tiles_x) * GS_TILE), ty0 = (float)((tile / tiles_x) * GS_TILE);
  int mask = 0;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float qx = tx0 + (float)((w & 1) * 8), qy = ty0 + (float)((w >> 1) * 8);
    // quadrant pixel centres span [q + 0.5, q + 7.5]; box test first (cheap)
    if (bb.y < qx + 0.5f || bb.x > qx + 7.5f || bb.w < qy + 0.5f || bb.z > qy + 7.5f) continue;
    const float v = rect_qmin(co.x, co.y, co.z, rbc, rba, qx - 0.5f - m.x, qx + 8.5f - m.x,
                              qy - 0.5f - m.y, qy + 8.5f - m.y);
    if (v <= lim) mask |= 1 << w;
  }
  return mask;
}

// Staged per-Gaussian colours: one float4 per Gaussian when at most four
// channels (one shared load per Gaussian), channel-major otherwise.
template <int CMAX, int N>
struct ColStage {
  static constexpr bool kV4 = CMAX >= 1 && CMAX <= 4;
  float4 v4[kV4 ? N : 1];
  float s[kV4 ? 1 : (CMAX > 0 ? CMAX : 1)][kV4 ? 1 : N];
  __device__ __forceinline__ void put(int ch, int j, float x) {
    if (kV4)
      (&v4[j].x)[ch] = x;
    else
      s[ch][j] = x;
  }
  __device__ __forceinline__ void get(int j, float* out) const {
    if (kV4) {
      const float4 q = v4[j];
      const float t[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int ch = 0; ch < CMAX; ++ch) out[ch] = t[ch];
    } else {
#pragma unroll
      for (int ch = 0; ch < CMAX; ++ch) out[ch] = s[ch][j];
    }
  }
};

// Forward compositor.  One CTA of 128 threads per tile (TilePixels layout);
// each thread owns two pixels, so every staged Gaussian is read from shared
// memory once per two pixels.  After staging a batch, each warp compacts
// the indices of the Gaussians whose quad_mask covers its quadrant into a
// list (ballot + prefix popcount) and loops over that list only.  Front-to-back blending per pixel exactly as
// rasterize.py:74-87: skip power > 0, skip alpha < 1/255, stop before
// compositing once T would drop below 1e-4.  The CTA leaves the tile when
// all of its pixels have stopped (counted at every batch boundary).
constexpr int kFwdThreads = 128;
constexpr int kFwdBatch = 256;

template <int CMAX, bool DEPTH>
__global__ void __launch_bounds__(kFwdThreads) k_raster_fwd(const RasterArgs a) {
  constexpr int NC = CMAX > 0 ? CMAX : 1;
  __shared__ float4 s_xy[kFwdBatch];  // x, y, power floor
  __shared__ float4 s_co[kFwdBatch];  // conic a, b, c, opacity
  __shared__ int s_qm[kFwdBatch];     // quad_mask
  __shared__ ColStage<CMAX, kFwdBatch> s_col;
  __shared__ float s_z[DEPTH ? kFwdBatch : 1];
  __shared__ short s_list[kFwdThreads / 32][kFwdBatch];

  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const TilePixels tp(tile, a.tiles_x);
  const int px = tp.px, py0 = tp.py0;
  const float pxf = (float)px + 0.5f;
  const int start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  const int num = end - start;

  bool inside[2], done[2];
  float pyf[2], T[2], dacc[2];
  float acc[2][NC];
  int last[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    inside[p] = px < a.width && py0 + p < a.height;
    done[p] = !inside[p];
    pyf[p] = (float)(py0 + p) + 0.5f;
    T[p] = 1.0f;
    dacc[p] = 0.0f;
    last[p] = 0;
#pragma unroll
    for (int ch = 0; ch < NC; ++ch) acc[p][ch] = 0.0f;
  }

  for (int b0 = 0; b0 < num; b0 += kFwdBatch) {
    // Barrier before the batch overwrites shared memory; also ends the tile
    // once every pixel has terminated.
    if (__syncthreads_count(done[0] && done[1]) == kFwdThreads) break;
#pragma unroll
    for (int r = 0; r < kFwdBatch / kFwdThreads; ++r) {
      const int t = threadIdx.x + r * kFwdThreads;
      const int li = start + b0 + t;
      if (li < end) {
        const int g = __ldg(a.ids + li);
        const float2 m = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
        const float o = __ldg(a.opac + g);
        const float4 co = make_float4(__ldg(a.conics + 3 * g), __ldg(a.conics + 3 * g + 1),
                                      __ldg(a.conics + 3 * g + 2), o);
        const float pf = power_floor(o);
        s_xy[t] = make_float4(m.x, m.y, pf, 0.0f);
        // -a/2 and -c/2: scaling by a power of two commutes with rounding, so
        // (-a/2 dx) dx + (-c/2 dy) dy == -0.5 ((a dx) dx + (c dy) dy) exactly
        s_co[t] = make_float4(-0.5f * co.x, co.y, -0.5f * co.z, co.w);
        s_qm[t] = quad_mask(m, co, pf, cull_box(m, co, pf), tile, a.tiles_x);
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch)
          if (ch < a.cc) s_col.put(ch, t, __ldg(a.colors + (int64_t)g * a.c_total + a.c0 + ch));
        if (DEPTH) s_z[t] = __ldg(a.depths + g);
      }
    }
    __syncthreads();
    const int bs = min(kFwdBatch, num - b0);
    // this warp's hits of the batch, in order
    int cnt = 0;
    const int lane = threadIdx.x & 31;
    for (int c = 0; c < bs; c += 32) {
      const int jj = c + lane;
      const bool hit = jj < bs && ((s_qm[jj] >> warp) & 1);
      const unsigned bal = __ballot_sync(0xffffffffu, hit);
      if (hit) s_list[warp][cnt + __popc(bal & ((1u << lane) - 1u))] = (short)jj;
      cnt += __popc(bal);
    }
    __syncwarp();
    for (int t = 0; t < cnt; ++t) {
      if (done[0] && done[1]) break;
      const int j = s_list[warp][t];
      const float4 mq = s_xy[j];
      const float2 m = make_float2(mq.x, mq.y);
      const float4 co = s_co[j];
      const float pf = mq.z;
      const float dx = gs_sub(m.x, pxf);
      const float adxdx = gs_mul(gs_mul(co.x, dx), dx);  // co.x = -a/2
      const float bdx = gs_mul(co.y, dx);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float dy = gs_sub(m.y, pyf[p]);
        const float power =
            gs_sub(gs_add(adxdx, gs_mul(gs_mul(co.z, dy), dy)), gs_mul(bdx, dy));
        // Predicated (no per-pixel branches): the exponential's argument is
        // replaced by 0 where the pixel does not take the Gaussian, and
        // every state update is a select, so composited values are the
        // exact ones of the branchy form.  fminf == gs_minf here (no NaN).
        bool take = !done[p] && power <= 0.0f && power >= pf;
        const float alpha = fminf(GS_ALPHA_MAX, gs_mul(co.w, gs_expf_nonpos(take ? power : 0.0f)));
        take = take && alpha >= GS_ALPHA_MIN;
        const float next_T = gs_mul(T[p], gs_sub(1.0f, alpha));
        const bool stop = take && next_T < GS_T_MIN;
        done[p] = done[p] || stop;
        take = take && !stop;
        const float w = gs_mul(alpha, T[p]);
        float cj[NC];
        s_col.get(j, cj);
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch) {
          const float na = gs_add(acc[p][ch], gs_mul(cj[ch], w));
          acc[p][ch] = take ? na : acc[p][ch];
        }
        if (DEPTH) {
          const float nd = gs_add(dacc[p], gs_mul(s_z[j], w));
          dacc[p] = take ? nd : dacc[p];
        }
        T[p] = take ? next_T : T[p];
        last[p] = take ? b0 + j + 1 : last[p];
      }
    }
  }
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    if (!inside[p]) continue;
    const int64_t pid = (int64_t)(py0 + p) * a.width + px;
    if (a.image) {
#pragma unroll
      for (int ch = 0; ch < CMAX; ++ch) {
        if (ch < a.cc) {
          const float bgv = a.bg ? a.bg[a.c0 + ch] : 0.0f;
          a.image[pid * a.c_total + a.c0 + ch] = gs_add(acc[p][ch], gs_mul(T[p], bgv));
        }
      }
    }
    if (a.write_aux) {
      if (a.final_T) a.final_T[pid] = T[p];
      if (a.n_contrib) a.n_contrib[pid] = last[p];
      if (DEPTH && a.depth) {
        const float al = gs_sub(1.0f, T[p]);
        a.depth[pid] = al > 1e-6f ? gs_div(dacc[p], al) : 0.0f;
      }
    }
  }
}

struct RasterBwdArgs {
  RasterArgs f;
  const float *grad_image, *grad_final_T;
  int use_grad_final_T;
  float *g_means2d, *g_conics, *g_colors, *g_opac;
};

// Sum over the 32 lanes of a warp of eight per-lane values v[0..7], leaving
// the total of value ((lane>>4)&1)*4 + ((lane>>3)&1)*2 + ((lane>>2)&1) in
// every lane: three halving exchanges (4 + 2 + 1 shuffles) followed by a
// two-step butterfly — 9 shuffles instead of 8 x 5 for separate butterflies.
__device__ __forceinline__ float warp_reduce8(const float* v, int lane) {
  const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4;
  float a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = u16 ? v[i] : v[i + 4];
    const float keep = u16 ? v[i + 4] : v[i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float b[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = u8 ? a[i] : a[i + 2];
    const float keep = u8 ? a[i + 2] : a[i];
    b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float send = u4 ? b[0] : b[1];
  float c = (u4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, send, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Backward compositor.  One CTA of 128 threads per tile (TilePixels layout),
// each thread owning two pixels of its warp's 8x8 quadrant.  For every
// staged Gaussian j (back to front) each thread sums its two pixels'
// gradient contributions in registers, the warp reduces them
// (warp_reduce8), the per-warp totals go to shared memory without atomics,
// and after the batch one thread per Gaussian adds the warps' totals to the
// global gradients with one atomic per value.
//
// Gradient values per Gaussian: 0-1 means2d, 2-4 conic, 5 opacity,
// 6.. colour channels.
constexpr int kBwdThreads = 128;
constexpr int kBwdWarps = kBwdThreads / 32;

template <int CMAX>
__global__ void __launch_bounds__(kBwdThreads) k_raster_bwd(const RasterBwdArgs g) {
  const RasterArgs& a = g.f;
  constexpr int NV = 6 + CMAX;
  constexpr int NV8 = (NV / 8) * 8;  // values reduced by warp_reduce8
  constexpr int BATCH = CMAX <= 4 ? 128 : 64;
  __shared__ int s_id[BATCH];
  __shared__ float4 s_xy[BATCH];
  __shared__ float4 s_co[BATCH];
  __shared__ int s_qm[BATCH];
  __shared__ ColStage<CMAX, BATCH> s_col;
  // per-warp gradient totals; the +1 pitch puts the eight values a warp
  // stores for one Gaussian in eight different banks
  __shared__ float s_gw[kBwdWarps][NV][BATCH + 1];
  __shared__ int s_max_last;
  __shared__ short s_blist[kBwdWarps][BATCH];

  const int tile = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const TilePixels tp(tile, a.tiles_x);
  const int px = tp.px, py0 = tp.py0;
  const float pxf = (float)px + 0.5f;
  const int start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  const int num = end - start;

  // Per-pixel state of the back-to-front replay.  The reference keeps the
  // colour composited behind the current Gaussian, accum (rasterize.py:183),
  // and uses (c - accum) . dL/dpix * T.  Since T_i * accum_i . dL/dpix =
  // R_i / (1 - alpha_i) with R_i = sum_{j > i} (c_j . dL/dpix) alpha_j T_j,
  // one scalar R per pixel carries the same information; it starts at the
  // background term T_final * (bg . dL/dpix + dL/dT_final), which enters
  // every dL/dalpha the same way.
  bool inside[2];
  float pyf[2], T[2], R[2];
  int last[2];
  float dpix[2][CMAX];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int py = py0 + p;
    inside[p] = px < a.width && py < a.height;
    pyf[p] = (float)py + 0.5f;
    const int64_t pid = (int64_t)py * a.width + px;
    const float T_final = inside[p] ? a.final_T[pid] : 1.0f;
    T[p] = T_final;
    last[p] = inside[p] ? a.n_contrib[pid] : 0;
    float bg_dot = 0.0f;
#pragma unroll
    for (int ch = 0; ch < CMAX; ++ch) {
      dpix[p][ch] = 0.0f;
      if (inside[p] && ch < a.cc) {
        dpix[p][ch] = g.grad_image[pid * a.c_total + a.c0 + ch];
        if (a.bg) bg_dot += a.bg[a.c0 + ch] * dpix[p][ch];
      }
    }
    if (inside[p] && g.use_grad_final_T && g.grad_final_T) bg_dot += g.grad_final_T[pid];
    R[p] = T_final * bg_dot;
  }

  // Nothing at or beyond the largest n_contrib of a warp (block) matters.
  int wmax = max(last[0], last[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  if (threadIdx.x == 0) s_max_last = 0;
  __syncthreads();
  if (lane == 0) atomicMax(&s_max_last, wmax);
  __syncthreads();
  const int nbat = (s_max_last + BATCH - 1) / BATCH;

  for (int b = nbat - 1; b >= 0; --b) {
    const int b0 = b * BATCH;
    __syncthreads();
    if (threadIdx.x < BATCH) {
      const int li = start + b0 + threadIdx.x;
      if (li < end) {
        const int gid = __ldg(a.ids + li);
        s_id[threadIdx.x] = gid;
        const float2 m = __ldg(reinterpret_cast<const float2*>(a.means2d) + gid);
        const float o = __ldg(a.opac + gid);
        const float4 co = make_float4(__ldg(a.conics + 3 * gid), __ldg(a.conics + 3 * gid + 1),
                                      __ldg(a.conics + 3 * gid + 2), o);
        const float pf = power_floor(o);
        s_xy[threadIdx.x] = make_float4(m.x, m.y, pf, 0.0f);
        s_co[threadIdx.x] = make_float4(-0.5f * co.x, co.y, -0.5f * co.z, co.w);  // see the forward
        s_qm[threadIdx.x] = quad_mask(m, co, pf, cull_box(m, co, pf), tile, a.tiles_x);
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch)
          s_col.put(ch, threadIdx.x, ch < a.cc ? __ldg(a.colors + (int64_t)gid * a.c_total + a.c0 + ch) : 0.0f);
      }
    }
    for (int e = threadIdx.x; e < kBwdWarps * NV * (BATCH + 1); e += kBwdThreads) (&s_gw[0][0][0])[e] = 0.0f;
    __syncthreads();
    const int bs = min(BATCH, num - b0);
    const int jtop = min(bs, wmax - b0) - 1;
    // this warp's hits among entries 0..jtop, replayed back to front
    int cnt = 0;
    for (int c = 0; c <= jtop; c += 32) {
      const int jj = c + lane;
      const bool hit = jj <= jtop && ((s_qm[jj] >> warp) & 1);
      const unsigned bal = __ballot_sync(0xffffffffu, hit);
      if (hit) s_blist[warp][cnt + __popc(bal & ((1u << lane) - 1u))] = (short)jj;
      cnt += __popc(bal);
    }
    __syncwarp();
    for (int t = cnt - 1; t >= 0; --t) {
      const int j = s_blist[warp][t];

      const float4 co = s_co[j];
      const float4 mq = s_xy[j];
      const float2 m = make_float2(mq.x, mq.y);
      const float pf = mq.z;
      // Cheap test first: power and the opacity floor decide every pair
      // except those in the floor's 1e-3 margin, so a step in which no lane
      // passes it (about a fifth of them at C2) skips the rest.
      const float dx = gs_sub(m.x, pxf);
      float dyv[2], pw[2];
      bool pre[2];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        dyv[p] = gs_sub(m.y, pyf[p]);
        pw[p] = gs_sub(gs_add(gs_mul(gs_mul(co.x, dx), dx), gs_mul(gs_mul(co.z, dyv[p]), dyv[p])),
                       gs_mul(gs_mul(co.y, dx), dyv[p]));
        pre[p] = b0 + j < last[p] && pw[p] <= 0.0f && pw[p] >= pf;
      }
      if (!__any_sync(0xffffffffu, pre[0] || pre[1])) continue;
      float gv[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) gv[k] = 0.0f;
      bool any = false;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float dy = dyv[p];
        const float power = pw[p];
        // Predicated (no per-pixel branches): lanes that do not composite
        // this Gaussian evaluate the same arithmetic and add zeros.  The
        // gradient needs e^power only to float accuracy, but the skip
        // decision alpha < 1/255 must be the forward's: take the hardware
        // exponential (relative error ~1e-7) and redo it exactly only when
        // alpha lands within 1e-5 of the threshold.
        bool take = pre[p];
        float G = __expf(take ? power : 0.0f);
        float alpha = gs_minf(GS_ALPHA_MAX, gs_mul(co.w, G));
        if (take && fabsf(alpha - GS_ALPHA_MIN) < 1e-5f * GS_ALPHA_MIN) {
          G = gs_expf(power);
          alpha = gs_minf(GS_ALPHA_MAX, gs_mul(co.w, G));
        }
        take = take && alpha >= GS_ALPHA_MIN;
        any = any || take;
        const float ra = __fdividef(1.0f, 1.0f - alpha);
        const float Tn = T[p] * ra;
        const float aT = alpha * Tn;
        float cd = 0.0f;
        float cj[CMAX];
        s_col.get(j, cj);
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch) cd += cj[ch] * dpix[p][ch];
        const float dL_dalpha = Tn * cd - R[p] * ra;
        const float gdl = take ? G * dL_dalpha : 0.0f;
        const float aTm = take ? aT : 0.0f;
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch) gv[6 + ch] += aTm * dpix[p][ch];
        // d power / d(mean, conic) with u = G dL/dG (co.x = -a/2, co.z = -c/2):
        //   means2d: -u (a dx + b dy), -u (b dx + c dy)
        //   conic:   -u dx^2 / 2, -u dx dy, -u dy^2 / 2
        // are linear in the sums of u dx, u dy, u dx^2, u dx dy, u dy^2 over
        // the pixels (a, b, c fixed per Gaussian): those five sums are
        // accumulated and reduced, and the conic applied once per Gaussian.
        const float u = co.w * gdl;
        const float ux = u * dx, uy = u * dy;
        gv[0] += ux;
        gv[1] += uy;
        gv[2] += ux * dx;
        gv[3] += ux * dy;
        gv[4] += uy * dy;
        gv[5] += gdl;
        T[p] = take ? Tn : T[p];
        R[p] = take ? R[p] + cd * aT : R[p];
      }
      const unsigned takers = __ballot_sync(0xffffffffu, any);
      if (!takers) continue;
      if ((takers & (takers - 1u)) == 0u) {
        // one lane composited: its sums are the warp's, no reduction
        if (any) {
#pragma unroll
          for (int k = 0; k < NV; ++k)
            if (k < 6 + a.cc) s_gw[warp][k][j] = gv[k];
        }
        continue;
      }
#pragma unroll
      for (int k8 = 0; k8 < NV8; k8 += 8) {
        const float t = warp_reduce8(gv + k8, lane);
        if ((lane & 3) == 0) {
          const int idx = k8 + ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
          if (idx < 6 + a.cc) s_gw[warp][idx][j] = t;
        }
      }
#pragma unroll
      for (int k = NV8; k < NV; ++k) {
        if (k >= 6 + a.cc) break;
        const float t = warp_sum(gv[k]);
        if (lane == 0) s_gw[warp][k][j] = t;
      }
    }
    __syncthreads();
    if (threadIdx.x < bs) {
      const int t = threadIdx.x;
      float tot[NV];
      bool hit = false;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kBwdWarps; ++w) v += s_gw[w][k][t];
        tot[k] = v;
        hit |= v != 0.0f;
      }
      if (hit) {
        // sums of u dx, u dy, u dx^2, u dx dy, u dy^2 -> gradients
        const float4 cq = s_co[t];  // -a/2, b, -c/2
        const float sx = tot[0], sy = tot[1];
        tot[0] = 2.0f * cq.x * sx - cq.y * sy;
        tot[1] = 2.0f * cq.z * sy - cq.y * sx;
        tot[2] = -0.5f * tot[2];
        tot[3] = -tot[3];
        tot[4] = -0.5f * tot[4];
        const int gid = s_id[t];
        atomicAdd(reinterpret_cast<float2*>(g.g_means2d) + gid, make_float2(tot[0], tot[1]));
        atomicAdd(g.g_conics + 3 * gid, tot[2]);
        atomicAdd(g.g_conics + 3 * gid + 1, tot[3]);
        atomicAdd(g.g_conics + 3 * gid + 2, tot[4]);
        atomicAdd(g.g_opac + gid, tot[5]);
#pragma unroll
        for (int ch = 0; ch < CMAX; ++ch)
          if (ch < a.cc) atomicAdd(g.g_colors + (int64_t)gid * a.c_total + a.c0 + ch, tot[6 + ch]);
      }
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
    k_raster_fwd<CMAX, true><<<grid, kFwdThreads, 0, s>>>(a);
  else
    k_raster_fwd<CMAX, false><<<grid, kFwdThreads, 0, s>>>(a);
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
    case 1: k_raster_bwd<1><<<grid, kBwdThreads, 0, s>>>(g); break;
    case 2: k_raster_bwd<2><<<grid, kBwdThreads, 0, s>>>(g); break;
    case 3: k_raster_bwd<3><<<grid, kBwdThreads, 0, s>>>(g); break;
    case 4: k_raster_bwd<4><<<grid, kBwdThreads, 0, s>>>(g); break;
    case 8: k_raster_bwd<8><<<grid, kBwdThreads, 0, s>>>(g); break;
    default: k_raster_bwd<16><<<grid, kBwdThreads, 0, s>>>(g); break;
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
  // Per-Gaussian inputs may be NULL only when every tile range is empty
  // (a scene with no Gaussians).
  if (!tile_ranges || !final_T)
    return set_error(GS_ERR_INVALID_ARG, "gs_rasterize_forward: NULL tile_ranges / final_T");
  if (channels > 0 && !image)
    return set_error(GS_ERR_INVALID_ARG, "image must be given when channels > 0");
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
  if (n == 0) return GS_OK;  // no Gaussians, no gradients
  if (!means2d || !conics || !colors || !opacities || !sorted_ids || !tile_ranges || !final_T ||
      !n_contrib || !grad_image || !grad_means2d || !grad_conics || !grad_colors || !grad_opacities)
    return set_error(GS_ERR_INVALID_ARG, "gs_rasterize_backward: NULL pointer");
  if (!aligned(means2d, 8) || !aligned(grad_means2d, 8))
    return set_error(GS_ERR_INVALID_ARG, "means2d / grad_means2d must be 8-byte aligned");
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
