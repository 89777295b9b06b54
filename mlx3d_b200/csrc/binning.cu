// Tile binning: depth order, duplication per touched tile, stable sort by
// tile, per-tile ranges (src/mlx3d/splatting/tiles.py:19-182).
//
// The reference sorts the D duplicates once by the int64 key
// tile * N + rank(depth) (tiles.py:166-173).  The same order is produced
// here with far fewer bits moved over D:
//   1. LSD radix sort of the N per-Gaussian depth keys (float bits; every
//      touching Gaussian has depth > znear > 0, so the bits order like the
//      values).  Gaussians that touch no tile get the key 0xFFFFFFFF.  The
//      sort is stable over an index-ordered input, so equal depths keep
//      Gaussian index order — exactly the order of distinct ranks.
//   2. Duplicates are emitted in that depth order.
//   3. A stable LSD radix sort of the duplicates by tile id alone
//      (ceil(log2(tiles)/8) passes, 1-2 for every configuration here).
// Stable (tile, then depth order) == sort by tile * N + rank.
//
// Each radix pass is reduce-then-scan (per-block digit histograms, a scan
// over them, a stable scatter), so no block ever waits on another block.
#include <algorithm>
#include <utility>

#include "gs_common.cuh"

namespace gs {

constexpr int RS_THREADS = 256;
constexpr int RS_WARPS = RS_THREADS / 32;
constexpr int RS_ITEMS = 8;
constexpr int RS_TILE = RS_THREADS * RS_ITEMS;  // keys per block
constexpr int RS_RADIX = 256;
constexpr int DEPTH_PASSES = 4;
constexpr int MAX_TILE_PASSES = 4;

// ------------------------------------------------------------- radix passes
// Per-block histogram of one 8-bit digit; block digit counts are stored
// digit-major (hist[d * nb + block]) and summed into gtot[d].
__global__ void __launch_bounds__(RS_THREADS)
k_rs_upsweep(const uint32_t* __restrict__ keys, int64_t n, int shift, uint32_t* __restrict__ hist,
             uint32_t* __restrict__ gtot, int nb) {
  __shared__ uint32_t h[RS_WARPS][RS_RADIX];
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < RS_WARPS * RS_RADIX; i += RS_THREADS) (&h[0][0])[i] = 0;
  __syncthreads();
  // RS_ITEMS consecutive keys per thread, loaded as 16-byte vectors (key
  // buffers are 256-byte aligned and blocks start at multiples of RS_TILE),
  // all loads issued before the shared-memory counting.
  const int64_t first = (int64_t)blockIdx.x * RS_TILE + (int64_t)threadIdx.x * RS_ITEMS;
  uint32_t k[RS_ITEMS];
  if (first + RS_ITEMS <= n) {
#pragma unroll
    for (int v = 0; v < RS_ITEMS / 4; ++v) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(keys + first) + v);
      k[4 * v] = q.x; k[4 * v + 1] = q.y; k[4 * v + 2] = q.z; k[4 * v + 3] = q.w;
    }
#pragma unroll
    for (int it = 0; it < RS_ITEMS; ++it) atomicAdd(&h[warp][(k[it] >> shift) & 255u], 1u);
  } else {
    for (int it = 0; it < RS_ITEMS; ++it)
      if (first + it < n) atomicAdd(&h[warp][(__ldg(keys + first + it) >> shift) & 255u], 1u);
  }
  __syncthreads();
  const int d = threadIdx.x;
  uint32_t s = 0;
#pragma unroll
  for (int w = 0; w < RS_WARPS; ++w) s += h[w][d];
  hist[(int64_t)d * nb + blockIdx.x] = s;
  if (s) atomicAdd(gtot + d, s);
}

// Exclusive scan of one digit's row of block counts, offset by the counts of
// all smaller digits.  One block per digit.
__global__ void __launch_bounds__(RS_THREADS)
k_rs_scan(uint32_t* __restrict__ hist, const uint32_t* __restrict__ gtot, int nb) {
  __shared__ uint32_t warp_sums[RS_WARPS];
  __shared__ uint32_t carry;
  const int d = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // base = sum of gtot[0..d)
  uint32_t v = threadIdx.x < d ? gtot[threadIdx.x] : 0u;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) warp_sums[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = 0;
    for (int w = 0; w < RS_WARPS; ++w) b += warp_sums[w];
    carry = b;
  }
  __syncthreads();
  uint32_t* row = hist + (int64_t)d * nb;
  for (int start = 0; start < nb; start += RS_THREADS) {
    const int i = start + threadIdx.x;
    const uint32_t x = i < nb ? row[i] : 0u;
    // inclusive warp scan
    uint32_t s = x;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += t;
    }
    __syncthreads();  // previous iteration's readers of warp_sums / carry are done
    if (lane == 31) warp_sums[warp] = s;
    __syncthreads();
    uint32_t wpre = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < RS_WARPS; ++w) {
      const uint32_t ws = warp_sums[w];
      if (w < warp) wpre += ws;
      tot += ws;
    }
    const uint32_t c = carry;
    if (i < nb) row[i] = c + wpre + s - x;
    __syncthreads();
    if (threadIdx.x == 0) carry = c + tot;
  }
}

// Stable scatter of one block of keys (and values) by one 8-bit digit.
// Items are ranked warp by warp in index order with __match_any_sync, then
// offset by the per-digit counts of earlier warps in the block and by the
// block's scanned global offset.
template <bool KEYS_OUT>
__global__ void __launch_bounds__(RS_THREADS)
k_rs_downsweep(const uint32_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
               uint32_t* __restrict__ keys_out, int32_t* __restrict__ vals_out, int64_t n,
               int shift, const uint32_t* __restrict__ hist, int nb) {
  __shared__ uint32_t wcnt[RS_WARPS][RS_RADIX];
  __shared__ uint32_t gbase[RS_RADIX];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < RS_WARPS * RS_RADIX; i += RS_THREADS) (&wcnt[0][0])[i] = 0;
  gbase[threadIdx.x] = hist[(int64_t)threadIdx.x * nb + blockIdx.x];
  __syncthreads();
  const int64_t seg = (int64_t)blockIdx.x * RS_TILE + warp * (32 * RS_ITEMS);
  const unsigned lt = (1u << lane) - 1u;
  uint32_t k[RS_ITEMS];
  int32_t v[RS_ITEMS];
  uint32_t rank[RS_ITEMS];
#pragma unroll
  for (int it = 0; it < RS_ITEMS; ++it) {
    const int64_t idx = seg + it * 32 + lane;
    const bool valid = idx < n;
    k[it] = valid ? __ldg(keys_in + idx) : 0u;
    v[it] = valid ? __ldg(vals_in + idx) : 0;
    const uint32_t d = valid ? ((k[it] >> shift) & 255u) : 256u;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const uint32_t cnt = valid ? wcnt[warp][d] : 0u;
    __syncwarp();
    if (valid && (peers & lt) == 0u) wcnt[warp][d] = cnt + __popc(peers);
    __syncwarp();
    rank[it] = cnt + __popc(peers & lt);
  }
  __syncthreads();
  {
    const int d = threadIdx.x;
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < RS_WARPS; ++w) {
      const uint32_t t = wcnt[w][d];
      wcnt[w][d] = run;
      run += t;
    }
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < RS_ITEMS; ++it) {
    const int64_t idx = seg + it * 32 + lane;
    if (idx < n) {
      const uint32_t d = (k[it] >> shift) & 255u;
      const uint32_t pos = gbase[d] + wcnt[warp][d] + rank[it];
      if (KEYS_OUT) keys_out[pos] = k[it];
      vals_out[pos] = v[it];
    }
  }
}

// --------------------------------------------------------- binning kernels
// Sum of the tiles-touched counts (= D) into *total (zeroed by the caller).
__global__ void k_count_total(const int32_t* __restrict__ counts, int64_t n,
                              unsigned long long* __restrict__ total) {
  unsigned long long s = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    s += (unsigned)counts[i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0 && s) atomicAdd(total, s);
}

__global__ void k_depth_keys(const float* __restrict__ depths, const int32_t* __restrict__ counts,
                             int64_t n, uint32_t* __restrict__ keys, int32_t* __restrict__ vals) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  keys[i] = counts[i] > 0 ? gs_float_to_bits(depths[i]) : 0xFFFFFFFFu;
  vals[i] = (int32_t)i;
}

// Device-wide exclusive scan of counts[perm[i]] (int32), reduce-then-scan.
constexpr int SC_THREADS = 256, SC_ITEMS = 16, SC_TILE = SC_THREADS * SC_ITEMS;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t x, uint32_t* warp_sums,
                                                        uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t s = x;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += t;
  }
  if (lane == 31) warp_sums[warp] = s;
  __syncthreads();
  uint32_t pre = 0, tot = 0;
  for (int w = 0; w < SC_THREADS / 32; ++w) {
    const uint32_t ws = warp_sums[w];
    if (w < warp) pre += ws;
    tot += ws;
  }
  __syncthreads();
  total = tot;
  return pre + s - x;
}

__global__ void __launch_bounds__(SC_THREADS)
k_scan_reduce(const int32_t* __restrict__ counts, const int32_t* __restrict__ perm, int64_t n,
              unsigned long long* __restrict__ bsum) {
  __shared__ unsigned long long ws[SC_THREADS / 32];
  const int64_t base = (int64_t)blockIdx.x * SC_TILE;
  unsigned long long s = 0;
  for (int i = threadIdx.x; i < SC_TILE; i += SC_THREADS) {
    const int64_t idx = base + i;
    if (idx < n) s += (unsigned)counts[perm[idx]];
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int w = 0; w < SC_THREADS / 32; ++w) t += ws[w];
    bsum[blockIdx.x] = t;
  }
}

// Single block: exclusive scan of the block sums; writes the grand total.
constexpr int SB_THREADS = 1024;
__global__ void __launch_bounds__(SB_THREADS)
k_scan_bsums(unsigned long long* __restrict__ bsum, int nb, int64_t* __restrict__ total) {
  __shared__ unsigned long long warp_sums[SB_THREADS / 32];
  __shared__ unsigned long long carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  for (int start = 0; start < nb; start += SB_THREADS) {
    const int i = start + threadIdx.x;
    const unsigned long long x = i < nb ? bsum[i] : 0ull;
    unsigned long long s = x;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long t = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += t;
    }
    __syncthreads();
    if (lane == 31) warp_sums[warp] = s;
    __syncthreads();
    unsigned long long pre = 0, tot = 0;
    for (int w = 0; w < SB_THREADS / 32; ++w) {
      const unsigned long long ws = warp_sums[w];
      if (w < warp) pre += ws;
      tot += ws;
    }
    const unsigned long long c = carry;
    if (i < nb) bsum[i] = c + pre + s - x;
    __syncthreads();
    if (threadIdx.x == 0) carry = c + tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) *total = (int64_t)carry;
}

__global__ void __launch_bounds__(SC_THREADS)
k_scan_down(const int32_t* __restrict__ counts, const int32_t* __restrict__ perm, int64_t n,
            const unsigned long long* __restrict__ bsum, uint32_t* __restrict__ offsets) {
  __shared__ uint32_t warp_sums[SC_THREADS / 32];
  const int64_t base = (int64_t)blockIdx.x * SC_TILE + (int64_t)threadIdx.x * SC_ITEMS;
  uint32_t c[SC_ITEMS];
  uint32_t local = 0;
#pragma unroll
  for (int j = 0; j < SC_ITEMS; ++j) {
    const int64_t idx = base + j;
    c[j] = idx < n ? (uint32_t)counts[perm[idx]] : 0u;
    local += c[j];
  }
  uint32_t total;
  uint32_t run = block_exclusive_scan(local, warp_sums, total) + (uint32_t)bsum[blockIdx.x];
#pragma unroll
  for (int j = 0; j < SC_ITEMS; ++j) {
    const int64_t idx = base + j;
    if (idx < n) offsets[idx] = run;
    run += c[j];
  }
}

// AccuTile refinement of one (Gaussian, tile) pair (tiles.py:91-141): the
// exact minimum over the tile rectangle of the conic form
// a dx^2 + 2 b dx dy + c dy^2 (corners plus the four clipped edge
// minimisers; 0 when the centre lies inside), kept if <= 12.  Float32
// operations in the reference's order.
__device__ __forceinline__ bool refine_keep(const float* __restrict__ co, float gx, float gy, int tx,
                                            int ty, int width, int height) {
  const float x0 = (float)(tx * GS_TILE), y0 = (float)(ty * GS_TILE);
  const float x1 = (float)min((tx + 1) * GS_TILE, width), y1 = (float)min((ty + 1) * GS_TILE, height);
  const float dxl = gs_sub(x0, gx), dxr = gs_sub(x1, gx);
  const float dyb = gs_sub(y0, gy), dyt = gs_sub(y1, gy);
  const float a = co[0], b = co[1], c = co[2];
  const float b2 = gs_mul(2.0f, b);
  auto q = [&](float dx, float dy) {
    return gs_add(gs_add(gs_mul(gs_mul(a, dx), dx), gs_mul(gs_mul(b2, dx), dy)), gs_mul(gs_mul(c, dy), dy));
  };
  auto clip = [](float v, float lo, float hi) { return gs_minf(gs_maxf(v, lo), hi); };
  const float nbc = -gs_div(b, c), nba = -gs_div(b, a);
  const float dy_left = clip(gs_mul(nbc, dxl), dyb, dyt);
  const float dy_right = clip(gs_mul(nbc, dxr), dyb, dyt);
  const float dx_bottom = clip(gs_mul(nba, dyb), dxl, dxr);
  const float dx_top = clip(gs_mul(nba, dyt), dxl, dxr);
  float qm = q(dxl, dyb);
  qm = gs_minf(qm, q(dxl, dyt));
  qm = gs_minf(qm, q(dxr, dyb));
  qm = gs_minf(qm, q(dxr, dyt));
  qm = gs_minf(qm, q(dxl, dy_left));
  qm = gs_minf(qm, q(dxr, dy_right));
  qm = gs_minf(qm, q(dx_bottom, dyb));
  qm = gs_minf(qm, q(dx_top, dyt));
  const bool inside = dxl <= 0.0f && dxr >= 0.0f && dyb <= 0.0f && dyt >= 0.0f;
  return (inside ? 0.0f : qm) <= 12.0f;
}

// Inclusive tile rectangle of an on-screen Gaussian (tiles.py:54-62); false
// when it touches no tile.
__device__ __forceinline__ bool gauss_rect(float2 m, float r, int width, int height, int tiles_x,
                                           int tiles_y, int& x0, int& y0, int& x1, int& y1) {
  const float fx1 = (float)(tiles_x - 1), fy1 = (float)(tiles_y - 1);
  const float T = (float)GS_TILE;
  const bool on = (r > 0.0f) && (gs_add(m.x, r) >= 0.0f) && (gs_sub(m.x, r) < (float)width) &&
                  (gs_add(m.y, r) >= 0.0f) && (gs_sub(m.y, r) < (float)height);
  if (!on) return false;
  x0 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_sub(m.x, r), T)), 0.0f), fx1);
  x1 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_add(m.x, r), T)), 0.0f), fx1);
  y0 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_sub(m.y, r), T)), 0.0f), fy1);
  y1 = (int)gs_minf(gs_maxf(floorf(gs_div(gs_add(m.y, r), T)), 0.0f), fy1);
  return true;
}

// Tiles kept by the refinement, per Gaussian (the refined "tiles touched").
__global__ void k_tile_counts_refined(const float* __restrict__ means2d, const float* __restrict__ radii,
                                      const float* __restrict__ conics, int64_t n, int width, int height,
                                      int tiles_x, int tiles_y, int32_t* __restrict__ counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float2 m = reinterpret_cast<const float2*>(means2d)[i];
  int x0, y0, x1, y1, c = 0;
  if (gauss_rect(m, radii[i], width, height, tiles_x, tiles_y, x0, y0, x1, y1))
    for (int ty = y0; ty <= y1; ++ty)
      for (int tx = x0; tx <= x1; ++tx) c += refine_keep(conics + 3 * i, m.x, m.y, tx, ty, width, height);
  counts[i] = c;
}

// One thread per Gaussian in depth order: write (tile id, Gaussian id) for
// every tile of its rectangle, row-major (tiles.py:77-89), or, with REFINE,
// for every tile the refinement keeps (tiles.py:141-163).
template <bool REFINE>
__global__ void k_duplicate(const float* __restrict__ means2d, const float* __restrict__ radii,
                            const float* __restrict__ conics, const int32_t* __restrict__ perm,
                            const uint32_t* __restrict__ offsets, int64_t n, int64_t d, int width,
                            int height, int tiles_x, int tiles_y, uint32_t* __restrict__ tkeys,
                            int32_t* __restrict__ tvals) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t g = perm[i];
  const float2 m = reinterpret_cast<const float2*>(means2d)[g];
  int x0, y0, x1, y1;
  if (!gauss_rect(m, radii[g], width, height, tiles_x, tiles_y, x0, y0, x1, y1)) return;
  uint32_t o = offsets[i];
  for (int ty = y0; ty <= y1; ++ty)
    for (int tx = x0; tx <= x1; ++tx) {
      if (REFINE && !refine_keep(conics + 3 * (int64_t)g, m.x, m.y, tx, ty, width, height)) continue;
      if ((int64_t)o >= d) return;  // never past the caller's D (counts are recomputed exactly)
      tkeys[o] = (uint32_t)(ty * tiles_x + tx);
      tvals[o] = g;
      ++o;
    }
}

// [start, end) of every non-empty tile from the tile-sorted keys; empty
// tiles keep the zero-initialised [0, 0) (tiles.py:175-180).
__global__ void k_tile_ranges(const uint32_t* __restrict__ tkeys, int64_t d,
                              int32_t* __restrict__ ranges) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d) return;
  const uint32_t t = tkeys[i];
  if (i == 0 || tkeys[i - 1] != t) ranges[2 * (int64_t)t] = (int32_t)i;
  if (i == d - 1 || tkeys[i + 1] != t) ranges[2 * (int64_t)t + 1] = (int32_t)(i + 1);
}

// --------------------------------------------------------- workspace layout
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct NLayout {
  size_t keys0, keys1, vals0, vals1, offsets, hist, gtot, bsum, total;
  int nb_rs, nb_sc;
  NLayout(int64_t n) {
    nb_rs = (int)ceil_div(n > 0 ? n : 1, RS_TILE);
    nb_sc = (int)ceil_div(n > 0 ? n : 1, SC_TILE);
    size_t o = 0;
    keys0 = o; o += align256(4 * (size_t)n);
    keys1 = o; o += align256(4 * (size_t)n);
    vals0 = o; o += align256(4 * (size_t)n);
    vals1 = o; o += align256(4 * (size_t)n);
    offsets = o; o += align256(4 * (size_t)n);
    hist = o; o += align256(4 * (size_t)RS_RADIX * nb_rs);
    gtot = o; o += align256(4 * (size_t)RS_RADIX * DEPTH_PASSES);
    bsum = o; o += align256(8 * (size_t)nb_sc);
    total = o;
  }
};

struct DLayout {
  size_t keys0, keys1, vals0, vals1, hist, gtot, total;
  int nb_rs;
  DLayout(int64_t d) {
    nb_rs = (int)ceil_div(d > 0 ? d : 1, RS_TILE);
    size_t o = 0;
    keys0 = o; o += align256(4 * (size_t)d);
    keys1 = o; o += align256(4 * (size_t)d);
    vals0 = o; o += align256(4 * (size_t)d);
    vals1 = o; o += align256(4 * (size_t)d);
    hist = o; o += align256(4 * (size_t)RS_RADIX * nb_rs);
    gtot = o; o += align256(4 * (size_t)RS_RADIX * MAX_TILE_PASSES);
    total = o;
  }
};

template <typename T>
static T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(base) + off);
}

// Runs `passes` 8-bit LSD passes starting at bit 0 over (keys, vals); the
// last pass writes its values to vals_final (and its keys to keys_final if
// not NULL).  Buffers k0/v0 hold the input; k1/v1 are scratch.
static int radix_sort(uint32_t* k0, int32_t* v0, uint32_t* k1, int32_t* v1, int64_t n, int passes,
                      uint32_t* hist, uint32_t* gtot, int nb, uint32_t* keys_final,
                      int32_t* vals_final, cudaStream_t s) {
  if (cudaMemsetAsync(gtot, 0, sizeof(uint32_t) * RS_RADIX * passes, s) != cudaSuccess)
    return set_error(GS_ERR_CUDA, "cudaMemsetAsync failed");
  uint32_t* kin = k0;
  int32_t* vin = v0;
  uint32_t* kout = k1;
  int32_t* vout = v1;
  for (int p = 0; p < passes; ++p) {
    const int shift = 8 * p;
    const bool last = p == passes - 1;
    uint32_t* gt = gtot + RS_RADIX * p;
    k_rs_upsweep<<<nb, RS_THREADS, 0, s>>>(kin, n, shift, hist, gt, nb);
    k_rs_scan<<<RS_RADIX, RS_THREADS, 0, s>>>(hist, gt, nb);
    uint32_t* ko = last ? keys_final : kout;
    int32_t* vo = last ? vals_final : vout;
    if (ko)
      k_rs_downsweep<true><<<nb, RS_THREADS, 0, s>>>(kin, vin, ko, vo, n, shift, hist, nb);
    else
      k_rs_downsweep<false><<<nb, RS_THREADS, 0, s>>>(kin, vin, nullptr, vo, n, shift, hist, nb);
    if (int e = check_launch("radix pass", 3)) return e;
    // The next pass reads what this one wrote.
    std::swap(kin, kout);
    std::swap(vin, vout);
  }
  return GS_OK;
}

static int tile_bits(int num_tiles) {
  int b = 0;
  while ((1ll << b) < num_tiles) ++b;
  return b;
}

}  // namespace gs

using namespace gs;

static int bin_end_impl(const float* means2d, const float* radii, const float* conics, int64_t n, int64_t d, int width,
               int height, void* ws_n, size_t ws_n_bytes, void* ws_d, size_t ws_d_bytes,
               int32_t* sorted_ids, int32_t* tile_ranges, void* stream) {
  clear_error();
  cudaStream_t s = as_stream(stream);
  if (width <= 0 || height <= 0) return set_error(GS_ERR_INVALID_ARG, "image size must be positive");
  if (d < 0 || d > INT32_MAX)
    return set_error(GS_ERR_CAPACITY, "duplicate count %lld exceeds int32 range", (long long)d);
  const int tiles_x = (int)ceil_div(width, GS_TILE), tiles_y = (int)ceil_div(height, GS_TILE);
  const int num_tiles = tiles_x * tiles_y;
  if (!tile_ranges) return set_error(GS_ERR_INVALID_ARG, "tile_ranges is NULL");
  if (cudaMemsetAsync(tile_ranges, 0, sizeof(int32_t) * 2 * (size_t)num_tiles, s) != cudaSuccess)
    return set_error(GS_ERR_CUDA, "cudaMemsetAsync failed");
  if (d == 0 || n == 0) return GS_OK;
  const NLayout L(n);
  const DLayout M(d);
  if (!ws_n || ws_n_bytes < L.total)
    return set_error(GS_ERR_CAPACITY, "workspace_n too small: %zu < %zu", ws_n_bytes, L.total);
  if (!ws_d || ws_d_bytes < M.total)
    return set_error(GS_ERR_CAPACITY, "workspace_d too small: %zu < %zu", ws_d_bytes, M.total);
  if (!means2d || !radii || !sorted_ids) return set_error(GS_ERR_INVALID_ARG, "gs_bin_end: NULL pointer");
  const int32_t* perm = at<int32_t>(ws_n, L.vals0);
  const uint32_t* offsets = at<uint32_t>(ws_n, L.offsets);
  uint32_t* tk0 = at<uint32_t>(ws_d, M.keys0);
  uint32_t* tk1 = at<uint32_t>(ws_d, M.keys1);
  int32_t* tv0 = at<int32_t>(ws_d, M.vals0);
  int32_t* tv1 = at<int32_t>(ws_d, M.vals1);
  if (conics)
    k_duplicate<true><<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(
        means2d, radii, conics, perm, offsets, n, d, width, height, tiles_x, tiles_y, tk0, tv0);
  else
    k_duplicate<false><<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(
        means2d, radii, nullptr, perm, offsets, n, d, width, height, tiles_x, tiles_y, tk0, tv0);
  if (int e = check_launch("k_duplicate")) return e;
  const int bits = tile_bits(num_tiles);
  const int passes = bits == 0 ? 1 : (bits + 7) / 8;
  // Final keys land in whichever key buffer the last pass does not read.
  uint32_t* kfinal = (passes % 2 == 1) ? tk1 : tk0;
  int e = radix_sort(tk0, tv0, tk1, tv1, d, passes, at<uint32_t>(ws_d, M.hist),
                     at<uint32_t>(ws_d, M.gtot), M.nb_rs, kfinal, sorted_ids, s);
  if (e) return e;
  k_tile_ranges<<<(unsigned)ceil_div(d, 256), 256, 0, s>>>(kfinal, d, tile_ranges);
  return check_launch("k_tile_ranges");
}


extern "C" {

size_t gs_bin_workspace_n_bytes(int64_t n) { return NLayout(n < 0 ? 0 : n).total; }

int gs_bin_total(const int32_t* tiles_touched, int64_t n, int64_t* d_total, void* stream) {
  clear_error();
  cudaStream_t s = as_stream(stream);
  if (!d_total) return set_error(GS_ERR_INVALID_ARG, "d_total is NULL");
  if (n < 0) return set_error(GS_ERR_INVALID_ARG, "n must be >= 0");
  if (cudaMemsetAsync(d_total, 0, sizeof(int64_t), s) != cudaSuccess)
    return set_error(GS_ERR_CUDA, "cudaMemsetAsync failed");
  if (n == 0) return GS_OK;
  if (!tiles_touched) return set_error(GS_ERR_INVALID_ARG, "tiles_touched is NULL");
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 4);
  k_count_total<<<grid, 256, 0, s>>>(tiles_touched, n, reinterpret_cast<unsigned long long*>(d_total));
  return check_launch("k_count_total");
}
size_t gs_bin_workspace_d_bytes(int64_t d) { return DLayout(d < 0 ? 0 : d).total; }

int gs_bin_begin(const float* depths, const int32_t* tiles_touched, int64_t n, void* ws_n,
                 size_t ws_n_bytes, int64_t* d_total, void* stream) {
  clear_error();
  cudaStream_t s = as_stream(stream);
  if (n < 0 || n > INT32_MAX) return set_error(GS_ERR_INVALID_ARG, "n out of range: %lld", (long long)n);
  if (!d_total) return set_error(GS_ERR_INVALID_ARG, "d_total is NULL");
  if (n == 0) {
    if (cudaMemsetAsync(d_total, 0, sizeof(int64_t), s) != cudaSuccess)
      return set_error(GS_ERR_CUDA, "cudaMemsetAsync failed");
    return GS_OK;
  }
  const NLayout L(n);
  if (!ws_n || ws_n_bytes < L.total)
    return set_error(GS_ERR_CAPACITY, "workspace_n too small: %zu < %zu", ws_n_bytes, L.total);
  if (!depths || !tiles_touched) return set_error(GS_ERR_INVALID_ARG, "gs_bin_begin: NULL pointer");
  uint32_t* k0 = at<uint32_t>(ws_n, L.keys0);
  uint32_t* k1 = at<uint32_t>(ws_n, L.keys1);
  int32_t* v0 = at<int32_t>(ws_n, L.vals0);
  int32_t* v1 = at<int32_t>(ws_n, L.vals1);
  k_depth_keys<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(depths, tiles_touched, n, k0, v0);
  // Pass p writes buffer (p + 1) % 2; with an even pass count the sorted
  // permutation lands in v0 (the last pass reads v1).  Keys are dropped.
  static_assert(DEPTH_PASSES % 2 == 0, "depth permutation buffer assumes an even pass count");
  int e = radix_sort(k0, v0, k1, v1, n, DEPTH_PASSES, at<uint32_t>(ws_n, L.hist),
                     at<uint32_t>(ws_n, L.gtot), L.nb_rs, nullptr, v0, s);
  if (e) return e;
  const int32_t* perm = v0;
  unsigned long long* bsum = at<unsigned long long>(ws_n, L.bsum);
  uint32_t* offsets = at<uint32_t>(ws_n, L.offsets);
  k_scan_reduce<<<L.nb_sc, SC_THREADS, 0, s>>>(tiles_touched, perm, n, bsum);
  k_scan_bsums<<<1, SB_THREADS, 0, s>>>(bsum, L.nb_sc, d_total);
  k_scan_down<<<L.nb_sc, SC_THREADS, 0, s>>>(tiles_touched, perm, n, bsum, offsets);
  return check_launch("gs_bin_begin", 4);  // k_depth_keys + 3 scan kernels
}

int gs_bin_end(const float* means2d, const float* radii, int64_t n, int64_t d, int width,
               int height, void* ws_n, size_t ws_n_bytes, void* ws_d, size_t ws_d_bytes,
               int32_t* sorted_ids, int32_t* tile_ranges, void* stream) {
  return bin_end_impl(means2d, radii, nullptr, n, d, width, height, ws_n, ws_n_bytes, ws_d, ws_d_bytes,
                      sorted_ids, tile_ranges, stream);
}

int gs_bin_end_refined(const float* means2d, const float* radii, const float* conics, int64_t n,
                       int64_t d, int width, int height, void* ws_n, size_t ws_n_bytes, void* ws_d,
                       size_t ws_d_bytes, int32_t* sorted_ids, int32_t* tile_ranges, void* stream) {
  if (!conics && n > 0) return set_error(GS_ERR_INVALID_ARG, "gs_bin_end_refined: conics is NULL");
  return bin_end_impl(means2d, radii, conics, n, d, width, height, ws_n, ws_n_bytes, ws_d, ws_d_bytes,
                      sorted_ids, tile_ranges, stream);
}

int gs_tile_counts_refined(const float* means2d, const float* radii, const float* conics, int64_t n,
                           int width, int height, int32_t* tiles_touched, void* stream) {
  clear_error();
  if (width <= 0 || height <= 0) return set_error(GS_ERR_INVALID_ARG, "image size must be positive");
  if (n <= 0) return GS_OK;
  if (!means2d || !radii || !conics || !tiles_touched)
    return set_error(GS_ERR_INVALID_ARG, "gs_tile_counts_refined: NULL pointer");
  if (!aligned(means2d, 8)) return set_error(GS_ERR_INVALID_ARG, "means2d must be 8-byte aligned");
  const int tx = (int)ceil_div(width, GS_TILE), ty = (int)ceil_div(height, GS_TILE);
  k_tile_counts_refined<<<(unsigned)ceil_div(n, 256), 256, 0, as_stream(stream)>>>(
      means2d, radii, conics, n, width, height, tx, ty, tiles_touched);
  return check_launch("k_tile_counts_refined");
}

}  // extern "C"
