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
// Between 1 and 2, one chained-scan kernel turns the tiles-touched counts
// (in depth order) into output offsets and D; 2 runs one warp per equal
// chunk of the D outputs; 3 ends with the per-tile ranges.
#include <algorithm>
#include <utility>

#include "gs_common.cuh"

namespace gs {

// ------------------------------------------------------------- radix passes
// One kernel per 8-bit pass ("onesweep" structure):
//   * the digit histograms of every pass come from the kernel that produces
//     the keys (k_depth_keys, k_duplicate), so no pass re-reads its input to
//     count;
//   * a block takes the next partition of OS_TILE keys in launch order
//     (atomic counter), ranks its keys stably by digit (warp multisplit by
//     ballots), publishes its per-digit counts and finds the counts of all
//     earlier partitions by a decoupled look-back with pointer jumping over
//     a per-partition status array;
//   * the keys are reordered by digit in shared memory and written out in
//     digit runs, so consecutive threads store to consecutive addresses.
// A partition only waits on partitions with smaller indices, which were
// taken by blocks that are already running, so every wait ends; each wait is
// still bounded (g_wait_limit polls), after which the block counts the
// failure in g_wait_failures, sets its stage's bit in the call's status word
// (BinFail) and writes nothing.  Every later kernel that would index memory
// with values the failed stage should have produced reads the status word
// first and does nothing when a bit it depends on is set; the tile ranges
// then stay all-empty, so a compositor launched afterwards reads no ids.
//
// Status words: pass + 1 (8 bits) | reach (24 bits) | count (32 bits): the
// count of one digit over the `reach` partitions ending at this one.  One
// zeroed status array serves every pass of a sort: words of earlier passes
// read as "not ready".
constexpr int OS_THREADS = 256;
constexpr int OS_WARPS = OS_THREADS / 32;
constexpr int OS_ITEMS = 12;
constexpr int OS_TILE = OS_THREADS * OS_ITEMS;  // keys per partition
constexpr int OS_RADIX = 256;
constexpr int DEPTH_PASSES = 4;
constexpr int MAX_TILE_PASSES = 4;
constexpr int kLookbackSpins = 1 << 22;

// Polls a look-back may make before it gives up (per device; set by
// gs_set_wait_limit, for tests).  With 0, every look-back that has to read
// an earlier partition's word gives up before its first read.
__device__ int g_wait_limit = kLookbackSpins;
__device__ unsigned long long g_wait_failures;

// Bits of the per-call status word (in workspace_n, zeroed by gs_bin_begin).
enum BinFail : uint32_t { kFailDepthSort = 1u, kFailScan = 2u, kFailTileSort = 4u };

__device__ __forceinline__ uint32_t ld_status(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Lanes of the warp holding the same 9-bit value as this lane (values
// 0..256; 256 marks "no key"): nine ballots, one per bit (a warp multisplit;
// __match_any_sync takes hundreds of cycles when most lanes differ).
__device__ __forceinline__ unsigned digit_peers(uint32_t d) {
  unsigned m = 0xffffffffu;
#pragma unroll
  for (int b = 0; b < 9; ++b) {
    const unsigned bal = __ballot_sync(0xffffffffu, (d >> b) & 1u);
    m &= ((d >> b) & 1u) ? bal : ~bal;
  }
  return m;
}

// Exclusive scan of one value per thread over a 256-thread block.
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
  for (int w = 0; w < 256 / 32; ++w) {
    const uint32_t ws = warp_sums[w];
    if (w < warp) pre += ws;
    tot += ws;
  }
  __syncthreads();
  total = tot;
  return pre + s - x;
}

// Increment of h[digit] by every lane of a full warp (digit 256 = no key):
// one shared atomic when all lanes share the digit (the common case for
// high digits), else one per lane.
__device__ __forceinline__ void count_digit(uint32_t* h, uint32_t digit) {
  const uint32_t d0 = __shfl_sync(0xffffffffu, digit, 0);
  if (__all_sync(0xffffffffu, digit == d0)) {
    if ((threadIdx.x & 31) == 0 && d0 < 256u) atomicAdd(&h[d0], 32u);
  } else if (digit < 256u) {
    atomicAdd(&h[digit], 1u);
  }
}

// Adds the per-block shared histograms h[passes][256] into ghist.
__device__ __forceinline__ void flush_hist(const uint32_t (*h)[OS_RADIX], int passes,
                                           uint32_t* __restrict__ ghist) {
  for (int i = threadIdx.x; i < passes * OS_RADIX; i += blockDim.x) {
    const uint32_t c = h[i / OS_RADIX][i % OS_RADIX];
    if (c) atomicAdd(ghist + i, c);
  }
}

template <bool KEYS_OUT>
__global__ void __launch_bounds__(OS_THREADS, 4)
k_onesweep(const uint32_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
           uint32_t* __restrict__ keys_out, int32_t* __restrict__ vals_out, int64_t n, int pass,
           const uint32_t* __restrict__ ghist, unsigned long long* __restrict__ status,
           uint32_t* __restrict__ part_ctr, uint32_t* __restrict__ fail, uint32_t fail_bit) {
  __shared__ uint32_t wcnt[OS_WARPS][OS_RADIX];
  __shared__ uint32_t s_keys[OS_TILE];
  __shared__ int32_t s_vals[OS_TILE];
  __shared__ uint32_t s_lstart[OS_RADIX];  // first local index of each digit
  __shared__ uint32_t s_base[OS_RADIX];    // global index of local index 0, per digit
  __shared__ uint32_t warp_sums[OS_WARPS];
  __shared__ int s_part, s_fail;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int shift = 8 * pass;
  if (threadIdx.x == 0) {
    s_part = (int)atomicAdd(part_ctr, 1u);
    s_fail = 0;
  }
  for (int i = threadIdx.x; i < OS_WARPS * OS_RADIX; i += OS_THREADS) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int part = s_part;
  const int64_t first = (int64_t)part * OS_TILE;
  const int nvalid = (int)(n - first < OS_TILE ? n - first : OS_TILE);

  // Stable ranks within the warp's OS_ITEMS x 32 keys (index order), per digit.
  const int64_t seg = first + warp * (32 * OS_ITEMS);
  const unsigned lt = (1u << lane) - 1u;
  uint32_t k[OS_ITEMS];
  int32_t v[OS_ITEMS];
  uint32_t rank[OS_ITEMS];
#pragma unroll
  for (int it = 0; it < OS_ITEMS; ++it) {
    const int64_t idx = seg + it * 32 + lane;
    const bool valid = idx < n;
    k[it] = valid ? __ldg(keys_in + idx) : 0u;
    v[it] = valid ? __ldg(vals_in + idx) : 0;
  }
  // Peer masks of all items first (independent ballots), then the running
  // per-warp digit counters in shared memory, item by item.
  unsigned peers[OS_ITEMS];
#pragma unroll
  for (int it = 0; it < OS_ITEMS; ++it) {
    const bool valid = seg + it * 32 + lane < n;
    peers[it] = digit_peers(valid ? ((k[it] >> shift) & 255u) : 256u);
  }
#pragma unroll
  for (int it = 0; it < OS_ITEMS; ++it) {
    const bool valid = seg + it * 32 + lane < n;
    const uint32_t d = (k[it] >> shift) & 255u;
    const uint32_t cnt = valid ? wcnt[warp][d] : 0u;
    __syncwarp();
    if (valid && (peers[it] & lt) == 0u) wcnt[warp][d] = cnt + __popc(peers[it]);
    __syncwarp();
    rank[it] = cnt + __popc(peers[it] & lt);
  }
  __syncthreads();

  // Per digit (one thread each): block count, earlier warps' counts.
  const int d = threadIdx.x;
  uint32_t cnt_d = 0;
#pragma unroll
  for (int w = 0; w < OS_WARPS; ++w) {
    const uint32_t t = wcnt[w][d];
    wcnt[w][d] = cnt_d;
    cnt_d += t;
  }
  unsigned long long* my = status + (int64_t)part * OS_RADIX + d;
  const unsigned long long tag = (unsigned long long)(pass + 1) << 56;
  st_relaxed_u64(my, tag | (1ull << 32) | cnt_d);

  uint32_t tot;
  const uint32_t lstart = block_exclusive_scan(cnt_d, warp_sums, tot);
  const uint32_t gpre = block_exclusive_scan(ghist[d], warp_sums, tot);
  s_lstart[d] = lstart;

  // Look-back by pointer jumping: the word of partition j holds the count of
  // digit d over partitions [j - reach + 1, j]; a reader adds it and jumps
  // to j - reach, and republishes its own, longer range after every step,
  // so ranges roughly double per step and every block is done after about
  // log2(partitions) reads.
  uint32_t acc = cnt_d;  // count over [cur + 1, part]
  int64_t cur = part - 1;
  int spins = 0;
  const int limit = g_wait_limit;
  while (cur >= 0) {
    if (spins >= limit) {
      s_fail = 1;
      break;
    }
    const unsigned long long w = ld_relaxed_u64(status + cur * OS_RADIX + d);
    if ((w & (0xFFull << 56)) != tag) {  // not yet written in this pass
      ++spins;
      __nanosleep(32);
      continue;
    }
    acc += (uint32_t)w;
    cur -= (int64_t)((w >> 32) & 0xFFFFFFull);
    st_relaxed_u64(my, tag | ((unsigned long long)(part - cur) << 32) | acc);
  }
  const uint32_t excl = acc - cnt_d;
  s_base[d] = gpre + excl - lstart;
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) {
      atomicAdd(&g_wait_failures, 1ull);
      atomicOr(fail, fail_bit);
    }
    return;
  }

  // Reorder by digit in shared memory, then write digit runs.
#pragma unroll
  for (int it = 0; it < OS_ITEMS; ++it) {
    if (seg + it * 32 + lane < n) {
      const uint32_t dd = (k[it] >> shift) & 255u;
      const uint32_t li = s_lstart[dd] + wcnt[warp][dd] + rank[it];
      s_keys[li] = k[it];
      s_vals[li] = v[it];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nvalid; i += OS_THREADS) {
    const uint32_t key = s_keys[i];
    const uint32_t pos = s_base[(key >> shift) & 255u] + (uint32_t)i;
    if ((int64_t)pos >= n) continue;  // only if the histograms disagree with the keys (inconsistent inputs)
    if (KEYS_OUT) keys_out[pos] = key;
    vals_out[pos] = s_vals[i];
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

// Depth keys (float bits; 0xFFFFFFFF for Gaussians touching no tile),
// identity values, and the digit histograms of all DEPTH_PASSES passes.
__global__ void __launch_bounds__(256)
k_depth_keys(const float* __restrict__ depths, const int32_t* __restrict__ counts, int64_t n,
             uint32_t* __restrict__ keys, int32_t* __restrict__ vals, uint32_t* __restrict__ ghist) {
  __shared__ uint32_t h[DEPTH_PASSES][OS_RADIX];
  for (int i = threadIdx.x; i < DEPTH_PASSES * OS_RADIX; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  // whole warps iterate together so the digit counts can be warp-aggregated
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x; b < n; b += stride) {
    const int64_t i = b + threadIdx.x;
    const bool valid = i < n;
    uint32_t key = 0;
    if (valid) {
      key = counts[i] > 0 ? gs_float_to_bits(depths[i]) : 0xFFFFFFFFu;
      keys[i] = key;
      vals[i] = (int32_t)i;
    }
#pragma unroll
    for (int p = 0; p < DEPTH_PASSES; ++p) count_digit(h[p], valid ? (key >> (8 * p)) & 255u : 256u);
  }
  __syncthreads();
  flush_hist(h, DEPTH_PASSES, ghist);
}

// Device-wide exclusive scan of counts[perm[i]] (int32) in one kernel: a
// block takes the next SC_TILE-element partition in launch order, scans it,
// and finds the total of all earlier partitions by the same pointer-jumping
// look-back as the radix passes (one word per partition: tag | reach | sum;
// sums stay below 2^31 because D does).  The last partition writes D.
constexpr int SC_THREADS = 256, SC_ITEMS = 16, SC_TILE = SC_THREADS * SC_ITEMS;

__global__ void __launch_bounds__(SC_THREADS)
k_scan_chained(const int32_t* __restrict__ counts, const int32_t* __restrict__ perm, int64_t n, int nb,
               unsigned long long* __restrict__ status, uint32_t* __restrict__ part_ctr,
               uint32_t* __restrict__ offsets, int64_t* __restrict__ total_out, uint32_t* __restrict__ fail) {
  __shared__ uint32_t warp_sums[SC_THREADS / 32];
  __shared__ int s_part, s_fail;
  __shared__ uint32_t s_excl;
  // perm comes from the depth sort: if one of its look-backs gave up, perm
  // may hold stale values and must not index counts.
  if (ld_status(fail) & kFailDepthSort) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *total_out = 0;
    return;
  }
  if (threadIdx.x == 0) {
    s_part = (int)atomicAdd(part_ctr, 1u);
    s_fail = 0;
  }
  __syncthreads();
  const int part = s_part;
  const int64_t base = (int64_t)part * SC_TILE + (int64_t)threadIdx.x * SC_ITEMS;
  uint32_t c[SC_ITEMS];
  uint32_t local = 0;
#pragma unroll
  for (int j = 0; j < SC_ITEMS; ++j) {
    const int64_t idx = base + j;
    c[j] = idx < n ? (uint32_t)counts[perm[idx]] : 0u;
    local += c[j];
  }
  uint32_t tot;
  const uint32_t pre = block_exclusive_scan(local, warp_sums, tot);
  if (threadIdx.x == 0) {
    const unsigned long long tag = 1ull << 56;
    unsigned long long* my = status + part;
    st_relaxed_u64(my, tag | (1ull << 32) | tot);
    uint32_t acc = tot;  // sum over partitions [cur + 1, part]
    int64_t cur = part - 1;
    int spins = 0;
    const int limit = g_wait_limit;
    while (cur >= 0) {
      if (spins >= limit) {
        s_fail = 1;
        break;
      }
      const unsigned long long w = ld_relaxed_u64(status + cur);
      if ((w & (0xFFull << 56)) != tag) {
        ++spins;
        __nanosleep(32);
        continue;
      }
      acc += (uint32_t)w;
      cur -= (int64_t)((w >> 32) & 0xFFFFFFull);
      st_relaxed_u64(my, tag | ((unsigned long long)(part - cur) << 32) | acc);
    }
    s_excl = acc - tot;
    if (part == nb - 1) *total_out = s_fail ? 0 : (int64_t)acc;
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) {
      atomicAdd(&g_wait_failures, 1ull);
      atomicOr(fail, (uint32_t)kFailScan);
    }
    return;
  }
  uint32_t run = s_excl + pre;
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

// Duplication (tiles.py:77-89): (tile id, Gaussian id) for every tile of
// each Gaussian's rectangle, row-major, Gaussians in depth order.  The D
// outputs are split into equal chunks of kDupChunk, one warp each, so a
// Gaussian covering thousands of tiles is spread over many warps.  A warp
// finds the Gaussian owning its first output by a 32-way search of the
// offsets (an exclusive scan in depth order, so the owner of entry q is the
// last Gaussian whose offset is <= q), then walks windows of 32 consecutive
// Gaussians: entry q of a window belongs to the last lane whose start is
// <= q (a binary search over the lanes' starts by shuffles) and is tile
// k = q - start of that lane's rectangle.  Consecutive lanes store
// consecutive entries.  The digit counts of the `passes` tile-sort passes
// are taken on the way.
constexpr int kDupChunk = 1024;

template <bool HIST>
__global__ void __launch_bounds__(256)
k_duplicate(const float* __restrict__ means2d, const float* __restrict__ radii,
            const int32_t* __restrict__ perm, const uint32_t* __restrict__ offsets, int64_t n,
            int64_t d, int width, int height, int tiles_x, int tiles_y, uint32_t* __restrict__ tkeys,
            int32_t* __restrict__ tvals, int passes, uint32_t* __restrict__ ghist,
            const uint32_t* __restrict__ fail) {
  __shared__ uint32_t h[MAX_TILE_PASSES][OS_RADIX];
  // perm and offsets come from gs_bin_begin; skip if either stage gave up.
  if (ld_status(fail) & (kFailDepthSort | kFailScan)) return;
  if (HIST) {
    for (int i = threadIdx.x; i < MAX_TILE_PASSES * OS_RADIX; i += blockDim.x) (&h[0][0])[i] = 0;
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t q_begin = wid * kDupChunk;
  if (q_begin < d) {
    const int64_t q_end = min(d, q_begin + kDupChunk);
    // owner of q_begin: last i with offsets[i] <= q_begin (offsets[0] = 0)
    int64_t lo = 0, hi = n;
    while (hi - lo > 32) {
      const int64_t step = (hi - lo + 31) / 32;
      const int64_t pidx = lo + lane * step;
      const bool le = pidx < hi && (int64_t)offsets[pidx] <= q_begin;
      const int last = 31 - __clz(__ballot_sync(0xffffffffu, le));  // lane 0 always qualifies
      lo += last * step;
      hi = min(hi, lo + step);
    }
    {
      const int64_t pidx = lo + lane;
      const bool le = pidx < hi && (int64_t)offsets[pidx] <= q_begin;
      lo += 31 - __clz(__ballot_sync(0xffffffffu, le));
    }
    int64_t iw = lo;  // first Gaussian of the current window
    int64_t q = q_begin;
    while (q < q_end && iw < n) {
      const int64_t i = iw + lane;
      int x0 = 0, y0 = 0, x1 = -1, y1 = -1;
      int32_t g = 0;
      int64_t start = INT64_MAX, end = 0;
      if (i < n) {
        g = perm[i];
        start = offsets[i];
        end = start;
        if (gauss_rect(reinterpret_cast<const float2*>(means2d)[g], radii[g], width, height, tiles_x,
                       tiles_y, x0, y0, x1, y1))
          end = start + (int64_t)(x1 - x0 + 1) * (y1 - y0 + 1);
      }
      const int wd = x1 - x0 + 1;
      int64_t wend = end;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) wend = max(wend, __shfl_xor_sync(0xffffffffu, wend, o));
      const int64_t stop = min(q_end, wend);
      for (int64_t qb = q; qb < stop; qb += 32) {
        const int64_t qq = qb + lane;
        int j = 0;
#pragma unroll
        for (int st = 16; st > 0; st >>= 1) {
          const int64_t r = __shfl_sync(0xffffffffu, start, j + st);
          if (r <= qq) j += st;
        }
        const int k = (int)(qq - __shfl_sync(0xffffffffu, start, j));
        const int wj = __shfl_sync(0xffffffffu, wd, j);
        const int x0j = __shfl_sync(0xffffffffu, x0, j), y0j = __shfl_sync(0xffffffffu, y0, j);
        const int32_t gj = __shfl_sync(0xffffffffu, g, j);
        const bool act = qq < stop;
        uint32_t key = 0;
        if (act) {
          key = (uint32_t)((y0j + k / wj) * tiles_x + x0j + k % wj);
          tkeys[qq] = key;
          tvals[qq] = gj;
        }
        if (HIST)
          for (int p = 0; p < passes; ++p) count_digit(h[p], act ? (key >> (8 * p)) & 255u : 256u);
      }
      if (stop > q) q = stop;
      iw += 32;
    }
  }
  if (HIST) {
    __syncthreads();
    flush_hist(h, passes, ghist);
  }
}

// Refined duplication (tiles.py:141-163): one thread per Gaussian in depth
// order writes the tiles the refinement keeps; the digit counts follow in
// k_tile_hist.
__global__ void k_duplicate_refined(const float* __restrict__ means2d, const float* __restrict__ radii,
                                    const float* __restrict__ conics, const int32_t* __restrict__ perm,
                                    const uint32_t* __restrict__ offsets, int64_t n, int64_t d, int width,
                                    int height, int tiles_x, int tiles_y, uint32_t* __restrict__ tkeys,
                                    int32_t* __restrict__ tvals, const uint32_t* __restrict__ fail) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (ld_status(fail) & (kFailDepthSort | kFailScan)) return;
  const int32_t g = perm[i];
  const float2 m = reinterpret_cast<const float2*>(means2d)[g];
  int x0, y0, x1, y1;
  if (!gauss_rect(m, radii[g], width, height, tiles_x, tiles_y, x0, y0, x1, y1)) return;
  uint32_t o = offsets[i];
  for (int ty = y0; ty <= y1; ++ty)
    for (int tx = x0; tx <= x1; ++tx) {
      if (!refine_keep(conics + 3 * (int64_t)g, m.x, m.y, tx, ty, width, height)) continue;
      if ((int64_t)o >= d) return;  // never past the caller's D (counts are recomputed exactly)
      tkeys[o] = (uint32_t)(ty * tiles_x + tx);
      tvals[o] = g;
      ++o;
    }
}

// Digit counts of the tile-sort passes over written keys.
__global__ void __launch_bounds__(256)
k_tile_hist(const uint32_t* __restrict__ tkeys, int64_t d, int passes, uint32_t* __restrict__ ghist) {
  __shared__ uint32_t h[MAX_TILE_PASSES][OS_RADIX];
  for (int i = threadIdx.x; i < MAX_TILE_PASSES * OS_RADIX; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x; b < d; b += stride) {
    const int64_t i = b + threadIdx.x;
    const uint32_t key = i < d ? tkeys[i] : 0u;
    for (int p = 0; p < passes; ++p) count_digit(h[p], i < d ? (key >> (8 * p)) & 255u : 256u);
  }
  __syncthreads();
  flush_hist(h, passes, ghist);
}

// [start, end) of every non-empty tile from the tile-sorted keys; empty
// tiles keep the zero-initialised [0, 0) (tiles.py:175-180).
__global__ void k_tile_ranges(const uint32_t* __restrict__ tkeys, int64_t d, int num_tiles,
                              int32_t* __restrict__ ranges, const uint32_t* __restrict__ fail) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d) return;
  // Any stage that gave up: every tile keeps the empty range [0, 0).
  if (ld_status(fail) != 0u) return;
  const uint32_t t = tkeys[i];
  if (t >= (uint32_t)num_tiles) return;  // inconsistent inputs only
  if (i == 0 || tkeys[i - 1] != t) ranges[2 * (int64_t)t] = (int32_t)i;
  if (i == d - 1 || tkeys[i + 1] != t) ranges[2 * (int64_t)t + 1] = (int32_t)(i + 1);
}

// --------------------------------------------------------- workspace layout
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Sort bookkeeping, zeroed by one memset per sort: digit histograms of
// every pass, the partition counters, the look-back status words.
struct SortState {
  size_t ghist, ctr, status, end;
  int nb;
  SortState(int64_t n, int passes, size_t o) {
    nb = (int)ceil_div(n > 0 ? n : 1, OS_TILE);
    ghist = o; o += 4 * (size_t)OS_RADIX * passes;
    ctr = o; o += align256(4 * (size_t)passes);
    status = o; o += align256(8 * (size_t)OS_RADIX * nb);
    end = o;
  }
};

struct NLayout {
  size_t keys0, keys1, vals0, vals1, offsets, scan_status, scan_ctr, fail, total;
  int nb_sc;
  SortState st;
  NLayout(int64_t n) : st(n, DEPTH_PASSES, 0) {
    nb_sc = (int)ceil_div(n > 0 ? n : 1, SC_TILE);
    size_t o = 0;
    keys0 = o; o += align256(4 * (size_t)n);
    keys1 = o; o += align256(4 * (size_t)n);
    vals0 = o; o += align256(4 * (size_t)n);
    vals1 = o; o += align256(4 * (size_t)n);
    offsets = o; o += align256(4 * (size_t)n);
    st = SortState(n, DEPTH_PASSES, o);
    o = st.end;  // the scan's look-back words follow, inside the same zeroed range
    scan_status = o; o += 8 * (size_t)nb_sc;
    scan_ctr = o; o += 128;
    fail = o; o += 128;  // BinFail status word of this call
    total = o;
  }
};

struct DLayout {
  size_t keys0, keys1, vals0, vals1, total;
  SortState st;
  DLayout(int64_t d) : st(d, MAX_TILE_PASSES, 0) {
    size_t o = 0;
    keys0 = o; o += align256(4 * (size_t)d);
    keys1 = o; o += align256(4 * (size_t)d);
    vals0 = o; o += align256(4 * (size_t)d);
    vals1 = o; o += align256(4 * (size_t)d);
    st = SortState(d, MAX_TILE_PASSES, o);
    total = st.end;
  }
};

template <typename T>
static T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(base) + off);
}

static int zero_range(void* base, size_t begin, size_t end, cudaStream_t s) {
  if (cudaMemsetAsync(at<char>(base, begin), 0, end - begin, s) != cudaSuccess)
    return set_error(GS_ERR_CUDA, "cudaMemsetAsync failed");
  return GS_OK;
}

// Runs `passes` 8-bit LSD passes starting at bit 0 over (keys, vals), whose
// digit histograms are already in the state; the last pass writes its values
// to vals_final (and its keys to keys_final if not NULL).  Buffers k0/v0
// hold the input; k1/v1 are scratch.
static int radix_sort(uint32_t* k0, int32_t* v0, uint32_t* k1, int32_t* v1, int64_t n, int passes,
                      void* base, const SortState& st, uint32_t* keys_final, int32_t* vals_final,
                      uint32_t* fail, uint32_t fail_bit, cudaStream_t s) {
  const uint32_t* ghist = at<uint32_t>(base, st.ghist);
  uint32_t* ctr = at<uint32_t>(base, st.ctr);
  unsigned long long* status = at<unsigned long long>(base, st.status);
  uint32_t* kin = k0;
  int32_t* vin = v0;
  uint32_t* kout = k1;
  int32_t* vout = v1;
  for (int p = 0; p < passes; ++p) {
    const bool last = p == passes - 1;
    uint32_t* ko = last ? keys_final : kout;
    int32_t* vo = last ? vals_final : vout;
    if (ko)
      k_onesweep<true><<<st.nb, OS_THREADS, 0, s>>>(kin, vin, ko, vo, n, p, ghist + OS_RADIX * p, status,
                                                     ctr + p, fail, fail_bit);
    else
      k_onesweep<false><<<st.nb, OS_THREADS, 0, s>>>(kin, vin, nullptr, vo, n, p, ghist + OS_RADIX * p,
                                                      status, ctr + p, fail, fail_bit);
    if (int e = check_launch("k_onesweep")) return e;
    // The next pass reads what this one wrote.
    std::swap(kin, kout);
    std::swap(vin, vout);
  }
  return GS_OK;
}

int binning_set_wait_limit(int polls) {
  return (int)cudaMemcpyToSymbol(g_wait_limit, &polls, sizeof(polls));
}

int binning_wait_failures(unsigned long long* out, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_wait_failures, sizeof(*out));
  if (e == cudaSuccess && reset) {
    const unsigned long long z = 0;
    e = cudaMemcpyToSymbol(g_wait_failures, &z, sizeof(z));
  }
  return (int)e;
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
  uint32_t* fail = at<uint32_t>(ws_n, L.fail);
  uint32_t* tk0 = at<uint32_t>(ws_d, M.keys0);
  uint32_t* tk1 = at<uint32_t>(ws_d, M.keys1);
  int32_t* tv0 = at<int32_t>(ws_d, M.vals0);
  int32_t* tv1 = at<int32_t>(ws_d, M.vals1);
  const int bits = tile_bits(num_tiles);
  const int passes = bits == 0 ? 1 : (bits + 7) / 8;
  if (passes > MAX_TILE_PASSES) return set_error(GS_ERR_CAPACITY, "too many tiles: %d", num_tiles);
  if (int e = zero_range(ws_d, M.st.ghist, M.st.end, s)) return e;
  uint32_t* ghist = at<uint32_t>(ws_d, M.st.ghist);
  if (conics) {
    k_duplicate_refined<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(
        means2d, radii, conics, perm, offsets, n, d, width, height, tiles_x, tiles_y, tk0, tv0, fail);
    k_tile_hist<<<(unsigned)std::min<int64_t>(ceil_div(d, 256), 148 * 8), 256, 0, s>>>(tk0, d, passes, ghist);
    if (int e = check_launch("k_duplicate_refined", 2)) return e;
  } else {
    const unsigned grid = (unsigned)ceil_div(d, (int64_t)kDupChunk * 8);
    k_duplicate<true><<<grid, 256, 0, s>>>(means2d, radii, perm, offsets, n, d, width, height, tiles_x, tiles_y,
                                           tk0, tv0, passes, ghist, fail);
    if (int e = check_launch("k_duplicate")) return e;
  }
  // Final keys land in whichever key buffer the last pass does not read.
  uint32_t* kfinal = (passes % 2 == 1) ? tk1 : tk0;
  int e = radix_sort(tk0, tv0, tk1, tv1, d, passes, ws_d, M.st, kfinal, sorted_ids, fail, kFailTileSort, s);
  if (e) return e;
  k_tile_ranges<<<(unsigned)ceil_div(d, 256), 256, 0, s>>>(kfinal, d, num_tiles, tile_ranges, fail);
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
  if (int e = zero_range(ws_n, L.st.ghist, L.total, s)) return e;
  k_depth_keys<<<(unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 8), 256, 0, s>>>(
      depths, tiles_touched, n, k0, v0, at<uint32_t>(ws_n, L.st.ghist));
  if (int e0 = check_launch("k_depth_keys")) return e0;
  // Pass p writes buffer (p + 1) % 2; with an even pass count the sorted
  // permutation lands in v0 (the last pass reads v1).  Keys are dropped.
  static_assert(DEPTH_PASSES % 2 == 0, "depth permutation buffer assumes an even pass count");
  uint32_t* fail = at<uint32_t>(ws_n, L.fail);
  int e = radix_sort(k0, v0, k1, v1, n, DEPTH_PASSES, ws_n, L.st, nullptr, v0, fail, kFailDepthSort, s);
  if (e) return e;
  const int32_t* perm = v0;
  uint32_t* offsets = at<uint32_t>(ws_n, L.offsets);
  k_scan_chained<<<L.nb_sc, SC_THREADS, 0, s>>>(tiles_touched, perm, n, L.nb_sc,
                                               at<unsigned long long>(ws_n, L.scan_status),
                                               at<uint32_t>(ws_n, L.scan_ctr), offsets, d_total, fail);
  return check_launch("k_scan_chained");
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

int gs_bin_status(const void* ws_n, size_t ws_n_bytes, int64_t n, uint32_t* status_out, void* stream) {
  clear_error();
  if (!status_out) return set_error(GS_ERR_INVALID_ARG, "status_out is NULL");
  if (n < 0 || n > INT32_MAX) return set_error(GS_ERR_INVALID_ARG, "n out of range: %lld", (long long)n);
  const NLayout L(n);
  if (n == 0) {  // gs_bin_begin / gs_bin_end launch nothing for n == 0
    *status_out = 0;
    return GS_OK;
  }
  if (!ws_n || ws_n_bytes < L.total)
    return set_error(GS_ERR_CAPACITY, "workspace_n too small: %zu < %zu", ws_n_bytes, L.total);
  cudaStream_t s = as_stream(stream);
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, at<char>(const_cast<void*>(ws_n), L.fail), sizeof(v),
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return set_error(GS_ERR_CUDA, "gs_bin_status: %s", cudaGetErrorString(e));
  *status_out = v;
  if (v)
    return set_error(GS_ERR_TIMEOUT,
                     "a bounded device wait of the binning gave up (status 0x%x: %s%s%s); every tile range "
                     "was left empty",
                     v, (v & kFailDepthSort) ? "depth sort " : "", (v & kFailScan) ? "offsets scan " : "",
                     (v & kFailTileSort) ? "tile sort" : "");
  return GS_OK;
}

size_t gs_bin_status_offset(int64_t n) { return NLayout(n < 0 ? 0 : n).fail; }

}  // extern "C"
