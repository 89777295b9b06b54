// Shared host/device helpers of the sm_100a splatting library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/gsplat_b200.h"
#include "gs_math.h"

namespace gs {

// Records a message for gs_last_error() (thread-local) and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();
// Adds `n` to the process-wide count of kernels this library launched.
void note_launches(int n);

inline int check_launch(const char* what, int launches = 1) {
  note_launches(launches);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return GS_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Device counters of bounded waits that ran out, one per translation unit
// that waits (read synchronously, optionally reset; gs_wait_failures sums
// them).  Return a cudaError_t.
int binning_wait_failures(unsigned long long* out, int reset);
// Sets the poll limit of the binning look-backs on the current device.
int binning_set_wait_limit(int polls);
int preprocess_wait_failures(unsigned long long* out, int reset);

// ------------------------------------------------ bulk (TMA) copies
// One-shot shared-memory mbarrier tracking bulk global->shared copies
// (cp.async.bulk, the Blackwell/Hopper TMA engine without a tensor map;
// never the cluster-multicast form).  Protocol: one thread calls
// mbar_init, every thread passes a __syncthreads, one thread posts
// mbar_arrive_expect_tx with the total byte count and issues bulk_g2s for
// each piece, every thread calls mbar_wait(parity 0).  Addresses and sizes
// of bulk copies are multiples of 16 bytes.
__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// Bounded wait for phase `parity` of the barrier; false if it never completed.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity) {
  for (int i = 0; i < (1 << 22); ++i) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// ------------------------------------------------ row staging through smem
// A block of `rows` consecutive rows of `row_len` floats (row stride `stride`
// floats) is copied into shared memory so that every global access is
// coalesced.  When the block is one contiguous, 16-byte-aligned chunk and the
// row length is odd, it is copied with 16-byte cp.async transfers (many in
// flight per thread) into an unpadded buffer (pitch = row_len; odd pitches
// make "thread i reads row i" conflict-free); otherwise with scalar loads
// into a buffer of odd pitch row_len | 1.

__device__ __forceinline__ bool rows_contiguous(const float* g, int64_t stride, int row_len) {
  return stride == row_len && (row_len & 1) && (reinterpret_cast<uintptr_t>(g) & 15) == 0;
}

// True when a row block can be fetched with one bulk copy: contiguous,
// 16-byte aligned (rows_contiguous) and a whole number of 16-byte units.
__device__ __forceinline__ bool rows_bulk(const float* g, int64_t stride, int row_len, int rows) {
  return rows_contiguous(g, stride, row_len) && ((rows * row_len) & 3) == 0;
}

// Shared-memory pitch stage_rows uses for this row block.
__device__ __forceinline__ int stage_pitch(const float* g, int64_t stride, int row_len) {
  return rows_contiguous(g, stride, row_len) ? row_len : (row_len | 1);
}

__device__ __forceinline__ void cp_async16(float* smem_dst, const float* gsrc) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gsrc) : "memory");
}

// Completes every cp.async this thread issued; follow with __syncthreads().
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// Issues the copy of a row block into `dst` (16-byte aligned, pitch
// stage_pitch(...)).  Call cp_async_wait_all() and __syncthreads() before
// reading it.
template <int BLK>
__device__ __forceinline__ void stage_rows(float* dst, const float* __restrict__ src, int64_t stride,
                                           int row_len, int rows) {
  const int total = rows * row_len;
  if (rows_contiguous(src, stride, row_len)) {
    const int nv = total >> 2;
    for (int v = threadIdx.x; v < nv; v += BLK) cp_async16(dst + 4 * v, src + 4 * v);
    for (int e = (nv << 2) + threadIdx.x; e < total; e += BLK) dst[e] = __ldg(src + e);
    return;
  }
  const int ld = row_len | 1;
#pragma unroll 4
  for (int e = threadIdx.x; e < total; e += BLK) {
    const int row = e / row_len;
    const int col = e - row * row_len;
    dst[row * ld + col] = __ldg(src + (int64_t)row * stride + col);
  }
}

// Coalesced write-back of a shared-memory row block of pitch `ld` to global
// rows of stride `stride` (vector stores when both sides allow it).
template <int BLK>
__device__ __forceinline__ void unstage_rows(float* __restrict__ dst, int64_t stride,
                                             const float* src, int ld, int row_len, int rows) {
  const int total = rows * row_len;
  if (ld == row_len && rows_contiguous(dst, stride, row_len)) {
    const int nv = total >> 2;
    for (int v = threadIdx.x; v < nv; v += BLK)
      reinterpret_cast<float4*>(dst)[v] = reinterpret_cast<const float4*>(src)[v];
    for (int e = (nv << 2) + threadIdx.x; e < total; e += BLK) dst[e] = src[e];
    return;
  }
  for (int e = threadIdx.x; e < total; e += BLK) {
    const int row = e / row_len;
    const int col = e - row * row_len;
    dst[(int64_t)row * stride + col] = src[row * ld + col];
  }
}

}  // namespace gs
