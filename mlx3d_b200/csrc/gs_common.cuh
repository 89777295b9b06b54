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

// Cooperative copy of `rows` rows of `row_len` floats (source row stride
// `stride` floats) into shared memory with row pitch `ld`.  Consecutive
// threads read consecutive floats of the flattened chunk, so global loads are
// coalesced whatever the row width.
template <int BLK>
__device__ __forceinline__ void stage_rows(float* dst, int ld, const float* __restrict__ src,
                                           int64_t stride, int row_len, int rows) {
  const int total = rows * row_len;
  for (int e = threadIdx.x; e < total; e += BLK) {
    const int row = e / row_len;
    const int col = e - row * row_len;
    dst[row * ld + col] = __ldg(src + (int64_t)row * stride + col);
  }
}

// Inverse of stage_rows: coalesced write-back of a shared-memory row block.
template <int BLK>
__device__ __forceinline__ void unstage_rows(float* __restrict__ dst, int64_t stride,
                                             const float* src, int ld, int row_len, int rows) {
  const int total = rows * row_len;
  for (int e = threadIdx.x; e < total; e += BLK) {
    const int row = e / row_len;
    const int col = e - row * row_len;
    dst[(int64_t)row * stride + col] = src[row * ld + col];
  }
}

}  // namespace gs
