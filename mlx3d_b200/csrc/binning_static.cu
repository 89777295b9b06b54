// Tile binning without any device allocation by the caller.
//
// Some callers of this library cannot call cudaMalloc: a renderer embedded
// in a host application whose GPU memory is owned by another allocator (a
// game engine, a plugin host, an inference server with a fixed memory pool)
// is not allowed to allocate device memory of its own, and a caller that
// must never fail on an out-of-memory error mid-frame cannot allocate per
// call either.  gs_bin_gaussians_static gives them binning with the
// scratch space (radix-sort keys, values, histograms, per-Gaussian counts)
// taken from one file-scope __device__ array of fixed size instead of a
// caller-provided workspace.  The caller still provides the inputs and the
// outputs (sorted_ids with a capacity, tile_ranges).
//
// The array is GS_STATIC_BIN_SCRATCH_BYTES (20 MiB); every GPU that loads
// this library keeps it until the process exits.  It bounds the sizes:
// n <= GS_STATIC_BIN_MAX_N Gaussians and D <= GS_STATIC_BIN_MAX_D
// duplicates.
//
// The binning itself is the same code as gs_tile_counts + gs_bin_begin +
// gs_bin_end (those entry points are called on slices of the array), so the
// results are identical to theirs.
//
// Set-up: the first call on a device looks up the device address of the
// array (cudaGetSymbolAddress, with that device current) and caches it;
// make that first call before any stream capture.  The cache is not
// invalidated: after a cudaDeviceReset the module is reloaded at another
// address, so this entry point must not be called again in that process.  Each call reads the
// duplicate count D back to the host (one stream synchronisation, as the
// reference's bin_gaussians does with .item()).  Nothing here calls
// cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "gs_common.cuh"

namespace gs {

constexpr size_t kStaticScratchBytes = GS_STATIC_BIN_SCRATCH_BYTES;

// Shared by every call on a device; calls whose work overlaps on the GPU
// (different streams, or different host threads) race on it.
static __device__ __align__(256) unsigned char g_bin_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {};
static std::mutex g_scratch_mu;

// Device address of g_bin_scratch for the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GS_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(GS_ERR_CUDA, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bin_scratch);
    if (e != cudaSuccess || !p)
      return set_error(GS_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return GS_OK;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace gs

using namespace gs;

extern "C" int gs_bin_gaussians_static(const float* means2d, const float* radii,
                                       const float* depths, int64_t n, int width, int height,
                                       int64_t d_capacity, int32_t* sorted_ids,
                                       int32_t* tile_ranges, int64_t* d_out, void* stream) {
  clear_error();
  if (!d_out) return set_error(GS_ERR_INVALID_ARG, "d_out is NULL");
  *d_out = 0;
  if (n < 0 || n > GS_STATIC_BIN_MAX_N)
    return set_error(GS_ERR_CAPACITY,
                     "gs_bin_gaussians_static: n = %lld exceeds the static limit of %d Gaussians",
                     (long long)n, GS_STATIC_BIN_MAX_N);
  if (width <= 0 || height <= 0) return set_error(GS_ERR_INVALID_ARG, "image size must be positive");
  if (!tile_ranges) return set_error(GS_ERR_INVALID_ARG, "tile_ranges is NULL");
  void* base = nullptr;
  if (int e = scratch_address(&base)) return e;
  // Slices: [counts n int32][d_total int64][workspace_n][workspace_d]
  const size_t counts_off = 0;
  const size_t total_off = align256(counts_off + 4 * (size_t)GS_STATIC_BIN_MAX_N);
  const size_t wsn_off = align256(total_off + sizeof(int64_t));
  const size_t wsn_bytes = gs_bin_workspace_n_bytes(GS_STATIC_BIN_MAX_N);
  const size_t wsd_off = align256(wsn_off + wsn_bytes);
  const size_t wsd_bytes = gs_bin_workspace_d_bytes(GS_STATIC_BIN_MAX_D);
  if (wsd_off + wsd_bytes > kStaticScratchBytes)
    return set_error(GS_ERR_CAPACITY, "static scratch too small for its stated limits");
  char* b = reinterpret_cast<char*>(base);
  int32_t* counts = reinterpret_cast<int32_t*>(b + counts_off);
  int64_t* d_total = reinterpret_cast<int64_t*>(b + total_off);
  cudaStream_t s = as_stream(stream);
  if (n > 0) {
    if (int e = gs_tile_counts(means2d, radii, n, width, height, counts, stream)) return e;
  }
  // gs_bin_begin writes *d_total (it needs no zeroed scratch: every buffer it
  // reads is written earlier in the same call).
  if (int e = gs_bin_begin(depths, counts, n, b + wsn_off, wsn_bytes, d_total, stream)) return e;
  int64_t d = 0;
  cudaError_t ce = cudaMemcpyAsync(&d, d_total, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) return set_error(GS_ERR_CUDA, "reading D: %s", cudaGetErrorString(ce));
  *d_out = d;
  uint32_t st = 0;  // the depth sort and scan have finished: their status is final
  if (n > 0) {
    if (int e = gs_bin_status(b + wsn_off, wsn_bytes, n, &st, stream)) return e;
  }
  if (d > GS_STATIC_BIN_MAX_D)
    return set_error(GS_ERR_CAPACITY,
                     "gs_bin_gaussians_static: %lld duplicates exceed the static limit of %d",
                     (long long)d, GS_STATIC_BIN_MAX_D);
  if (d > d_capacity)
    return set_error(GS_ERR_CAPACITY, "sorted_ids holds %lld entries, %lld needed",
                     (long long)d_capacity, (long long)d);
  return gs_bin_end(means2d, radii, n, d, width, height, b + wsn_off, wsn_bytes, b + wsd_off,
                    wsd_bytes, sorted_ids, tile_ranges, stream);
}
