// Training-step kernels of the 3DGS recipe (src/mlx3d/splatting/trainer.py:
// 261-355): the photometric loss (1 - lambda) * L1 + lambda * (1 - SSIM)
// (losses/image_metrics.py:29-85) with its gradient, and the per-parameter
// Adam update (mlx.optimizers.Adam, eps = 1e-15, trainer.py:128).
//
// SSIM: Gaussian window w (11 taps, sigma 1.5, normalised), depthwise
// "same" convolution with zero padding, written as two separable passes over
// a 16x16 output tile plus halo staged in shared memory.  The forward pass
// produces the SSIM and L1 sums and, per pixel and channel, the partial
// derivatives of ssim_map with respect to mu_p = w*p, P = w*(p*p) and
// X = w*(p*t); the backward pass filters those three maps with the same
// (symmetric) window — the transpose of the convolution — and combines them:
//   d mean(ssim_map) / d p(x) = [ (w*D_mu)(x) + 2 p(x) (w*D_P)(x) + t(x) (w*D_X)(x) ] / numel
#include <algorithm>
#include <cmath>

#include "gs_common.cuh"

namespace gs {

constexpr int kLT = 16;   // output tile edge
constexpr int kMaxR = 7;  // largest window radius supported (15 taps)
constexpr int kLossThreads = kLT * kLT;

struct SsimArgs {
  const float *pred, *target;
  int H, W, C;
  int radius;
  float w[2 * kMaxR + 1];
  float c1, c2;
  float* dmaps;      // (H, W, C, 3): dS/dmu_p, dS/dP, dS/dX
  double* partials;  // per block: (sum ssim_map, sum |p - t|)
};

// One channel's tile with halo r, zero outside the image.
__device__ __forceinline__ void load_halo(float* dst, const float* src, int H, int W, int C, int ch,
                                          int x0, int y0, int r) {
  const int E = kLT + 2 * r;
  for (int e = threadIdx.x; e < E * E; e += kLossThreads) {
    const int yy = e / E, xx = e - yy * E;
    const int gy = y0 - r + yy, gx = x0 - r + xx;
    dst[e] = (gy >= 0 && gy < H && gx >= 0 && gx < W) ? src[((int64_t)gy * W + gx) * C + ch] : 0.0f;
  }
}

__global__ void __launch_bounds__(kLossThreads) k_ssim_fwd(const SsimArgs a) {
  constexpr int E = kLT + 2 * kMaxR;
  __shared__ float s_p[E * E], s_t[E * E];
  __shared__ float s_h[5][E][kLT];  // horizontally filtered p, t, pp, tt, pt
  __shared__ double s_red[2][kLossThreads / 32];
  const int r = a.radius, Er = kLT + 2 * r;
  const int ch = blockIdx.z;
  const int x0 = blockIdx.x * kLT, y0 = blockIdx.y * kLT;
  load_halo(s_p, a.pred, a.H, a.W, a.C, ch, x0, y0, r);
  load_halo(s_t, a.target, a.H, a.W, a.C, ch, x0, y0, r);
  __syncthreads();
  for (int e = threadIdx.x; e < Er * kLT; e += kLossThreads) {
    const int yy = e / kLT, xx = e - yy * kLT;
    float hp = 0.f, ht = 0.f, hpp = 0.f, htt = 0.f, hpt = 0.f;
    for (int k = 0; k <= 2 * r; ++k) {
      const float p = s_p[yy * Er + xx + k], t = s_t[yy * Er + xx + k], wk = a.w[k];
      hp += wk * p;
      ht += wk * t;
      hpp += wk * p * p;
      htt += wk * t * t;
      hpt += wk * p * t;
    }
    s_h[0][yy][xx] = hp;
    s_h[1][yy][xx] = ht;
    s_h[2][yy][xx] = hpp;
    s_h[3][yy][xx] = htt;
    s_h[4][yy][xx] = hpt;
  }
  __syncthreads();
  const int lx = threadIdx.x % kLT, ly = threadIdx.x / kLT;
  const int x = x0 + lx, y = y0 + ly;
  double ssim_sum = 0.0, l1_sum = 0.0;
  if (x < a.W && y < a.H) {
    float mp = 0.f, mt = 0.f, P = 0.f, T = 0.f, X = 0.f;
    for (int k = 0; k <= 2 * r; ++k) {
      const float wk = a.w[k];
      mp += wk * s_h[0][ly + k][lx];
      mt += wk * s_h[1][ly + k][lx];
      P += wk * s_h[2][ly + k][lx];
      T += wk * s_h[3][ly + k][lx];
      X += wk * s_h[4][ly + k][lx];
    }
    const float sp = P - mp * mp, st = T - mt * mt, spt = X - mp * mt;
    const float A = 2.0f * mp * mt + a.c1, B = mp * mp + mt * mt + a.c1;
    const float Cn = 2.0f * spt + a.c2, Dn = sp + st + a.c2;
    const float lum = A / B, cs = Cn / Dn;
    const float S = lum * cs;
    // partials of S(mu_p, P, X) with mu_t and T fixed
    const float dS_dX = lum * 2.0f / Dn;
    const float dS_dP = -S / Dn;
    const float dS_dmu =
        cs * (2.0f * mt - 2.0f * mp * lum) / B + lum * (-2.0f * mt + 2.0f * mp * cs) / Dn;
    float* d = a.dmaps + (((int64_t)y * a.W + x) * a.C + ch) * 3;
    d[0] = dS_dmu;
    d[1] = dS_dP;
    d[2] = dS_dX;
    ssim_sum = S;
    l1_sum = fabsf(s_p[(ly + r) * Er + lx + r] - s_t[(ly + r) * Er + lx + r]);
  }
  for (int o = 16; o > 0; o >>= 1) {
    ssim_sum += __shfl_xor_sync(0xffffffffu, ssim_sum, o);
    l1_sum += __shfl_xor_sync(0xffffffffu, l1_sum, o);
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_red[0][warp] = ssim_sum;
    s_red[1][warp] = l1_sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a0 = 0.0, a1 = 0.0;
    for (int w = 0; w < kLossThreads / 32; ++w) {
      a0 += s_red[0][w];
      a1 += s_red[1][w];
    }
    const int64_t b = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    a.partials[2 * b] = a0;
    a.partials[2 * b + 1] = a1;
  }
}

// loss[0] = (1 - lambda) * l1 + lambda * (1 - ssim), loss[1] = l1,
// loss[2] = ssim (means over H*W*C); one block, fixed summation order.
__global__ void k_loss_finish(const double* __restrict__ partials, int nblocks, double numel,
                              float lambda, float* __restrict__ loss) {
  __shared__ double s0[256], s1[256];
  double a0 = 0.0, a1 = 0.0;
  for (int b = threadIdx.x; b < nblocks; b += blockDim.x) {
    a0 += partials[2 * b];
    a1 += partials[2 * b + 1];
  }
  s0[threadIdx.x] = a0;
  s1[threadIdx.x] = a1;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) {
      s0[threadIdx.x] += s0[threadIdx.x + o];
      s1[threadIdx.x] += s1[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double ssim = s0[0] / numel, l1 = s1[0] / numel;
    loss[0] = (float)((1.0 - lambda) * l1 + lambda * (1.0 - ssim));
    loss[1] = (float)l1;
    loss[2] = (float)ssim;
  }
}

struct SsimBwdArgs {
  SsimArgs f;
  float lambda, scale;
  const float* scale_dev;  // if set, the scale is scale * scale_dev[0]
  int accumulate;          // grad += instead of grad =
  float* grad;             // (H, W, C)
};

__global__ void __launch_bounds__(kLossThreads) k_ssim_bwd(const SsimBwdArgs g) {
  const SsimArgs& a = g.f;
  constexpr int E = kLT + 2 * kMaxR;
  __shared__ float s_d[3][E * E];
  __shared__ float s_h[3][E][kLT];
  const int r = a.radius, Er = kLT + 2 * r;
  const int ch = blockIdx.z;
  const int x0 = blockIdx.x * kLT, y0 = blockIdx.y * kLT;
  for (int e = threadIdx.x; e < Er * Er; e += kLossThreads) {
    const int yy = e / Er, xx = e - yy * Er;
    const int gy = y0 - r + yy, gx = x0 - r + xx;
    const bool in = gy >= 0 && gy < a.H && gx >= 0 && gx < a.W;
    const int64_t o = in ? (((int64_t)gy * a.W + gx) * a.C + ch) * 3 : 0;
    s_d[0][e] = in ? a.dmaps[o] : 0.0f;
    s_d[1][e] = in ? a.dmaps[o + 1] : 0.0f;
    s_d[2][e] = in ? a.dmaps[o + 2] : 0.0f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < Er * kLT; e += kLossThreads) {
    const int yy = e / kLT, xx = e - yy * kLT;
    float h0 = 0.f, h1 = 0.f, h2 = 0.f;
    for (int k = 0; k <= 2 * r; ++k) {
      const float wk = a.w[k];
      h0 += wk * s_d[0][yy * Er + xx + k];
      h1 += wk * s_d[1][yy * Er + xx + k];
      h2 += wk * s_d[2][yy * Er + xx + k];
    }
    s_h[0][yy][xx] = h0;
    s_h[1][yy][xx] = h1;
    s_h[2][yy][xx] = h2;
  }
  __syncthreads();
  const int lx = threadIdx.x % kLT, ly = threadIdx.x / kLT;
  const int x = x0 + lx, y = y0 + ly;
  if (x >= a.W || y >= a.H) return;
  float f0 = 0.f, f1 = 0.f, f2 = 0.f;
  for (int k = 0; k <= 2 * r; ++k) {
    const float wk = a.w[k];
    f0 += wk * s_h[0][ly + k][lx];
    f1 += wk * s_h[1][ly + k][lx];
    f2 += wk * s_h[2][ly + k][lx];
  }
  const int64_t idx = ((int64_t)y * a.W + x) * a.C + ch;
  const float p = a.pred[idx], t = a.target[idx];
  const float numel = (float)((double)a.H * a.W * a.C);
  const float dssim = (f0 + 2.0f * p * f1 + t * f2) / numel;
  const float diff = p - t;
  const float sgn = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
  const float scale = g.scale_dev ? g.scale * g.scale_dev[0] : g.scale;
  const float v = scale * ((1.0f - g.lambda) * sgn / numel - g.lambda * dssim);
  g.grad[idx] = g.accumulate ? g.grad[idx] + v : v;
}

// ---------------------------------------------------------------- L1 loss
// mean |pred - target| over n values: per-block partial sums (float per
// thread, double per block) and one finishing block, fixed order, so the
// result does not depend on scheduling.
constexpr int kL1Blocks = 148 * 4;
constexpr int kL1Threads = 256;

__global__ void __launch_bounds__(kL1Threads)
k_l1_partial(const float* __restrict__ pred, const float* __restrict__ target, int64_t n,
             double* __restrict__ partials) {
  __shared__ double s[kL1Threads];
  float acc = 0.0f;
  const int64_t stride = (int64_t)gridDim.x * kL1Threads;
  const int64_t t0 = (int64_t)blockIdx.x * kL1Threads + threadIdx.x;
  int64_t tail = 0;
  if (((reinterpret_cast<uintptr_t>(pred) | reinterpret_cast<uintptr_t>(target)) & 15) == 0) {
    // 16-byte vectors, four in flight per thread
    const float4* p4 = reinterpret_cast<const float4*>(pred);
    const float4* t4 = reinterpret_cast<const float4*>(target);
    const int64_t nv = n >> 2;
#pragma unroll 4
    for (int64_t v = t0; v < nv; v += stride) {
      const float4 a = __ldg(p4 + v), b = __ldg(t4 + v);
      acc += (fabsf(a.x - b.x) + fabsf(a.y - b.y)) + (fabsf(a.z - b.z) + fabsf(a.w - b.w));
    }
    tail = nv << 2;
  }
  for (int64_t i = tail + t0; i < n; i += stride) acc += fabsf(pred[i] - target[i]);
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int o = kL1Threads / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) partials[blockIdx.x] = s[0];
}

__global__ void __launch_bounds__(kL1Threads)
k_l1_finish(const double* __restrict__ partials, int nb, double n, float* __restrict__ loss) {
  __shared__ double s[kL1Threads];
  double acc = 0.0;
  for (int b = threadIdx.x; b < nb; b += kL1Threads) acc += partials[b];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int o = kL1Threads / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) loss[0] = (float)(s[0] / n);
}

// grad = g[0] * sign(pred - target) / n  (sign(0) = 0, the subgradient of
// |x| that autodiff of abs uses).
__global__ void k_l1_bwd(const float* __restrict__ pred, const float* __restrict__ target, int64_t n,
                         const float* __restrict__ g, float* __restrict__ grad) {
  const float scale = g[0] / (float)n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float d = pred[i] - target[i];
    grad[i] = d > 0.0f ? scale : (d < 0.0f ? -scale : 0.0f);
  }
}

// ------------------------------------------------------------------- Adam
struct AdamArgs {
  gs_adam_group groups[GS_ADAM_MAX_GROUPS];
  float b1, b2, omb1, omb2, eps;
  int bias_correction;
  float bc1[GS_ADAM_MAX_GROUPS];  // lr / (1 - b1^step)
  float bc2;                      // 1 / sqrt(1 - b2^step)
};

// blockIdx.y = parameter group, grid-stride over its elements, in the
// operation order of mlx.optimizers.Adam.apply_single:
//   m = b1 m + (1 - b1) g ;  v = b2 v + (1 - b2) g^2 ;  p - lr m / (sqrt(v) + eps)
__global__ void __launch_bounds__(256) k_adam(const AdamArgs a) {
  const gs_adam_group& G = a.groups[blockIdx.y];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < G.n; i += stride) {
    const float g = G.grad[i];
    const float m = gs_add(gs_mul(a.b1, G.m[i]), gs_mul(a.omb1, g));
    const float v = gs_add(gs_mul(a.b2, G.v[i]), gs_mul(a.omb2, gs_mul(g, g)));
    G.m[i] = m;
    G.v[i] = v;
    const float p = G.param[i];
    if (a.bias_correction)
      G.param[i] = gs_sub(p, gs_div(gs_mul(a.bc1[blockIdx.y], m), gs_add(gs_mul(gs_sqrt(v), a.bc2), a.eps)));
    else
      G.param[i] = gs_sub(p, gs_div(gs_mul(G.lr, m), gs_add(gs_sqrt(v), a.eps)));
  }
}

// image_metrics.py:23-26: x = arange(size) - (size - 1) / 2,
// g = exp(-x^2 / (2 sigma^2)), normalised to sum 1 (float32).
static int fill_window(SsimArgs& a, int window_size, float sigma) {
  if (window_size < 1 || window_size % 2 == 0 || window_size > 2 * kMaxR + 1)
    return set_error(GS_ERR_INVALID_ARG, "window_size must be odd and <= %d (got %d)",
                     2 * kMaxR + 1, window_size);
  if (!(sigma > 0.0f)) return set_error(GS_ERR_INVALID_ARG, "sigma must be positive");
  a.radius = window_size / 2;
  float sum = 0.0f;
  for (int k = 0; k < window_size; ++k) {
    const float x = (float)k - (float)(window_size - 1) / 2.0f;
    a.w[k] = expf(-(x * x) / (2.0f * sigma * sigma));
    sum += a.w[k];
  }
  for (int k = 0; k < window_size; ++k) a.w[k] /= sum;
  return GS_OK;
}

static size_t dmaps_bytes(int h, int w, int c) {
  return ((size_t)h * w * c * 3 * sizeof(float) + 255) & ~(size_t)255;
}

}  // namespace gs

using namespace gs;

extern "C" {

size_t gs_l1_ssim_workspace_bytes(int height, int width, int channels) {
  const int64_t bx = ceil_div(width, kLT), by = ceil_div(height, kLT);
  return dmaps_bytes(height, width, channels) + (size_t)bx * by * channels * 2 * sizeof(double);
}

int gs_l1_ssim_forward(const float* pred, const float* target, int height, int width, int channels,
                       float lambda_dssim, float max_val, int window_size, float sigma,
                       void* workspace, size_t workspace_bytes, float* loss, void* stream) {
  clear_error();
  if (height <= 0 || width <= 0 || channels <= 0)
    return set_error(GS_ERR_INVALID_ARG, "image must be non-empty (got %dx%dx%d)", height, width,
                     channels);
  if (!pred || !target || !loss) return set_error(GS_ERR_INVALID_ARG, "gs_l1_ssim_forward: NULL pointer");
  if (!workspace || workspace_bytes < gs_l1_ssim_workspace_bytes(height, width, channels))
    return set_error(GS_ERR_CAPACITY, "loss workspace too small");
  SsimArgs a{};
  if (int e = fill_window(a, window_size, sigma)) return e;
  a.pred = pred; a.target = target; a.H = height; a.W = width; a.C = channels;
  a.c1 = (0.01f * max_val) * (0.01f * max_val);
  a.c2 = (0.03f * max_val) * (0.03f * max_val);
  a.dmaps = reinterpret_cast<float*>(workspace);
  a.partials = reinterpret_cast<double*>(reinterpret_cast<char*>(workspace) +
                                         dmaps_bytes(height, width, channels));
  const dim3 grid((unsigned)ceil_div(width, kLT), (unsigned)ceil_div(height, kLT), (unsigned)channels);
  cudaStream_t s = as_stream(stream);
  k_ssim_fwd<<<grid, kLossThreads, 0, s>>>(a);
  k_loss_finish<<<1, 256, 0, s>>>(a.partials, (int)(grid.x * grid.y * grid.z),
                                 (double)height * width * channels, lambda_dssim, loss);
  return check_launch("k_ssim_fwd", 2);
}

static int l1_ssim_backward(const float* pred, const float* target, int height, int width, int channels,
                            float lambda_dssim, int window_size, float sigma, const void* workspace,
                            size_t workspace_bytes, float grad_scale, const float* grad_scale_dev,
                            int accumulate, float* grad_pred, void* stream) {
  clear_error();
  if (height <= 0 || width <= 0 || channels <= 0)
    return set_error(GS_ERR_INVALID_ARG, "image must be non-empty");
  if (!pred || !target || !grad_pred)
    return set_error(GS_ERR_INVALID_ARG, "gs_l1_ssim_backward: NULL pointer");
  if (!workspace || workspace_bytes < gs_l1_ssim_workspace_bytes(height, width, channels))
    return set_error(GS_ERR_CAPACITY, "loss workspace too small");
  SsimBwdArgs g{};
  if (int e = fill_window(g.f, window_size, sigma)) return e;
  g.f.pred = pred; g.f.target = target; g.f.H = height; g.f.W = width; g.f.C = channels;
  g.f.dmaps = reinterpret_cast<float*>(const_cast<void*>(workspace));
  g.lambda = lambda_dssim;
  g.scale = grad_scale;
  g.scale_dev = grad_scale_dev;
  g.accumulate = accumulate;
  g.grad = grad_pred;
  const dim3 grid((unsigned)ceil_div(width, kLT), (unsigned)ceil_div(height, kLT), (unsigned)channels);
  k_ssim_bwd<<<grid, kLossThreads, 0, as_stream(stream)>>>(g);
  return check_launch("k_ssim_bwd");
}

int gs_l1_ssim_backward(const float* pred, const float* target, int height, int width, int channels,
                        float lambda_dssim, float max_val, int window_size, float sigma,
                        const void* workspace, size_t workspace_bytes, float grad_scale,
                        float* grad_pred, void* stream) {
  (void)max_val;  // the SSIM constants enter only through the forward's partial maps
  return l1_ssim_backward(pred, target, height, width, channels, lambda_dssim, window_size, sigma, workspace,
                          workspace_bytes, grad_scale, nullptr, 0, grad_pred, stream);
}

int gs_l1_ssim_backward_dev(const float* pred, const float* target, int height, int width, int channels,
                            float lambda_dssim, int window_size, float sigma, const void* workspace,
                            size_t workspace_bytes, const float* grad_scale, float grad_sign, int accumulate,
                            float* grad_pred, void* stream) {
  if (!grad_scale) return set_error(GS_ERR_INVALID_ARG, "gs_l1_ssim_backward_dev: grad_scale is NULL");
  return l1_ssim_backward(pred, target, height, width, channels, lambda_dssim, window_size, sigma, workspace,
                          workspace_bytes, grad_sign, grad_scale, accumulate, grad_pred, stream);
}

size_t gs_l1_workspace_bytes(int64_t n) {
  (void)n;
  return sizeof(double) * kL1Blocks;
}

int gs_l1_forward(const float* pred, const float* target, int64_t n, void* workspace, size_t workspace_bytes,
                  float* loss, void* stream) {
  clear_error();
  if (n <= 0) return set_error(GS_ERR_INVALID_ARG, "gs_l1_forward: n must be positive");
  if (!pred || !target || !loss) return set_error(GS_ERR_INVALID_ARG, "gs_l1_forward: NULL pointer");
  if (!workspace || workspace_bytes < gs_l1_workspace_bytes(n))
    return set_error(GS_ERR_CAPACITY, "gs_l1_forward: workspace too small");
  cudaStream_t s = as_stream(stream);
  double* partials = reinterpret_cast<double*>(workspace);
  k_l1_partial<<<kL1Blocks, kL1Threads, 0, s>>>(pred, target, n, partials);
  k_l1_finish<<<1, kL1Threads, 0, s>>>(partials, kL1Blocks, (double)n, loss);
  return check_launch("k_l1_partial", 2);
}

int gs_l1_backward(const float* pred, const float* target, int64_t n, const float* grad_loss, float* grad_pred,
                   void* stream) {
  clear_error();
  if (n <= 0) return set_error(GS_ERR_INVALID_ARG, "gs_l1_backward: n must be positive");
  if (!pred || !target || !grad_loss || !grad_pred)
    return set_error(GS_ERR_INVALID_ARG, "gs_l1_backward: NULL pointer");
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 8);
  k_l1_bwd<<<grid, 256, 0, as_stream(stream)>>>(pred, target, n, grad_loss, grad_pred);
  return check_launch("k_l1_bwd");
}

int gs_adam_step(const gs_adam_group* groups, int n_groups, double beta1, double beta2, float eps,
                 int bias_correction, int64_t step, void* stream) {
  clear_error();
  if (n_groups < 0 || n_groups > GS_ADAM_MAX_GROUPS)
    return set_error(GS_ERR_INVALID_ARG, "n_groups must be in [0, %d]", GS_ADAM_MAX_GROUPS);
  if (n_groups == 0) return GS_OK;
  if (!groups) return set_error(GS_ERR_INVALID_ARG, "groups is NULL");
  if (bias_correction && step < 1) return set_error(GS_ERR_INVALID_ARG, "step must be >= 1");
  AdamArgs a{};
  int64_t nmax = 0;
  for (int k = 0; k < n_groups; ++k) {
    const gs_adam_group& G = groups[k];
    if (G.n < 0 || (G.n > 0 && (!G.param || !G.grad || !G.m || !G.v)))
      return set_error(GS_ERR_INVALID_ARG, "Adam group %d: NULL pointer or negative size", k);
    a.groups[k] = G;
    nmax = std::max(nmax, G.n);
    if (bias_correction) a.bc1[k] = (float)((double)G.lr / (1.0 - pow(beta1, (double)step)));
  }
  a.b1 = (float)beta1;
  a.b2 = (float)beta2;
  a.omb1 = (float)(1.0 - beta1);
  a.omb2 = (float)(1.0 - beta2);
  a.eps = eps;
  a.bias_correction = bias_correction;
  a.bc2 = bias_correction ? (float)(1.0 / sqrt(1.0 - pow(beta2, (double)step))) : 1.0f;
  if (nmax == 0) return GS_OK;
  const unsigned gx = (unsigned)std::min<int64_t>(ceil_div(nmax, 256), 148 * 16);
  k_adam<<<dim3(gx, (unsigned)n_groups), 256, 0, as_stream(stream)>>>(a);
  return check_launch("k_adam");
}

}  // extern "C"
