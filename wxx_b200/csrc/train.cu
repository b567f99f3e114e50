// Training kernels: the backward passes, loss and optimiser the reference's
// autograd uses on GPT2's path (src/wxx/autograd/*.py backward methods,
// shaders/activations/{gelubackwards,softmaxbackwards}.wgsl,
// shaders/layers/{meanvarnormdx,embeddx}.wgsl, shaders/loss/cceloss.wgsl,
// shaders/optimizers/adamw.wgsl).  The matmul / linear gradients are
// products on the existing tcgen05 GEMM; the bias and LayerNorm-affine
// gradients are column sums on the existing reduction kernels.  Everything
// here is memory-bound: one pass over its inputs, 16-byte loads where the
// rows allow, a warp per row for the row-wise ops.

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

#include <cstring>

namespace {

constexpr int kT = 256;

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// dx = dy * gelu'(x), gelu the tanh form with the reference's clamps
// (gelu.wgsl: x > 10 -> x, x < -10 -> 0; so the slope is 1 / 0 there).
__global__ void gelu_backward_kernel(float* __restrict__ dx, const float* __restrict__ dy,
                                     const float* __restrict__ x, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    float slope;
    if (v > 10.0f) {
      slope = 1.0f;
    } else if (v < -10.0f) {
      slope = 0.0f;
    } else {
      const float c = 0.7978845608f;
      const float t = tanhf(c * (v + 0.044715f * v * v * v));
      const float du = c * (1.0f + 0.134145f * v * v);
      slope = 0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * du;
    }
    dx[i] = dy[i] * slope;
  }
}

// Softmax backward over rows of n (one warp per row, row in registers):
// dx = y * (dy - sum_j dy_j y_j).
template <int PER>
__global__ void __launch_bounds__(256) softmax_backward_kernel(float* __restrict__ dx,
                                                               const float* __restrict__ dy,
                                                               const float* __restrict__ y,
                                                               int64_t rows, int n) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (row >= rows) return;
  const float* yr = y + row * n;
  const float* gr = dy + row * n;
  float yv[PER], gv[PER];
  float dot = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = k * 32 + l;
    yv[k] = c < n ? yr[c] : 0.f;
    gv[k] = c < n ? gr[c] : 0.f;
    dot += yv[k] * gv[k];
  }
  dot = warp_sum_f(dot);
  float* out = dx + row * n;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = k * 32 + l;
    if (c < n) out[c] = yv[k] * (gv[k] - dot);
  }
}

// LayerNorm backward over rows of n (one warp per row) from the forward's
// saved mean and inverse standard deviation: xhat = (x - mean) inv,
// g = dy gamma, dx = inv (g - mean(g) - xhat mean(g xhat)); also writes
// dyxhat = dy * xhat, whose column sums are d gamma (d beta = column sums of
// dy).  A row with inv = 0 (zero variance) gets dx = 0.
template <int PER>
__global__ void __launch_bounds__(256) layernorm_backward_kernel(
    float* __restrict__ dx, float* __restrict__ dyxhat, const float* __restrict__ dy,
    const float* __restrict__ x, const float* __restrict__ mean, const float* __restrict__ inv,
    const float* __restrict__ gamma, int64_t rows, int n) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (row >= rows) return;
  const float mu = mean[row], is = inv[row];
  float xh[PER], g[PER];
  float sg = 0.f, sgx = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = k * 32 + l;
    const bool in = c < n;
    const float d = in ? dy[row * n + c] : 0.f;
    xh[k] = in ? (x[row * n + c] - mu) * is : 0.f;
    g[k] = in ? d * gamma[c] : 0.f;
    sg += g[k];
    sgx += g[k] * xh[k];
    if (in) dyxhat[row * n + c] = d * xh[k];
  }
  sg = warp_sum_f(sg) / (float)n;
  sgx = warp_sum_f(sgx) / (float)n;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = k * 32 + l;
    if (c < n) dx[row * n + c] = is * (g[k] - sg - xh[k] * sgx);
  }
}

// dW[ids[t], :] += dY[t, :] (dW zeroed by the caller); ids outside the table
// are skipped and raise WXX_DEV_ERR_BAD_INDEX, as the forward does.
__global__ void embedding_backward_kernel(float* __restrict__ dW,
                                          const uint32_t* __restrict__ ids,
                                          const float* __restrict__ dY, int64_t n_tokens, int D,
                                          uint32_t vocab, int* err) {
  const int64_t total = n_tokens * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / D;
    const int d = (int)(i - t * D);
    const uint32_t id = ids[t];
    if (id >= vocab) {
      if (d == 0) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
      continue;
    }
    atomicAdd(dW + (int64_t)id * D + d, dY[i]);
  }
}

// Softmax cross-entropy per row (cceloss.wgsl): loss[row] = log(sum exp z) -
// z[target] and dZ = softmax(z) - onehot(target), fp32 with the max shift.
__global__ void __launch_bounds__(kT) cce_kernel(float* __restrict__ loss, float* __restrict__ dZ,
                                                 const float* __restrict__ Z,
                                                 const uint32_t* __restrict__ targets, int K,
                                                 int* err) {
  __shared__ float red[kT / 32];
  const int64_t row = blockIdx.x;
  const float* z = Z + row * K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m = -1e38f;
  for (int c = threadIdx.x; c < K; c += kT) m = fmaxf(m, z[c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < kT / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float s = 0.f;
  for (int c = threadIdx.x; c < K; c += kT) s += expf(z[c] - m);
  s = warp_sum_f(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  s = 0.f;
#pragma unroll
  for (int w = 0; w < kT / 32; ++w) s += red[w];
  const uint32_t t = targets[row];
  const bool ok = t < (uint32_t)K;
  if (threadIdx.x == 0) {
    if (!ok) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
    loss[row] = ok ? logf(s) + m - z[t] : 0.f;
  }
  const float inv = 1.0f / s;
  float* g = dZ + row * K;
  for (int c = threadIdx.x; c < K; c += kT)
    g[c] = expf(z[c] - m) * inv - ((ok && (uint32_t)c == t) ? 1.0f : 0.0f);
}

// AdamW step (adamw.wgsl): m = b1 m + (1 - b1) g, v = b2 v + (1 - b2) g^2,
// p -= lr (m / bc1 / (sqrt(v / bc2) + eps) + wd p).
// bc_dev (when not NULL) holds {bc1, bc2} in device memory, written by
// adamw_advance_kernel: a step recorded in a CUDA graph then uses each
// replay's own bias corrections.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, int64_t n, float lr,
                             float b1, float b2, float eps, float wd, float bc1, float bc2,
                             const float* __restrict__ bc_dev) {
  if (bc_dev != nullptr) {
    bc1 = bc_dev[0];
    bc2 = bc_dev[1];
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float pi = p[i], gi = g[i];
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float step = (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi - lr * (step + wd * pi);
  }
}

// Up to kAdamwMulti parameters stepped by one launch (their pointers passed by
// value, so a recorded step replays with the same tensors): chunk c of the
// launch belongs to the tensor whose [start, start of the next) holds it.
constexpr int kAdamwMulti = 128;
constexpr int kAdamwChunk = 4096;
struct AdamwTable {
  int n;
  int64_t start[kAdamwMulti + 1];   // first chunk of each tensor, prefix
  float* p[kAdamwMulti];
  const float* g[kAdamwMulti];
  float* m[kAdamwMulti];
  float* v[kAdamwMulti];
  int64_t len[kAdamwMulti];
};

__global__ void adamw_multi_kernel(const __grid_constant__ AdamwTable tab, float lr, float b1,
                                   float b2, float eps, float wd, const float* __restrict__ bc) {
  const float bc1 = bc[0], bc2 = bc[1];
  const int64_t chunk = blockIdx.x;
  int lo = 0, hi = tab.n - 1;   // last tensor whose start <= chunk
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab.start[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  const int t = lo;
  const int64_t base = (chunk - tab.start[t]) * kAdamwChunk;
  const int64_t end = min(tab.len[t], base + kAdamwChunk);
  float* __restrict__ p = tab.p[t];
  const float* __restrict__ g = tab.g[t];
  float* __restrict__ m = tab.m[t];
  float* __restrict__ v = tab.v[t];
  for (int64_t i = base + threadIdx.x; i < end; i += blockDim.x) {
    const float pi = p[i], gi = g[i];
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float step = (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi - lr * (step + wd * pi);
  }
}

// step += 1; bc = {1 - beta1^step, 1 - beta2^step} (double, stored as float:
// the values nn/optimizer.py computes on the host).
__global__ void adamw_advance_kernel(int* step, float* bc, double b1, double b2) {
  const int t = ++step[0];
  bc[0] = (float)(1.0 - pow(b1, (double)t));
  bc[1] = (float)(1.0 - pow(b2, (double)t));
}

}  // namespace

// autograd gelu backward (gelubackwards.wgsl times grad_output): dx = dy * gelu'(x).
WXX_EXPORT int wxx_gelu_backward(float* dx, const float* dy, const float* x, int64_t n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 0, "wxx_gelu_backward: negative size");
  if (n == 0) return WXX_OK;
  gelu_backward_kernel<<<wxx::grid_for(n, kT), kT, 0, wxx::stream()>>>(dx, dy, x, n);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// autograd softmax backward over the last axis (softmaxbackwards.wgsl), rows of n <= 1024.
WXX_EXPORT int wxx_softmax_backward(float* dx, const float* dy, const float* y, int64_t rows,
                                    int64_t n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 1 && n <= 1024, "wxx_softmax_backward: row length %lld outside [1, 1024]",
              (long long)n);
  if (rows == 0) return WXX_OK;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  cudaStream_t s = wxx::stream();
  if (n <= 128) softmax_backward_kernel<4><<<grid, 256, 0, s>>>(dx, dy, y, rows, (int)n);
  else if (n <= 256) softmax_backward_kernel<8><<<grid, 256, 0, s>>>(dx, dy, y, rows, (int)n);
  else if (n <= 512) softmax_backward_kernel<16><<<grid, 256, 0, s>>>(dx, dy, y, rows, (int)n);
  else softmax_backward_kernel<32><<<grid, 256, 0, s>>>(dx, dy, y, rows, (int)n);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// autograd meanvarnorm backward (meanvarnormdx / meanvarnormdg) over rows of n <= 1024:
// dx and dyxhat = dy * xhat (column sums of dyxhat are d gamma).
WXX_EXPORT int wxx_layernorm_backward(float* dx, float* dyxhat, const float* dy, const float* x,
                                      const float* mean, const float* inv, const float* gamma,
                                      int64_t rows, int64_t n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 1 && n <= 1024, "wxx_layernorm_backward: row length %lld outside [1, 1024]",
              (long long)n);
  if (rows == 0) return WXX_OK;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  cudaStream_t s = wxx::stream();
  if (n <= 128)
    layernorm_backward_kernel<4><<<grid, 256, 0, s>>>(dx, dyxhat, dy, x, mean, inv, gamma, rows, (int)n);
  else if (n <= 256)
    layernorm_backward_kernel<8><<<grid, 256, 0, s>>>(dx, dyxhat, dy, x, mean, inv, gamma, rows, (int)n);
  else if (n <= 512)
    layernorm_backward_kernel<16><<<grid, 256, 0, s>>>(dx, dyxhat, dy, x, mean, inv, gamma, rows, (int)n);
  else
    layernorm_backward_kernel<32><<<grid, 256, 0, s>>>(dx, dyxhat, dy, x, mean, inv, gamma, rows, (int)n);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// autograd Embedding backward (embeddx.wgsl): dW (vocab, D), zeroed here, += dY rows by id.
WXX_EXPORT int wxx_embedding_backward(float* dW, const uint32_t* ids, const float* dY,
                                      int64_t n_tokens, int D, int vocab) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n_tokens >= 0 && D > 0 && vocab > 0, "wxx_embedding_backward: bad sizes");
  WXX_CUDA_CHECK(cudaMemsetAsync(dW, 0, (size_t)vocab * D * sizeof(float), wxx::stream()));
  if (n_tokens == 0) return WXX_OK;
  embedding_backward_kernel<<<wxx::grid_for(n_tokens * D, kT), kT, 0, wxx::stream()>>>(
      dW, ids, dY, n_tokens, D, (uint32_t)vocab, wxx::device_error_word());
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// functional.cceloss (cceloss.wgsl): loss (rows) and dZ = softmax - onehot for (rows, K) logits
// and u32 targets.
WXX_EXPORT int wxx_cceloss(float* loss, float* dZ, const float* Z, const uint32_t* targets,
                           int64_t rows, int K) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(rows >= 0 && K >= 1, "wxx_cceloss: bad sizes");
  WXX_REQUIRE(rows < (int64_t(1) << 31), "wxx_cceloss: too many rows");
  if (rows == 0) return WXX_OK;
  cce_kernel<<<(unsigned)rows, kT, 0, wxx::stream()>>>(loss, dZ, Z, targets, K,
                                                       wxx::device_error_word());
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// functional.adamw (adamw.wgsl): one AdamW step over n parameters in place.
WXX_EXPORT int wxx_adamw(float* p, const float* g, float* m, float* v, int64_t n, float lr,
                         float beta1, float beta2, float eps, float weight_decay, float bc1,
                         float bc2) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 0, "wxx_adamw: negative size");
  if (n == 0) return WXX_OK;
  adamw_kernel<<<wxx::grid_for(n, kT), kT, 0, wxx::stream()>>>(p, g, m, v, n, lr, beta1, beta2,
                                                               eps, weight_decay, bc1, bc2,
                                                               nullptr);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// nn.AdamW's step with the bias corrections read from device memory
// (bc[0] = bc1, bc[1] = bc2, from wxx_adamw_advance).
WXX_EXPORT int wxx_adamw_device(float* p, const float* g, float* m, float* v, int64_t n, float lr,
                                float beta1, float beta2, float eps, float weight_decay,
                                const float* bc) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 0 && bc != nullptr, "wxx_adamw_device: negative size or no bias corrections");
  if (n == 0) return WXX_OK;
  adamw_kernel<<<wxx::grid_for(n, kT), kT, 0, wxx::stream()>>>(p, g, m, v, n, lr, beta1, beta2,
                                                               eps, weight_decay, 1.f, 1.f, bc);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// wxx_adamw_device over n parameters with one launch per 128 of them: p[i],
// g[i], m[i], v[i] (host arrays of device pointers) of len[i] elements each.
WXX_EXPORT int wxx_adamw_device_multi(int n, float* const* p, const float* const* g,
                                      float* const* m, float* const* v, const int64_t* len,
                                      float lr, float beta1, float beta2, float eps,
                                      float weight_decay, const float* bc) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 0 && bc != nullptr, "wxx_adamw_device_multi: bad count or no bias corrections");
  int i = 0;
  while (i < n) {
    AdamwTable tab;
    memset(&tab, 0, sizeof(tab));
    int64_t chunks = 0;
    for (; i < n && tab.n < kAdamwMulti; ++i) {
      WXX_REQUIRE(len[i] >= 0 && p[i] && g[i] && m[i] && v[i],
                  "wxx_adamw_device_multi: tensor %d has a NULL pointer or negative size", i);
      if (len[i] == 0) continue;
      const int k = tab.n++;
      tab.start[k] = chunks;
      tab.p[k] = p[i];
      tab.g[k] = g[i];
      tab.m[k] = m[i];
      tab.v[k] = v[i];
      tab.len[k] = len[i];
      chunks += (len[i] + kAdamwChunk - 1) / kAdamwChunk;
    }
    if (tab.n == 0) continue;
    tab.start[tab.n] = chunks;
    WXX_REQUIRE(chunks < (int64_t(1) << 31), "wxx_adamw_device_multi: too many elements");
    adamw_multi_kernel<<<(unsigned)chunks, kT, 0, wxx::stream()>>>(tab, lr, beta1, beta2, eps,
                                                                   weight_decay, bc);
    WXX_LAUNCH_CHECK();
  }
  return WXX_OK;
}

// Advances an optimizer's device step counter (one int) and writes the// Advances an optimizer's device step counter (one int) and writes the
// step's bias corrections {1 - beta1^t, 1 - beta2^t} into bc (two floats).
WXX_EXPORT int wxx_adamw_advance(int* step, float* bc, double beta1, double beta2) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(step != nullptr && bc != nullptr, "wxx_adamw_advance: NULL pointer");
  adamw_advance_kernel<<<1, 1, 0, wxx::stream()>>>(step, bc, beta1, beta2);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
