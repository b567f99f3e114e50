// Elementwise, copy, gather and small stencil kernels (HBM-bound).
//
// Reference kernels restated (semantics kept, code our own):
//   pointwise.wgsl (broadcast strided add/sub/mul/div, functional/pointwise.py:29-98)
//   _pointwise.wgsl (in-place accumulate, functional/pointwise.py:232-291)
//   scalarpointwise.wgsl (functional/pointwise.py:101-146)
//   relu/gelu/sigmoid/sin/cos/selu + exp/log/sqrt/rsqrt/abs/sign/negate/square
//     (functional/activations.py:22-120, functional/pointwise.py:294-355)
//   contiguous.wgsl / assign.wgsl (functional/utils.py:29-101, 316-369)
//   embed.wgsl (functional/layers.py:161-206)
//   causal_conv1d.wgsl (functional/convolution.py:1188-1257)
//   decay_window.wgsl (functional/pointwise.py:357-404)
//   complex_mul.wgsl (functional/fft.py:168-213)
//
// Layout: all tensors are dense fp32 (or u32 / interleaved c64) in HBM; views
// are described by (offset, shape, stride) in elements.  Host code collapses
// mergeable dimensions before launch so most launches are rank 1-3 with
// 32-bit index arithmetic; a 64-bit path covers views beyond 2^31 elements.
#include "common.cuh"

#include <cmath>
#include <cstring>

namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------ strided index

template <typename Idx>
struct Dims {
  int rank;
  Idx shape[WXX_MAX_RANK];
  Idx sa[WXX_MAX_RANK];
  Idx sb[WXX_MAX_RANK];
  Idx oa, ob;
};

template <typename Idx>
__device__ __forceinline__ void offsets_of(const Dims<Idx>& d, Idx i, Idx& pa, Idx& pb) {
  Idx a = d.oa, b = d.ob;
#pragma unroll
  for (int k = WXX_MAX_RANK - 1; k >= 0; --k) {
    if (k < d.rank) {
      Idx s = d.shape[k];
      Idx c = i % s;
      i /= s;
      a += c * d.sa[k];
      b += c * d.sb[k];
    }
  }
  pa = a;
  pb = b;
}

// Collapses adjacent dimensions that are contiguous for both operands and drops
// size-1 dimensions.  Returns the new rank.
int collapse(int rank, int64_t* shape, int64_t* sa, int64_t* sb) {
  int64_t s2[WXX_MAX_RANK], a2[WXX_MAX_RANK], b2[WXX_MAX_RANK];
  int r = 0;
  for (int k = 0; k < rank; ++k) {
    if (shape[k] == 1) continue;
    if (r > 0 && sa[k] * shape[k] == a2[r - 1] && sb[k] * shape[k] == b2[r - 1]) {
      s2[r - 1] *= shape[k];
      a2[r - 1] = sa[k];
      b2[r - 1] = sb[k];
    } else {
      s2[r] = shape[k];
      a2[r] = sa[k];
      b2[r] = sb[k];
      ++r;
    }
  }
  if (r == 0) {
    s2[0] = 1;
    a2[0] = 0;
    b2[0] = 0;
    r = 1;
  }
  for (int k = 0; k < r; ++k) {
    shape[k] = s2[k];
    sa[k] = a2[k];
    sb[k] = b2[k];
  }
  return r;
}

bool fits32(int rank, const int64_t* shape, const int64_t* sa, const int64_t* sb, int64_t oa,
            int64_t ob, int64_t numel) {
  if (numel >= (int64_t(1) << 31)) return false;
  int64_t ma = oa, mb = ob;
  for (int k = 0; k < rank; ++k) {
    ma += (shape[k] - 1) * sa[k];
    mb += (shape[k] - 1) * sb[k];
  }
  return ma < (int64_t(1) << 31) && mb < (int64_t(1) << 31) && oa >= 0 && ob >= 0;
}

template <typename Idx>
Dims<Idx> make_dims(int rank, const int64_t* shape, const int64_t* sa, const int64_t* sb,
                    int64_t oa, int64_t ob) {
  Dims<Idx> d;
  memset(&d, 0, sizeof(d));
  d.rank = rank;
  for (int k = 0; k < rank; ++k) {
    d.shape[k] = (Idx)shape[k];
    d.sa[k] = (Idx)sa[k];
    d.sb[k] = (Idx)sb[k];
  }
  d.oa = (Idx)oa;
  d.ob = (Idx)ob;
  return d;
}

// ------------------------------------------------------------ binary ops

__device__ __forceinline__ float apply_binary(int op, float a, float b) {
  switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    case 3: return a / b;
    default: return a + b;
  }
}

template <typename Idx>
__global__ void binary_strided_kernel(float* __restrict__ out, const float* a, const float* b,
                                      Dims<Idx> d, Idx numel, int op) {
  for (Idx i = (Idx)blockIdx.x * blockDim.x + threadIdx.x; i < numel;
       i += (Idx)gridDim.x * blockDim.x) {
    Idx pa, pb;
    offsets_of(d, i, pa, pb);
    out[i] = apply_binary(op, a[pa], b[pb]);
  }
}

// Both operands dense with the output's shape: 128-bit loads and stores.
__global__ void binary_dense_vec4_kernel(float4* __restrict__ out, const float4* a,
                                         const float4* b, int64_t n4, int op) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 x = a[i], y = b[i], r;
    r.x = apply_binary(op, x.x, y.x);
    r.y = apply_binary(op, x.y, y.y);
    r.z = apply_binary(op, x.z, y.z);
    r.w = apply_binary(op, x.w, y.w);
    out[i] = r;
  }
}

// a dense, b broadcast along rows: out[r, c] = a[r, c] op b[c]  (bias, mask).
__global__ void binary_row_bcast_kernel(float* __restrict__ out, const float* __restrict__ a,
                                        const float* __restrict__ b, int64_t rows, int cols,
                                        int64_t b_row_period, int op) {
  int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / cols;
    int c = (int)(i - r * cols);
    out[i] = apply_binary(op, a[i], b[(r % b_row_period) * cols + c]);
  }
}

// ------------------------------------------------------------ scalar / unary

__device__ __forceinline__ float apply_scalar(int op, float x, float c, int reverse) {
  switch (op) {
    case 0: return x + c;
    case 1: return reverse ? c - x : x - c;
    case 2: return x * c;
    case 3:
      if (reverse) return powf(c, x);
      if (x < 0.0f) {
        if (c == truncf(c)) {
          float mag = powf(-x, c);
          bool odd = fmodf(fabsf(c), 2.0f) == 1.0f;
          return odd ? -mag : mag;
        }
        return __int_as_float(0x7fc00000);
      }
      return powf(x, c);
    case 4: return reverse ? c / x : x / c;
    case 5: return x != 0.0f ? x : c;  // masked fill of zeros (maskedfill.wgsl)
    default: return x;
  }
}

__global__ void clamp_kernel(float* __restrict__ out, const float* __restrict__ x, int64_t n,
                             float lo, float hi) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = fminf(fmaxf(x[i], lo), hi);
}

__device__ __forceinline__ float apply_unary(int op, float x) {
  switch (op) {
    case 0: return fmaxf(0.0f, x);                                    // relu
    case 1: return gelu_tanh(x);                                      // gelu (tanh form)
    case 2: {                                                         // sigmoid
      float xc = fminf(fmaxf(x, -88.0f), 88.0f);
      return 1.0f / (1.0f + expf(-xc));
    }
    case 3: return sinf(x);
    case 4: return cosf(x);
    case 5: return expf(x);
    case 6: return logf(x);
    case 7: return sqrtf(x);
    case 8: return rsqrtf(x);
    case 9: return fabsf(x);
    case 10: return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);     // sign
    case 11: return -x;
    case 12: return x * x;
    case 13: return silu_lib(x);                                      // silu = sigmoid(x) * x
    case 14: {                                                        // selu
      const float alpha = 1.6732632423543772848170429916717f;
      const float scale = 1.0507009873554804934193349852946f;
      return x > 0.0f ? scale * x : scale * alpha * (expf(x) - 1.0f);
    }
    default: return x;
  }
}

__global__ void scalar_kernel(float* __restrict__ out, const float* __restrict__ x, int64_t n,
                              int op, float c, int reverse) {
  int64_t n4 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) ? 0 : n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* o4 = reinterpret_cast<float4*>(out);
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n4; i += step) {
    float4 v = x4[i];
    v.x = apply_scalar(op, v.x, c, reverse);
    v.y = apply_scalar(op, v.y, c, reverse);
    v.z = apply_scalar(op, v.z, c, reverse);
    v.w = apply_scalar(op, v.w, c, reverse);
    o4[i] = v;
  }
  for (int64_t i = n4 * 4 + tid; i < n; i += step) out[i] = apply_scalar(op, x[i], c, reverse);
}

__global__ void unary_kernel(float* __restrict__ out, const float* __restrict__ x, int64_t n,
                             int op) {
  int64_t n4 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) ? 0 : n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* o4 = reinterpret_cast<float4*>(out);
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n4; i += step) {
    float4 v = x4[i];
    v.x = apply_unary(op, v.x);
    v.y = apply_unary(op, v.y);
    v.z = apply_unary(op, v.z);
    v.w = apply_unary(op, v.w);
    o4[i] = v;
  }
  for (int64_t i = n4 * 4 + tid; i < n; i += step) out[i] = apply_unary(op, x[i]);
}

// ------------------------------------------------------------ copies

// dst (strided, stride_a/offset_a) <- src (strided, stride_b/offset_b), for
// 4-byte or 8-byte elements.  A dense dst is the `contiguous` kernel.
template <typename T, typename Idx>
__global__ void strided_copy_kernel(T* dst, const T* src, Dims<Idx> d, Idx numel) {
  for (Idx i = (Idx)blockIdx.x * blockDim.x + threadIdx.x; i < numel;
       i += (Idx)gridDim.x * blockDim.x) {
    Idx pd, ps;
    offsets_of(d, i, pd, ps);
    dst[pd] = src[ps];
  }
}

template <typename T, typename Idx>
__global__ void strided_fill_kernel(T* dst, T value, Dims<Idx> d, Idx numel) {
  for (Idx i = (Idx)blockIdx.x * blockDim.x + threadIdx.x; i < numel;
       i += (Idx)gridDim.x * blockDim.x) {
    Idx pd, ps;
    offsets_of(d, i, pd, ps);
    dst[pd] = value;
  }
}

// 2-D transpose through shared memory: dst[c, r] = src[r, c] for a batch of
// (rows x cols) planes.  Used by `contiguous` on a swapped pair of dims.
__global__ void transpose_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                 int64_t batch, int rows, int cols, int64_t src_batch_stride,
                                 int64_t src_row_stride, int64_t src_offset) {
  __shared__ float tile[32][33];
  int64_t b = blockIdx.z;
  int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* s = src + src_offset + b * src_batch_stride;
  float* d = dst + b * (int64_t)rows * cols;
  for (int k = threadIdx.y; k < 32; k += 8) {
    int r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[k][threadIdx.x] = s[(int64_t)r * src_row_stride + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) {
    int c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) d[(int64_t)c * rows + r] = tile[threadIdx.x][k];
  }
}

// Stacked transposes in one launch: dst[b * cols + c, r] = src_b[r, c] for up
// to 8 dense (rows x cols) sources (blockIdx.z = b).  Builds the K-major
// (n * N, K) operand of a fused projection from n nn.Linear (K, N) weights.
struct StackSrc {
  const float* p[8];
};

__global__ void transpose_stack_kernel(float* __restrict__ dst, StackSrc srcs, int rows,
                                       int cols, int round_tf32) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* s = srcs.p[b];
  float* d = dst + (int64_t)b * rows * cols;
  for (int k = threadIdx.y; k < 32; k += 8) {
    int r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[k][threadIdx.x] = __ldg(s + (int64_t)r * cols + c);
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) {
    int c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) {
      const float v = tile[threadIdx.x][k];
      d[(int64_t)c * rows + r] = round_tf32 ? tf32_rna(v) : v;
    }
  }
}

// ------------------------------------------------------------ embed

// out[t, :] = W[ids[t], :]; one warp-row of float4 per token.  Ids outside the
// table write zeros and raise WXX_DEV_ERR_BAD_INDEX.
__global__ void embed_kernel(float* __restrict__ out, const uint32_t* __restrict__ ids,
                             const float* __restrict__ w, int64_t n_tokens, int dim,
                             uint32_t vocab, int* err) {
  bool vec = (dim % 4 == 0) && !((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15);
  int64_t total = vec ? n_tokens * (dim / 4) : n_tokens * dim;
  int per = vec ? dim / 4 : dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i / per;
    int c = (int)(i - t * per);
    uint32_t id = ids[t];
    if (vec) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (id < vocab) v = reinterpret_cast<const float4*>(w + (int64_t)id * dim)[c];
      else if (c == 0) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
      reinterpret_cast<float4*>(out + t * dim)[c] = v;
    } else {
      float v = 0.f;
      if (id < vocab) v = w[(int64_t)id * dim + c];
      else if (c == 0) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
      out[t * dim + c] = v;
    }
  }
}

// ------------------------------------------------------------ causal conv1d

// out[b, d, n] = bias[d] + sum_k w[d, k] * x[b, d, n - k]   (n - k >= 0)
// x is a strided (B, D, L) view; out is dense (B, D, L).  Threads run along L
// for coalesced writes; when x is the (B, L, D)->(B, D, L) transpose the reads
// are strided by D and are served by L2 (each input element is reused K times).
__global__ void causal_conv1d_kernel(float* __restrict__ out, const float* __restrict__ x,
                                     int64_t x_off, int64_t sb, int64_t sc, int64_t sl,
                                     const float* __restrict__ w, const float* __restrict__ bias,
                                     int B, int D, int L, int K) {
  int64_t total = (int64_t)B * D * L;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int n = (int)(i % L);
    int64_t rest = i / L;
    int d = (int)(rest % D);
    int b = (int)(rest / D);
    const float* xp = x + x_off + (int64_t)b * sb + (int64_t)d * sc;
    float acc = bias[d];
    for (int k = 0; k < K; ++k) {
      if (n >= k) acc = acc + w[d * K + k] * xp[(int64_t)(n - k) * sl];
    }
    out[i] = acc;
  }
}

// Transposed-input variant: x element (b, d, n) lives at x_off + b*sb + n*sl + d
// (sc == 1).  A CTA handles a 128(d) x 64(n) tile: the (64 + K - 1) input rows
// of 128 channels (512 contiguous bytes each) are read into shared memory
// with row pitch 129, so both the row stores (lanes along d) and the column
// reads (lanes along n) hit 32 distinct banks.  Warp w then produces channels
// 16w .. 16w+15, each lane two positions 32 apart, written coalesced along n;
// a channel's K taps are warp-uniform loads.
constexpr int kConvTileD = 128;
constexpr int kConvTileN = 64;
constexpr int kConvPitch = kConvTileD + 1;
constexpr int kConvMaxK = 8;

__global__ void __launch_bounds__(256) causal_conv1d_tr_kernel(
    float* __restrict__ out, const float* __restrict__ x, int64_t x_off, int64_t sb, int64_t sl,
    const float* __restrict__ w, const float* __restrict__ bias, int B, int D, int L, int K) {
  extern __shared__ float tile[];  // (kConvTileN + K - 1) x kConvPitch
  const int b = blockIdx.z;
  const int d0 = blockIdx.y * kConvTileD, n0 = blockIdx.x * kConvTileN;
  const int rows = kConvTileN + K - 1;
  const float* xb = x + x_off + (int64_t)b * sb;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // all of this warp's rows (at most kRowsPerWarp) loaded before any store:
  // up to 36 loads in flight per thread
  constexpr int kRowsPerWarp = (kConvTileN + kConvMaxK - 1 + 7) / 8;
  float vals[kRowsPerWarp][kConvTileD / 32];
#pragma unroll
  for (int it = 0; it < kRowsPerWarp; ++it) {
    const int r = warp + 8 * it;
    const int n = n0 - (K - 1) + r;
    const bool in = r < rows && n >= 0 && n < L;
    const float* xr = xb + (int64_t)n * sl + d0;
#pragma unroll
    for (int j = 0; j < kConvTileD / 32; ++j) {
      const int dd = 32 * j + lane;
      vals[it][j] = (in && d0 + dd < D) ? __ldg(xr + dd) : 0.f;
    }
  }
#pragma unroll
  for (int it = 0; it < kRowsPerWarp; ++it) {
    const int r = warp + 8 * it;
    if (r < rows) {
#pragma unroll
      for (int j = 0; j < kConvTileD / 32; ++j) tile[r * kConvPitch + 32 * j + lane] = vals[it][j];
    }
  }
  __syncthreads();
#pragma unroll 4
  for (int c = 0; c < kConvTileD / 8; ++c) {
    const int dd = warp * (kConvTileD / 8) + c;
    const int dc = d0 + dd;
    if (dc >= D) break;
    float wk[kConvMaxK];
#pragma unroll
    for (int k = 0; k < kConvMaxK; ++k) wk[k] = k < K ? __ldg(w + dc * K + k) : 0.f;
    const float bv = __ldg(bias + dc);
    float* orow = out + ((int64_t)b * D + dc) * L;
#pragma unroll
    for (int q = 0; q < kConvTileN / 32; ++q) {
      const int i = lane + 32 * q;  // position inside the tile
      const int n = n0 + i;
      if (n >= L) continue;
      float acc = bv;
#pragma unroll
      for (int k = 0; k < kConvMaxK; ++k)
        if (k < K && n >= k) acc = acc + wk[k] * tile[(i + K - 1 - k) * kConvPitch + dd];
      orow[n] = acc;
    }
  }
}

// ------------------------------------------------------------ decay window

// W[d, t] = exp(-|decay[stage, d]| * t)
__global__ void decay_window_kernel(float* __restrict__ out, const float* __restrict__ decay,
                                    int channels, int length, int stage) {
  int64_t total = (int64_t)channels * length;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int t = (int)(i % length);
    int d = (int)(i / length);
    float rate = decay[(int64_t)stage * channels + d];
    out[i] = expf(-fabsf(rate) * (float)t);
  }
}

// ------------------------------------------------------------ complex multiply

template <typename Idx>
__global__ void complex_mul_kernel(float2* __restrict__ out, const float2* a, const float2* b,
                                   Dims<Idx> d, Idx numel, int conj_a, int conj_b) {
  for (Idx i = (Idx)blockIdx.x * blockDim.x + threadIdx.x; i < numel;
       i += (Idx)gridDim.x * blockDim.x) {
    Idx pa, pb;
    offsets_of(d, i, pa, pb);
    float2 x = a[pa], y = b[pb];
    if (conj_a) x.y = -x.y;
    if (conj_b) y.y = -y.y;
    out[i] = make_float2(x.x * y.x - x.y * y.y, x.x * y.y + x.y * y.x);
  }
}

__global__ void complex_conj_kernel(float2* __restrict__ out, const float2* __restrict__ x,
                                    int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float2 v = x[i];
    out[i] = make_float2(v.x, -v.y);
  }
}

__global__ void complex_add_inplace_kernel(float2* __restrict__ acc, const float2* __restrict__ x,
                                           int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float2 a = acc[i], v = x[i];
    acc[i] = make_float2(a.x + v.x, a.y + v.y);
  }
}

// ------------------------------------------------------------ equality / masked fill

__global__ void equal_kernel(float* __restrict__ out, const uint32_t* __restrict__ a,
                             const uint32_t* __restrict__ b, int64_t n, int mode, uint32_t number) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    bool eq;
    switch (mode) {
      case 0: eq = __uint_as_float(a[i]) == __uint_as_float(b[i]); break;
      case 1: eq = a[i] == b[i]; break;
      case 2: eq = __uint_as_float(a[i]) == __uint_as_float(number); break;
      default: eq = a[i] == number; break;
    }
    out[i] = eq ? 1.0f : 0.0f;
  }
}

int check_rank(int rank) {
  if (rank < 0 || rank > WXX_MAX_RANK) {
    wxx::set_error("rank %d outside [0, %d]", rank, WXX_MAX_RANK);
    return WXX_E_ARG;
  }
  return WXX_OK;
}

}  // namespace

// ============================================================ exports

// out (dense, numel) = a op b with broadcast strided operands.
// shape/stride_a/stride_b have `rank` entries (element units).  op: 0 add,
// 1 sub, 2 mul, 3 div.  `out` may alias `a` when a is dense (in-place
// accumulate, the reference's _pointwise).
WXX_EXPORT int wxx_binary(float* out, const float* a, int64_t a_off, const int64_t* stride_a,
                          const float* b, int64_t b_off, const int64_t* stride_b, int rank,
                          const int64_t* shape, int op) {
  WXX_REQUIRE_INIT();
  if (check_rank(rank)) return WXX_E_ARG;
  WXX_REQUIRE(op >= 0 && op <= 3, "wxx_binary: op %d not in 0..3", op);
  int64_t sh[WXX_MAX_RANK], sa[WXX_MAX_RANK], sb[WXX_MAX_RANK];
  int64_t numel = 1;
  for (int k = 0; k < rank; ++k) {
    sh[k] = shape[k];
    sa[k] = stride_a[k];
    sb[k] = stride_b[k];
    WXX_REQUIRE(sh[k] >= 0, "wxx_binary: negative dim");
    numel *= sh[k];
  }
  if (numel == 0) return WXX_OK;
  int r = collapse(rank, sh, sa, sb);
  cudaStream_t s = wxx::stream();
  // Dense fast path.
  if (r == 1 && sa[0] == 1 && sb[0] == 1 && numel % 4 == 0 &&
      !(((uintptr_t)(out) | (uintptr_t)(a + a_off) | (uintptr_t)(b + b_off)) & 15)) {
    binary_dense_vec4_kernel<<<wxx::grid_for(numel / 4, kThreads), kThreads, 0, s>>>(
        (float4*)out, (const float4*)(a + a_off), (const float4*)(b + b_off), numel / 4, op);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  // a dense, b a dense row vector / matrix repeated over leading rows.
  if (r == 2 && sa[1] == 1 && sa[0] == sh[1] && sb[1] == 1 && (sb[0] == 0)) {
    binary_row_bcast_kernel<<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        out, a + a_off, b + b_off, sh[0], (int)sh[1], 1, op);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  if (fits32(r, sh, sa, sb, a_off, b_off, numel)) {
    auto d = make_dims<int32_t>(r, sh, sa, sb, a_off, b_off);
    binary_strided_kernel<int32_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        out, a, b, d, (int32_t)numel, op);
  } else {
    auto d = make_dims<int64_t>(r, sh, sa, sb, a_off, b_off);
    binary_strided_kernel<int64_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        out, a, b, d, numel, op);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out = x op c (reverse: c op x), dense.  op: 0 add, 1 sub, 2 mul, 3 pow, 4 div,
// 5 masked fill (x != 0 ? x : c).
WXX_EXPORT int wxx_scalar(float* out, const float* x, int64_t n, int op, float c, int reverse) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(op >= 0 && op <= 5, "wxx_scalar: op %d not in 0..5", op);
  if (n <= 0) return WXX_OK;
  scalar_kernel<<<wxx::grid_for(n / 4 + 1, kThreads), kThreads, 0, wxx::stream()>>>(out, x, n, op, c,
                                                                                  reverse);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out = clamp(x, lo, hi), dense (clamp.wgsl, functional/pointwise.py:149-178).
WXX_EXPORT int wxx_clamp(float* out, const float* x, int64_t n, float lo, float hi) {
  WXX_REQUIRE_INIT();
  if (n <= 0) return WXX_OK;
  clamp_kernel<<<wxx::grid_for(n, kThreads), kThreads, 0, wxx::stream()>>>(out, x, n, lo, hi);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out = f(x), dense.  op: 0 relu, 1 gelu(tanh), 2 sigmoid, 3 sin, 4 cos, 5 exp,
// 6 log, 7 sqrt, 8 rsqrt, 9 abs, 10 sign, 11 negate, 12 square, 13 silu, 14 selu.
WXX_EXPORT int wxx_unary(float* out, const float* x, int64_t n, int op) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(op >= 0 && op <= 14, "wxx_unary: op %d not in 0..14", op);
  if (n <= 0) return WXX_OK;
  unary_kernel<<<wxx::grid_for(n / 4 + 1, kThreads), kThreads, 0, wxx::stream()>>>(out, x, n, op);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// dst[dst_off + sum(i_k * dst_stride_k)] = src[src_off + sum(i_k * src_stride_k)]
// over `shape`; elem_bytes is 4 (f32/u32) or 8 (c64).  A dense dst with
// contiguous strides is the reference's `contiguous`; a strided dst is `assign`.
WXX_EXPORT int wxx_strided_copy(void* dst, int64_t dst_off, const int64_t* dst_stride,
                                const void* src, int64_t src_off, const int64_t* src_stride,
                                int rank, const int64_t* shape, int elem_bytes) {
  WXX_REQUIRE_INIT();
  if (check_rank(rank)) return WXX_E_ARG;
  WXX_REQUIRE(elem_bytes == 4 || elem_bytes == 8, "wxx_strided_copy: elem_bytes must be 4 or 8");
  int64_t sh[WXX_MAX_RANK], sa[WXX_MAX_RANK], sb[WXX_MAX_RANK];
  int64_t numel = 1;
  for (int k = 0; k < rank; ++k) {
    sh[k] = shape[k];
    sa[k] = dst_stride[k];
    sb[k] = src_stride[k];
    numel *= sh[k];
  }
  if (numel == 0) return WXX_OK;
  int r = collapse(rank, sh, sa, sb);
  cudaStream_t s = wxx::stream();
  if (r == 1 && sa[0] == 1 && sb[0] == 1) {
    WXX_CUDA_CHECK(cudaMemcpyAsync((char*)dst + dst_off * elem_bytes,
                                   (const char*)src + src_off * elem_bytes, numel * elem_bytes,
                                   cudaMemcpyDeviceToDevice, s));
    return WXX_OK;
  }
  // Batched 2-D transpose.  Logical view (batch, I, J) with a dense
  // destination (strides J, 1) and a source that is unit-stride along I:
  // element (b, i, j) sits at src[b*sb0 + j*sbJ + i].  The source is then a
  // plane of J rows x I columns, transposed through shared memory.
  if (elem_bytes == 4 && r >= 2 && r <= 3 && sa[r - 1] == 1 && sa[r - 2] == sh[r - 1] &&
      sb[r - 2] == 1 && sb[r - 1] >= sh[r - 2] && (r == 2 || sa[0] == sh[1] * sh[2]) &&
      sh[r - 1] < (1 << 30) && sh[r - 2] < (1 << 30)) {
    int I = (int)sh[r - 2], J = (int)sh[r - 1];
    int64_t batch = r == 3 ? sh[0] : 1;
    int64_t sbatch = r == 3 ? sb[0] : 0;
    if (batch <= 65535) {
      dim3 grid((I + 31) / 32, (J + 31) / 32, (unsigned)batch);
      transpose_kernel<<<grid, dim3(32, 8), 0, s>>>((float*)dst + dst_off, (const float*)src, batch,
                                                   J, I, sbatch, sb[r - 1], src_off);
      WXX_LAUNCH_CHECK();
      return WXX_OK;
    }
  }
  bool small = fits32(r, sh, sa, sb, dst_off, src_off, numel);
  if (elem_bytes == 4) {
    if (small) {
      auto d = make_dims<int32_t>(r, sh, sa, sb, dst_off, src_off);
      strided_copy_kernel<uint32_t, int32_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
          (uint32_t*)dst, (const uint32_t*)src, d, (int32_t)numel);
    } else {
      auto d = make_dims<int64_t>(r, sh, sa, sb, dst_off, src_off);
      strided_copy_kernel<uint32_t, int64_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
          (uint32_t*)dst, (const uint32_t*)src, d, numel);
    }
  } else {
    if (small) {
      auto d = make_dims<int32_t>(r, sh, sa, sb, dst_off, src_off);
      strided_copy_kernel<uint2, int32_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
          (uint2*)dst, (const uint2*)src, d, (int32_t)numel);
    } else {
      auto d = make_dims<int64_t>(r, sh, sa, sb, dst_off, src_off);
      strided_copy_kernel<uint2, int64_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
          (uint2*)dst, (const uint2*)src, d, numel);
    }
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Fills a strided 4-byte-element view with the bit pattern `value_bits`.
WXX_EXPORT int wxx_strided_fill(void* dst, int64_t dst_off, const int64_t* dst_stride, int rank,
                                const int64_t* shape, uint32_t value_bits) {
  WXX_REQUIRE_INIT();
  if (check_rank(rank)) return WXX_E_ARG;
  int64_t sh[WXX_MAX_RANK], sa[WXX_MAX_RANK], sb[WXX_MAX_RANK];
  int64_t numel = 1;
  for (int k = 0; k < rank; ++k) {
    sh[k] = shape[k];
    sa[k] = dst_stride[k];
    sb[k] = 0;
    numel *= sh[k];
  }
  if (numel == 0) return WXX_OK;
  int r = collapse(rank, sh, sa, sb);
  cudaStream_t s = wxx::stream();
  if (fits32(r, sh, sa, sb, dst_off, 0, numel)) {
    auto d = make_dims<int32_t>(r, sh, sa, sb, dst_off, 0);
    strided_fill_kernel<uint32_t, int32_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        (uint32_t*)dst, value_bits, d, (int32_t)numel);
  } else {
    auto d = make_dims<int64_t>(r, sh, sa, sb, dst_off, 0);
    strided_fill_kernel<uint32_t, int64_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        (uint32_t*)dst, value_bits, d, numel);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out[t, :] = weight[ids[t], :] for t < n_tokens (dense, fp32 rows of `dim`).
WXX_EXPORT int wxx_embed(float* out, const uint32_t* ids, const float* weight, int64_t n_tokens,
                         int dim, uint32_t vocab) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(dim > 0, "wxx_embed: dim must be positive");
  if (n_tokens <= 0) return WXX_OK;
  int64_t work = n_tokens * ((dim % 4 == 0) ? dim / 4 : dim);
  embed_kernel<<<wxx::grid_for(work, kThreads), kThreads, 0, wxx::stream()>>>(
      out, ids, weight, n_tokens, dim, vocab, wxx::device_error_word());
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Depthwise causal conv over a strided (B, D, L) view x (element strides
// sb, sc, sl from offset x_off); w (D, K), bias (D,), out dense (B, D, L).
WXX_EXPORT int wxx_causal_conv1d(float* out, const float* x, int64_t x_off, int64_t sb,
                                 int64_t sc, int64_t sl, const float* w, const float* bias, int B,
                                 int D, int L, int K) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B >= 0 && D >= 0 && L >= 0 && K >= 1, "wxx_causal_conv1d: bad sizes");
  if ((int64_t)B * D * L == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  if (sc == 1 && K <= kConvMaxK && B <= 65535) {
    dim3 grid((L + kConvTileN - 1) / kConvTileN, (D + kConvTileD - 1) / kConvTileD, B);
    size_t smem = (size_t)(kConvTileN + K - 1) * kConvPitch * sizeof(float);
    causal_conv1d_tr_kernel<<<grid, 256, smem, s>>>(out, x, x_off, sb, sl, w, bias, B, D, L, K);
  } else {
    int64_t total = (int64_t)B * D * L;
    causal_conv1d_kernel<<<wxx::grid_for(total, kThreads), kThreads, 0, s>>>(
        out, x, x_off, sb, sc, sl, w, bias, B, D, L, K);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// dst (n * cols, rows) dense = the transposes of n dense (rows, cols) sources
// stacked along dst's rows; srcs is a host array of n device pointers, n <= 8.
// round_tf32 = 1 stores the values rounded to the nearest TF32 value (a copy
// read only as a TF32 GEMM operand).
WXX_EXPORT int wxx_transpose_stack(float* dst, const float* const* srcs, int n, int rows,
                                   int cols, int round_tf32) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 1 && n <= 8 && rows >= 0 && cols >= 0 && srcs != nullptr,
              "wxx_transpose_stack: n %d not in 1..8 or bad sizes", n);
  if ((int64_t)rows * cols == 0) return WXX_OK;
  StackSrc ss;
  memset(&ss, 0, sizeof(ss));
  for (int i = 0; i < n; ++i) {
    WXX_REQUIRE(srcs[i] != nullptr, "wxx_transpose_stack: source %d is NULL", i);
    ss.p[i] = srcs[i];
  }
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)n);
  WXX_REQUIRE(grid.y <= 65535, "wxx_transpose_stack: %d rows exceed the grid", rows);
  transpose_stack_kernel<<<grid, dim3(32, 8), 0, wxx::stream()>>>(dst, ss, rows, cols,
                                                                 round_tf32 ? 1 : 0);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

namespace {
// dst[i] = src[i] rounded to the nearest TF32 value (16-byte vectors when
// both are aligned and n % 4 == 0).
__global__ void round_tf32_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                  int64_t n) {
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) ==
                   0 && (n & 3) == 0;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
      float4 v = reinterpret_cast<const float4*>(src)[i];
      v = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
      reinterpret_cast<float4*>(dst)[i] = v;
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
      dst[i] = tf32_rna(src[i]);
  }
}
}  // namespace

// dst[0..n) = src[0..n) rounded to the nearest TF32 value: a weight copy read
// only by TF32 products (e.g. the tied LM head).
WXX_EXPORT int wxx_round_tf32(float* dst, const float* src, int64_t n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 0, "wxx_round_tf32: negative size");
  if (n == 0) return WXX_OK;
  round_tf32_kernel<<<wxx::grid_for(n / 4 + 1, kThreads), kThreads, 0, wxx::stream()>>>(dst, src,
                                                                                       n);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out (channels, length) = exp(-|decay[stage, d]| * t)
WXX_EXPORT int wxx_decay_window(float* out, const float* decay, int rows, int channels, int length,
                                int stage) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(stage >= 0 && stage < rows, "wxx_decay_window: stage %d outside [0, %d)", stage, rows);
  int64_t total = (int64_t)channels * length;
  if (total == 0) return WXX_OK;
  decay_window_kernel<<<wxx::grid_for(total, kThreads), kThreads, 0, wxx::stream()>>>(
      out, decay, channels, length, stage);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out (dense c64, numel of shape) = a * b with broadcast strided c64 operands
// (strides in complex elements); conj flags conjugate an operand first.
WXX_EXPORT int wxx_complex_mul(void* out, const void* a, int64_t a_off, const int64_t* stride_a,
                               const void* b, int64_t b_off, const int64_t* stride_b, int rank,
                               const int64_t* shape, int conj_a, int conj_b) {
  WXX_REQUIRE_INIT();
  if (check_rank(rank)) return WXX_E_ARG;
  int64_t sh[WXX_MAX_RANK], sa[WXX_MAX_RANK], sb[WXX_MAX_RANK];
  int64_t numel = 1;
  for (int k = 0; k < rank; ++k) {
    sh[k] = shape[k];
    sa[k] = stride_a[k];
    sb[k] = stride_b[k];
    numel *= sh[k];
  }
  if (numel == 0) return WXX_OK;
  int r = collapse(rank, sh, sa, sb);
  cudaStream_t s = wxx::stream();
  if (fits32(r, sh, sa, sb, a_off, b_off, numel)) {
    auto d = make_dims<int32_t>(r, sh, sa, sb, a_off, b_off);
    complex_mul_kernel<int32_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        (float2*)out, (const float2*)a, (const float2*)b, d, (int32_t)numel, conj_a, conj_b);
  } else {
    auto d = make_dims<int64_t>(r, sh, sa, sb, a_off, b_off);
    complex_mul_kernel<int64_t><<<wxx::grid_for(numel, kThreads), kThreads, 0, s>>>(
        (float2*)out, (const float2*)a, (const float2*)b, d, numel, conj_a, conj_b);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

WXX_EXPORT int wxx_complex_conj(void* out, const void* x, int64_t n) {
  WXX_REQUIRE_INIT();
  if (n <= 0) return WXX_OK;
  complex_conj_kernel<<<wxx::grid_for(n, kThreads), kThreads, 0, wxx::stream()>>>(
      (float2*)out, (const float2*)x, n);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

WXX_EXPORT int wxx_complex_add_inplace(void* acc, const void* x, int64_t n) {
  WXX_REQUIRE_INIT();
  if (n <= 0) return WXX_OK;
  complex_add_inplace_kernel<<<wxx::grid_for(n, kThreads), kThreads, 0, wxx::stream()>>>(
      (float2*)acc, (const float2*)x, n);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// out = (a == b) as 1.0 / 0.0.  mode 0 f32/f32, 1 u32/u32, 2 f32/scalar bits,
// 3 u32/scalar (functional/utils.py:509-582).
WXX_EXPORT int wxx_equal(float* out, const void* a, const void* b, int64_t n, int mode,
                         uint32_t number) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(mode >= 0 && mode <= 3, "wxx_equal: mode %d not in 0..3", mode);
  if (n <= 0) return WXX_OK;
  equal_kernel<<<wxx::grid_for(n, kThreads), kThreads, 0, wxx::stream()>>>(
      out, (const uint32_t*)a, (const uint32_t*)(b ? b : a), n, mode, number);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
