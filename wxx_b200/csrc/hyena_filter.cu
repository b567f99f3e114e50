// Hyena implicit long-convolution filters, one launch per operator.
//
// The reference builds each of an operator's `order` filters from the
// positional encoding with a small MLP and a decay window
// (src/wxx/nn/hyena.py:127-130 ImplicitFilter.forward and :236-239):
//   h_i = (Linear2_i(sin(omega * Linear1_i(pe))))^T * exp(-|decay[i, d]| * t)
// which as separate ops is two small GEMMs, a scale, a sine, the window, the
// window product and a transpose -- seven launches per filter, each moving
// the (L, hidden) or (L, D) intermediate through HBM.  Here one kernel
// evaluates all filters of an operator in exact fp32 and writes h as
// (order, D, L), the layout the FFT convolution reads.
//
// Work split: a CTA owns 32 positions (one per lane) of one filter.
//  1. hidden[l][j] = sin(omega * (b1[j] + sum_k pe[l][k] W1[k][j])) for the
//     CTA's 32 positions, j spread over the 8 warps, into shared memory;
//  2. each lane loads its position's hidden row into registers;
//  3. W2 is staged transposed in shared memory 64 channels at a time; warp w
//     computes channels w, w+8, ... of the chunk: acc = sum_j hidden[j] W2[j][d]
//     with W2 read as warp-uniform (broadcast) 16-byte loads, then
//     (acc + b2[d]) * exp(-|decay[i, d]| * l), stored along l (one 128-byte
//     run per warp and channel).
// The sums run in index order with fused multiply-adds; the scale, sine,
// bias, window and product are the unfused ops' fp32 expressions.

#include "common.cuh"

#include <cstring>

namespace {

constexpr int kFiltMaxN = 8;      // filters per launch (the operator's order)
constexpr int kFiltMaxF = 32;     // positional features
constexpr int kFiltMaxH = 64;     // hidden width (held in registers per lane)
constexpr int kFiltChunk = 64;    // W2 channels staged per pass
constexpr int kFiltThreads = 256;

struct FilterWeights {
  const float* w1[kFiltMaxN];   // (F, H)
  const float* b1[kFiltMaxN];   // (H)
  const float* w2[kFiltMaxN];   // (H, D)
  const float* b2[kFiltMaxN];   // (D)
};

__global__ void __launch_bounds__(kFiltThreads) hyena_filter_kernel(
    float* __restrict__ out, const float* __restrict__ pe, int L, int F, int H, int D,
    FilterWeights fw, float omega, const float* __restrict__ decay) {
  __shared__ float pes[32][kFiltMaxF + 1];
  __shared__ float hs[32][kFiltMaxH + 1];
  __shared__ __align__(16) float w2s[kFiltChunk][kFiltMaxH + 4];
  const int f = blockIdx.y;
  const int l0 = blockIdx.x * 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* W1 = fw.w1[f];
  const float* B1 = fw.b1[f];
  const float* W2 = fw.w2[f];
  const float* B2 = fw.b2[f];

  // positional encoding rows of the CTA's positions (zero past L)
  for (int i = threadIdx.x; i < 32 * F; i += kFiltThreads) {
    const int r = i / F, k = i - r * F;
    pes[r][k] = l0 + r < L ? __ldg(pe + (int64_t)(l0 + r) * F + k) : 0.f;
  }
  __syncthreads();
  // 1. hidden layer
  for (int j = warp; j < H; j += kFiltThreads / 32) {
    float acc = 0.f;
    for (int k = 0; k < F; ++k) acc = fmaf(pes[lane][k], __ldg(W1 + (int64_t)k * H + j), acc);
    const float y = acc + __ldg(B1 + j);
    hs[lane][j] = sinf(y * omega);
  }
  __syncthreads();
  // 2. this lane's hidden row
  float hid[kFiltMaxH];
#pragma unroll
  for (int j = 0; j < kFiltMaxH; ++j) hid[j] = j < H ? hs[lane][j] : 0.f;

  const int l = l0 + lane;
  const float t = (float)l;
  float* of = out + (int64_t)f * D * L;
  for (int c0 = 0; c0 < D; c0 += kFiltChunk) {
    const int cn = D - c0 < kFiltChunk ? D - c0 : kFiltChunk;
    __syncthreads();   // the previous chunk's reads are done
    for (int i = threadIdx.x; i < H * kFiltChunk; i += kFiltThreads) {
      const int j = i / kFiltChunk, dd = i - j * kFiltChunk;
      w2s[dd][j] = dd < cn ? __ldg(W2 + (int64_t)j * D + c0 + dd) : 0.f;
    }
    for (int i = threadIdx.x; i < kFiltChunk * (kFiltMaxH + 4 - H); i += kFiltThreads) {
      const int dd = i / (kFiltMaxH + 4 - H), j = H + i - dd * (kFiltMaxH + 4 - H);
      w2s[dd][j] = 0.f;   // tail of each row read by the 16-byte loads
    }
    __syncthreads();
    for (int dd = warp; dd < cn; dd += kFiltThreads / 32) {
      const float4* wr = reinterpret_cast<const float4*>(&w2s[dd][0]);
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q < kFiltMaxH / 4; ++q) {
        if (4 * q >= H) break;
        const float4 w = wr[q];
        acc = fmaf(hid[4 * q], w.x, acc);
        acc = fmaf(hid[4 * q + 1], w.y, acc);
        acc = fmaf(hid[4 * q + 2], w.z, acc);
        acc = fmaf(hid[4 * q + 3], w.w, acc);
      }
      const int d = c0 + dd;
      const float rate = __ldg(decay + (int64_t)f * D + d);
      const float y = (acc + __ldg(B2 + d)) * expf(-fabsf(rate) * t);
      if (l < L) of[(int64_t)d * L + l] = y;
    }
  }
}

}  // namespace

// out (n, D, L) dense: filter i = (sin(omega * (pe @ w1[i] + b1[i])) @ w2[i] + b2[i])^T
// times the window exp(-|decay[i, d]| * t).  pe (L, F) dense; w1[i] (F, H),
// b1[i] (H), w2[i] (H, D), b2[i] (D) dense device arrays given as host arrays
// of n device pointers; decay (n, D).  n <= 8, F <= 32, H <= 64 with H % 4 == 0
// (else WXX_E_UNSUPPORTED, nothing enqueued).
WXX_EXPORT int wxx_hyena_filters(float* out, const float* pe, int L, int F, int H, int D, int n,
                                 const float* const* w1, const float* const* b1,
                                 const float* const* w2, const float* const* b2, float omega,
                                 const float* decay) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(L >= 0 && F >= 1 && H >= 1 && D >= 0 && n >= 0,
              "wxx_hyena_filters: bad sizes (L %d, F %d, H %d, D %d, n %d)", L, F, H, D, n);
  WXX_REQUIRE(w1 && b1 && w2 && b2 && decay && pe, "wxx_hyena_filters: NULL argument");
  if (n > kFiltMaxN || F > kFiltMaxF || H > kFiltMaxH || H % 4 != 0) {
    wxx::set_error("wxx_hyena_filters: n %d, F %d, H %d outside n <= %d, F <= %d, H <= %d "
                   "(a multiple of 4)", n, F, H, kFiltMaxN, kFiltMaxF, kFiltMaxH);
    return WXX_E_UNSUPPORTED;
  }
  if ((int64_t)L * D * n == 0) return WXX_OK;
  FilterWeights fw;
  memset(&fw, 0, sizeof(fw));
  for (int i = 0; i < n; ++i) {
    WXX_REQUIRE(w1[i] && b1[i] && w2[i] && b2[i], "wxx_hyena_filters: filter %d weights NULL", i);
    fw.w1[i] = w1[i];
    fw.b1[i] = b1[i];
    fw.w2[i] = w2[i];
    fw.b2[i] = b2[i];
  }
  dim3 grid((unsigned)((L + 31) / 32), (unsigned)n);
  hyena_filter_kernel<<<grid, kFiltThreads, 0, wxx::stream()>>>(out, pe, L, F, H, D, fw, omega,
                                                                decay);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
