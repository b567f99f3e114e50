// ResNet's stem for small images in one kernel (nn/resnet.py:31-79 forward:
// conv1 -> bn1 -> relu -> maxpool, then the layout change to channels-last
// that the channels-last stages read):
//   conv 7x7 / stride 2 / pad 3 (Cin <= 4 input channels -> 64), the
//   convolution's bias, eval batchnorm and ReLU (conv_post, the convolution
//   epilogue's expression), max pool 3x3 / stride 2 / pad 1, and the store as
//   (B, Hp, Wp, 64).
// One CTA per image.  The padded image and all weights sit in shared memory;
// a thread makes 8 channels x 8 output pixels (every shared-memory value it
// loads feeds 8 FMAs), summing the taps in (channel, kh, kw) order like the
// direct convolution kernel, so the values are the same bits as the separate
// conv / maxpool / transpose launches.  The conv outputs then replace the
// image in shared memory (pixel-major, 65 floats a pixel: the pooling reads
// 32 consecutive channels without bank conflicts) and the pooled values are
// written channel-fastest (coalesced).
#include "tc_gemm.cuh"

#include <cstring>

using namespace wxx_tc;

namespace {

constexpr int kStemCout = 64;
constexpr int kStemThreads = 256;
constexpr int kStemCg = kStemCout / 8;                 // channel groups of 8
constexpr int kStemPixPerPass = (kStemThreads / kStemCg) * 8;   // 256 output pixels
constexpr int kStemLd = kStemCout + 1;                  // conv-output pixel stride

__global__ void __launch_bounds__(kStemThreads, 2)
    stem_kernel(float* __restrict__ Y, const float* __restrict__ X, const float* __restrict__ Wt,
                const float* __restrict__ bias, ConvPost post, int Cin, int H, int W, int Ho,
                int Wo, int Hp, int Wp, int packed) {
  extern __shared__ __align__(16) float sm[];
  const int Hpad = H + 6, Wpad = W + 6;
  const int taps = Cin * 49;
  const int img_floats = ((Cin * Hpad * Wpad) + 3) & ~3;
  float* img = sm;
  float* wts = sm + img_floats;           // taps x 64, channel fastest
  float* co = sm;                         // after the conv: Ho*Wo pixels x kStemLd
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const float* xb = X + (int64_t)b * Cin * H * W;
  for (int i = t; i < Cin * Hpad * Wpad; i += kStemThreads) {
    const int c = i / (Hpad * Wpad);
    const int r = i - c * Hpad * Wpad;
    const int y = r / Wpad - 3, x = r % Wpad - 3;
    img[i] = (y >= 0 && y < H && x >= 0 && x < W) ? xb[((int64_t)c * H + y) * W + x] : 0.f;
  }
  if (packed) {
    // already (taps, 64): a float4 copy
    const float4* src = reinterpret_cast<const float4*>(Wt);
    float4* dst = reinterpret_cast<float4*>(wts);
    for (int i = t; i < taps * kStemCout / 4; i += kStemThreads) dst[i] = __ldg(src + i);
  } else {
    for (int i = t; i < taps * kStemCout; i += kStemThreads) {
      const int tap = i / kStemCout, n = i - tap * kStemCout;
      wts[i] = Wt[(int64_t)n * taps + tap];
    }
  }
  __syncthreads();

  const int cg = t % kStemCg, pg = t / kStemCg;
  const int npix = Ho * Wo;
  const int pix0 = pg * 8;
  int off[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int pix = min(pix0 + i, npix - 1);
    const int ho = pix / Wo, wo = pix - (pix / Wo) * Wo;
    off[i] = 2 * ho * Wpad + 2 * wo;
  }
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const float4* w4 = reinterpret_cast<const float4*>(wts) + cg * 2;
  for (int c = 0; c < Cin; ++c) {
    const float* ic = img + c * Hpad * Wpad;
    for (int kh = 0; kh < 7; ++kh) {
#pragma unroll
      for (int kw = 0; kw < 7; ++kw) {
        const float* row = ic + kh * Wpad + kw;
        const float4 wa = w4[0], wb = w4[1];
        w4 += kStemCout / 4;
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xv = row[off[i]];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(xv, wv[j], acc[i][j]);
        }
      }
    }
  }
  __syncthreads();   // every thread is done with the image and the weights
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int pix = pix0 + i;
    if (pix < npix) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int n = cg * 8 + j;
        float o = acc[i][j];
        if (bias != nullptr) o += bias[n];
        co[pix * kStemLd + n] = conv_post(post, o, n, 0);
      }
    }
  }
  __syncthreads();
  float* yb = Y + (int64_t)b * Hp * Wp * kStemCout;
  for (int o = t; o < Hp * Wp * kStemCout; o += kStemThreads) {
    const int c = o % kStemCout, q = o / kStemCout;
    const int py = q / Wp, px = q - (q / Wp) * Wp;
    float best = -1e38f;   // the max-pool kernel's start value and strict compare
    for (int dy = 0; dy < 3; ++dy) {
      const int iy = 2 * py - 1 + dy;
      if (iy < 0 || iy >= Ho) continue;
      for (int dx = 0; dx < 3; ++dx) {
        const int ix = 2 * px - 1 + dx;
        if (ix < 0 || ix >= Wo) continue;
        const float v = co[(iy * Wo + ix) * kStemLd + c];
        if (v > best) best = v;
      }
    }
    yb[o] = best;
  }
}

}  // namespace

// ResNet stem (see the top of this file).  X (B, Cin, H, W) with Cin <= 4 and
// H, W <= 32; Wt (64, Cin, 7, 7), or with packed = 1 the same weights
// transposed to (Cin * 49, 64) and 16-byte aligned; bias (64) or NULL; batchnorm running mean /
// variance, gamma, beta (64 each) with eps, or rm == NULL for none; relu 0/1.
// Y (B, Hp, Wp, 64) channels-last with Ho = (H + 6 - 7) / 2 + 1 (Wo alike) and
// Hp = (Ho + 2 - 3) / 2 + 1 (Wp alike).
WXX_EXPORT int wxx_resnet_stem(float* Y, const float* X, const float* Wt, const float* bias,
                               const float* rm, const float* rv, const float* gamma,
                               const float* beta, float eps, int relu, int B, int Cin, int H,
                               int W, int packed) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B >= 0 && Cin >= 1 && Cin <= 4 && H >= 1 && W >= 1 && H <= 32 && W <= 32,
              "wxx_resnet_stem: needs 1..4 input channels and H, W in 1..32");
  WXX_REQUIRE(rm == nullptr || (rv != nullptr && gamma != nullptr && beta != nullptr),
              "wxx_resnet_stem: incomplete batchnorm parameters");
  WXX_REQUIRE(!packed || !(reinterpret_cast<uintptr_t>(Wt) & 15),
              "wxx_resnet_stem: packed weights must be 16-byte aligned");
  if (B == 0) return WXX_OK;
  const int Ho = (H + 6 - 7) / 2 + 1, Wo = (W + 6 - 7) / 2 + 1;
  const int Hp = (Ho + 2 - 3) / 2 + 1, Wp = (Wo + 2 - 3) / 2 + 1;
  WXX_REQUIRE(Ho * Wo <= kStemPixPerPass, "wxx_resnet_stem: too many output pixels");
  const int img_floats = ((Cin * (H + 6) * (W + 6)) + 3) & ~3;
  const size_t conv_bytes = (size_t)(img_floats + Cin * 49 * kStemCout) * sizeof(float);
  const size_t pool_bytes = (size_t)Ho * Wo * kStemLd * sizeof(float);
  const size_t smem = conv_bytes > pool_bytes ? conv_bytes : pool_bytes;
  static size_t smem_set = 0;
  if (smem > 48 * 1024 && smem > smem_set) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(stem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    smem_set = smem;
  }
  ConvPost post;
  memset(&post, 0, sizeof(post));
  post.rm = rm;
  post.rv = rv;
  post.g = gamma;
  post.b = beta;
  post.eps = eps;
  post.relu = relu ? 1 : 0;
  stem_kernel<<<(unsigned)B, kStemThreads, smem, wxx::stream()>>>(Y, X, Wt, bias, post, Cin, H, W,
                                                                  Ho, Wo, Hp, Wp, packed ? 1 : 0);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
