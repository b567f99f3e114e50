// 2-D pooling over NCHW (ResNet18 stem max-pool and head adaptive average pool).
//
// Reference semantics:
//   maxpool2d.wgsl (functional/convolution.py:60-125): padding cells are
//     excluded, the first strictly greater value wins (scan order kh, kw),
//     initial value -1e38 and index 0xFFFFFFFF; the index is the flat input
//     position.  Output size (H + 2p - k) / s + 1.
//   adaptive_avgpool2d.wgsl (functional/convolution.py:490-543): window
//     [floor(o*in/out), ceil((o+1)*in/out)) per axis, mean over the window.
#include "common.cuh"

namespace {

__global__ void maxpool2d_kernel(float* __restrict__ y, uint32_t* __restrict__ idx,
                                 const float* __restrict__ x, int B, int C, int H, int W, int Ho,
                                 int Wo, int KH, int KW, int sh, int sw, int ph, int pw) {
  int64_t total = (int64_t)B * C * Ho * Wo;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int ow = (int)(i % Wo);
    int64_t t = i / Wo;
    int oh = (int)(t % Ho);
    int64_t bc = t / Ho;
    int64_t base = bc * H * W;
    int h0 = oh * sh - ph, w0 = ow * sw - pw;
    float best = -1e38f;
    uint32_t arg = 0xFFFFFFFFu;
    for (int kh = 0; kh < KH; ++kh) {
      int ih = h0 + kh;
      if (ih < 0 || ih >= H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        int iw = w0 + kw;
        if (iw < 0 || iw >= W) continue;
        int64_t p = base + (int64_t)ih * W + iw;
        float v = x[p];
        if (v > best) {
          best = v;
          arg = (uint32_t)p;
        }
      }
    }
    y[i] = best;
    if (idx) idx[i] = arg;
  }
}

__global__ void adaptive_avgpool2d_kernel(float* __restrict__ y, const float* __restrict__ x,
                                          int B, int C, int H, int W, int Ho, int Wo) {
  int64_t total = (int64_t)B * C * Ho * Wo;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int ow = (int)(i % Wo);
    int64_t t = i / Wo;
    int oh = (int)(t % Ho);
    int64_t bc = t / Ho;
    int hs = (oh * H) / Ho, he = ((oh + 1) * H + Ho - 1) / Ho;
    int ws = (ow * W) / Wo, we = ((ow + 1) * W + Wo - 1) / Wo;
    const float* p = x + bc * H * W;
    float acc = 0.f;
    for (int h = hs; h < he; ++h)
      for (int w = ws; w < we; ++w) acc += p[(int64_t)h * W + w];
    y[i] = acc / (float)((he - hs) * (we - ws));
  }
}

// Global average pool (output 1x1): one warp per (b, c) plane.
__global__ void global_avgpool_kernel(float* __restrict__ y, const float* __restrict__ x,
                                      int64_t planes, int hw) {
  int64_t plane = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  int l = threadIdx.x & 31;
  if (plane >= planes) return;
  const float* p = x + plane * hw;
  float acc = 0.f;
  for (int i = l; i < hw; i += 32) acc += p[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (l == 0) y[plane] = acc / (float)hw;
}

}  // namespace

WXX_EXPORT int wxx_maxpool2d(float* Y, uint32_t* idx, const float* X, int B, int C, int H, int W,
                             int KH, int KW, int sh, int sw, int ph, int pw) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(KH > 0 && KW > 0 && sh > 0 && sw > 0 && ph >= 0 && pw >= 0,
              "wxx_maxpool2d: bad window");
  int Ho = (H + 2 * ph - KH) / sh + 1;
  int Wo = (W + 2 * pw - KW) / sw + 1;
  WXX_REQUIRE(Ho > 0 && Wo > 0, "wxx_maxpool2d: empty output");
  int64_t total = (int64_t)B * C * Ho * Wo;
  if (total == 0) return WXX_OK;
  maxpool2d_kernel<<<wxx::grid_for(total, 256), 256, 0, wxx::stream()>>>(Y, idx, X, B, C, H, W, Ho,
                                                                        Wo, KH, KW, sh, sw, ph, pw);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

WXX_EXPORT int wxx_adaptive_avgpool2d(float* Y, const float* X, int B, int C, int H, int W, int Ho,
                                      int Wo) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(Ho > 0 && Wo > 0 && H > 0 && W > 0, "wxx_adaptive_avgpool2d: bad sizes");
  int64_t total = (int64_t)B * C * Ho * Wo;
  if (total == 0) return WXX_OK;
  if (Ho == 1 && Wo == 1) {
    int64_t planes = (int64_t)B * C;
    global_avgpool_kernel<<<(unsigned)((planes + 7) / 8), 256, 0, wxx::stream()>>>(Y, X, planes,
                                                                                  H * W);
  } else {
    adaptive_avgpool2d_kernel<<<wxx::grid_for(total, 256), 256, 0, wxx::stream()>>>(Y, X, B, C, H,
                                                                                   W, Ho, Wo);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
