// Shared definitions for the wxx B200 kernel library (libwxx_cuda.so).
//
// Every exported entry point is `extern "C"`, takes plain pointers and sizes,
// enqueues its work on the library's per-process stream and returns an int
// status (0 = ok, negative = error).  The message of the last error is kept
// per host thread and returned by wxx_last_error().
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

#define WXX_OK 0
#define WXX_E_ARG (-1)
#define WXX_E_CUDA (-2)
#define WXX_E_TIMEOUT (-3)
#define WXX_E_UNSUPPORTED (-4)
#define WXX_E_STATE (-5)

// Codes written into the device-side error word (first writer wins).
#define WXX_DEV_ERR_MBAR_TIMEOUT 1
#define WXX_DEV_ERR_BAD_INDEX 2

#define WXX_EXPORT extern "C" __attribute__((visibility("default")))

namespace wxx {

void set_error(const char* fmt, ...);
void count_launch();                // one kernel launch enqueued by this library
// After every launch: counts it and checks the launch error.  In check mode
// (WXX_CHECK=1 at wxx_init, or wxx_set_check_mode(1)) it also waits for the
// kernel and reads the device error word, so a failing kernel is reported by
// the call that launched it (file:line) instead of by a later one.
int after_launch(const char* file, int line);
int require_init();                 // WXX_OK once wxx_init() succeeded
cudaStream_t stream();              // library stream of the current device
int num_sms();                      // SM count of the current device
int* device_error_word();           // device pointer to the error word
int fft_init_tables();              // FFT twiddle tables (fft.cu), run by wxx_init

// Grid size for a grid-stride elementwise kernel: enough CTAs to fill the
// GPU (a multiple of the SM count) but never more than the work needs.
inline unsigned grid_for(int64_t work_items, int threads_per_cta, int ctas_per_sm = 8) {
  int64_t need = (work_items + threads_per_cta - 1) / threads_per_cta;
  int64_t cap = (int64_t)num_sms() * ctas_per_sm;
  if (need < 1) need = 1;
  return (unsigned)(need < cap ? need : cap);
}

}  // namespace wxx

#define WXX_CUDA_CHECK(expr)                                                      \
  do {                                                                            \
    cudaError_t _wxx_e = (expr);                                                  \
    if (_wxx_e != cudaSuccess) {                                                  \
      wxx::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_wxx_e), \
                     __FILE__, __LINE__);                                         \
      return WXX_E_CUDA;                                                          \
    }                                                                             \
  } while (0)

#define WXX_LAUNCH_CHECK()                                          \
  do {                                                              \
    int _wxx_s = wxx::after_launch(__FILE__, __LINE__);             \
    if (_wxx_s != WXX_OK) return _wxx_s;                            \
  } while (0)

#define WXX_REQUIRE(cond, ...)        \
  do {                                \
    if (!(cond)) {                    \
      wxx::set_error(__VA_ARGS__);    \
      return WXX_E_ARG;               \
    }                                 \
  } while (0)

#define WXX_REQUIRE_INIT()                   \
  do {                                       \
    int _wxx_s = wxx::require_init();        \
    if (_wxx_s != WXX_OK) return _wxx_s;     \
  } while (0)

// 2^x on the SFU (ex2.approx: relative error ~2^-22; 2^-inf = +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100's two-wide FP32 instructions): each half is the
// correctly rounded scalar result, so (d0, d1) are the same bits as two
// fmaf / + / * calls, in half the issue slots.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1,
                                     float c0, float c1) {
  asm("{\n.reg .b64 ra, rb, rc, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ void sub2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "sub.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
// max(a, b, c) in one instruction (sm_100 three-input max; a NaN input
// loses, as with fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// GELU, tanh form of shaders/activations/gelu.wgsl:20-27 (x > 10 -> x,
// x < -10 -> 0), u = 0.7978845608 (x + 0.044715 x^3).  Evaluated through the
// identity 0.5 x (1 + tanh u) = x / (1 + e^(-2u)): one SFU exp2 and one fast
// divide (denominator in [1, 2^126]), relative error a few ulp.  Shared by the
// unary kernel and the GEMM epilogue so fused and unfused paths give the same
// bits.
// Branch-free (selects), so the 32 values of an epilogue chunk interleave.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  const float e = fast_exp2(u * -2.8853900817779268f);   // e^(-2u) = 2^(-2u log2 e)
  float r = __fdividef(x, 1.0f + e);                      // e = inf -> -0, selected away
  r = (x > 10.0f) ? x : r;
  return (x < -10.0f) ? 0.0f : r;
}

// silu(x) = x * sigmoid(x) = x / (1 + e^(-x)), the exponent with the
// reference's +-88 sigmoid input clamp (sigmoid.wgsl:18-19), evaluated as
// 2^(-x log2 e) on the ex2 unit and a fast divide (a few ulp; no branch, no
// slow division path).  Shared by the unary kernel and the GEMM's GLU
// epilogue, so the fused and unfused forms agree.
__device__ __forceinline__ float silu_lib(float x) {
  const float xc = fminf(fmaxf(x, -88.0f), 88.0f);
  return __fdividef(x, 1.0f + fast_exp2(xc * -1.4426950408889634f));
}

// x rounded to the nearest TF32 value (10 explicit mantissa bits, ties away
// from zero), returned as an fp32 whose low 13 mantissa bits are zero.  A
// tcgen05 kind::tf32 product reads an fp32 operand by dropping those bits
// (truncation toward zero, a bias of half a TF32 ulp on average); a value
// stored already rounded is read exactly, so an activation that only ever
// feeds TF32 products loses half as much and without the bias.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Records the first device-side error code; later errors are dropped so the
// host sees the root cause.
__device__ __forceinline__ void wxx_device_fail(int* err_word, int code) {
  if (err_word) atomicCAS(err_word, 0, code);
}

// Strided view descriptor (element units) shared by the elementwise kernels.
#define WXX_MAX_RANK 8
struct WxxStrided {
  int rank;
  int64_t shape[WXX_MAX_RANK];
  int64_t stride_a[WXX_MAX_RANK];
  int64_t stride_b[WXX_MAX_RANK];
  int64_t offset_a;
  int64_t offset_b;
};
