// Allocation-free causal FFT convolution.
//
// wxx_fftconv_static computes exactly what wxx_fftconv computes (Hyena's
// fft_conv1d, nn/hyena.py:208-216 of the reference), but keeps the filter
// spectrum H = rfft(h, n) in a fixed device array compiled into this library
// instead of asking the allocator for it.  It never calls cudaMalloc,
// cudaFree, the library's stream-ordered pool or any other allocating
// routine.
//
// Who needs it: a caller that cannot allocate device memory at the moment it
// convolves.  Two such callers: a host process whose own caching allocator
// has already reserved the free HBM (the library's pool would fail or force
// that allocator to release memory in the middle of a step), and a
// latency-critical step that must not take the allocator's lock or wait
// while the pool grows.  The price is a fixed footprint (kStaticSpecBytes per
// device, held from module load) and the size limits below.
//
// Limits (checked on the host before anything is enqueued; a call beyond them
// returns WXX_E_ARG with a message and launches nothing):
//   * D * (n/2 + 2) <= kStaticSpecComplex = 256 * 16386 complex values
//     (32 MiB + 4 KiB of scratch): 256 filter rows at n = 32768, the largest
//     filter of the configured workloads;
//   * n <= 32768, the largest size whose rows are transformed in shared
//     memory (larger sizes need ping-pong buffers that would be allocated);
//   * 0 <= out_len <= n.
//
// The spectrum rows are stored n/2 + 2 complex values apart (a multiple of 16
// bytes), the same layout wxx_fftconv allocates, so the persistent staged
// kernel that bulk-copies each filter row into shared memory runs here too.
//
// Scratch contents: nothing has to start at zero.  Every call first writes the
// whole D x (n/2+2) prefix of the array (rfft of the zero-padded filter) and
// only then reads it, on the same stream.
//
// Concurrency: there is ONE scratch array per device.  Two calls that can
// overlap on the device (different streams, or host threads with their own
// streams) race on it and may read each other's spectrum.  Calls issued on the
// one library stream run in order and are safe.
//
// Setup: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and caches it; that lookup
// can load this library's device code onto the device.  Make that first call
// before any stream capture begins.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"

extern "C" int wxx_rfft(void* X, int64_t out_ld, const float* x, int64_t in_ld, int64_t rows,
                        int64_t in_len, int64_t n);
extern "C" int wxx_fftconv_spectrum(float* y, const float* x, int64_t x_off, int64_t sb,
                                    int64_t sd, int64_t sl, const void* H, int64_t h_ld, int B,
                                    int D, int L, int64_t n, int out_len);

namespace {

constexpr int64_t kStaticMaxN = 32768;                      // shared-memory FFT rows only
constexpr int64_t kStaticSpecComplex = 256 * (kStaticMaxN / 2 + 2);  // 4 194 816 values
constexpr int64_t kStaticSpecBytes = kStaticSpecComplex * 8;
constexpr int kMaxDevices = 64;
static_assert(kStaticSpecBytes == (int64_t(32) << 20) + 4096,
              "scratch size is documented as 32 MiB + 4 KiB");

static __device__ __align__(256) float2 g_static_spectrum[kStaticSpecComplex];

std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_static_spectrum on the current device (looked up once
// per device and cached).
int static_spectrum(void** out) {
  int dev = -1;
  WXX_CUDA_CHECK(cudaGetDevice(&dev));
  WXX_REQUIRE(dev >= 0 && dev < kMaxDevices, "wxx_fftconv_static: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_spectrum);
    if (e != cudaSuccess || p == nullptr) {
      wxx::set_error("wxx_fftconv_static: cudaGetSymbolAddress failed on device %d: %s", dev,
                     cudaGetErrorString(e));
      return WXX_E_CUDA;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return WXX_OK;
}

int pow2_log(int64_t n) {
  if (n < 1 || (n & (n - 1))) return -1;
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return l;
}

}  // namespace

// Same arguments and result as wxx_fftconv; no allocation (limits above).
WXX_EXPORT int wxx_fftconv_static(float* y, const float* x, int64_t x_off, int64_t sb,
                                  int64_t sd, int64_t sl, const float* h, int64_t h_ld, int Lh,
                                  int B, int D, int L, int64_t n, int out_len) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(pow2_log(n) >= 0, "wxx_fftconv_static: n=%lld is not a positive power of two",
              (long long)n);
  WXX_REQUIRE(n <= kStaticMaxN,
              "wxx_fftconv_static: n=%lld exceeds the allocation-free limit %lld",
              (long long)n, (long long)kStaticMaxN);
  WXX_REQUIRE(D >= 0 && B >= 0 && L >= 0 && Lh >= 0, "wxx_fftconv_static: negative size");
  WXX_REQUIRE(out_len >= 0 && out_len <= n, "wxx_fftconv_static: out_len=%d must be in [0, n]",
              out_len);
  const int64_t ld = n / 2 + 2;  // 16-byte multiple: the staged kernel's bulk copies apply
  WXX_REQUIRE((int64_t)D * ld <= kStaticSpecComplex,
              "wxx_fftconv_static: D*(n/2+2)=%lld complex values exceed the static scratch "
              "of %lld",
              (long long)((int64_t)D * ld), (long long)kStaticSpecComplex);
  void* Hs = nullptr;
  int st = static_spectrum(&Hs);
  if (st) return st;
  st = wxx_rfft(Hs, ld, h, h_ld, D, Lh, n);
  if (st) return st;
  return wxx_fftconv_spectrum(y, x, x_off, sb, sd, sl, Hs, ld, B, D, L, n, out_len);
}
