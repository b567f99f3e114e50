// Runtime: device selection, the per-process stream, a stream-ordered caching
// allocator, host<->device copies, events and the device error word.
//
// Replaces the wgpu plumbing of the reference (src/wxx/backend/device.py):
//   WebGPUContext (device.py:9-28)      -> wxx_init / the library stream
//   GPUBufferPool (device.py:31-141)    -> wxx_malloc / wxx_free / wxx_mem_stats
//   GPUCommandBuffer (device.py:144-255)-> every launch is stream-ordered on one
//                                          cudaStream_t; wxx_sync is the fence.
// The allocator is CUDA's stream-ordered pool (cudaMallocAsync) with an
// unbounded release threshold, so freed blocks stay cached in the pool and are
// reused by later allocations on the same stream without a device sync.  The
// reference caps its cache at 4 MiB (device.py:33,108); here large activation
// buffers are cached too.
#include "common.cuh"

#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

namespace {

struct State {
  bool ready = false;
  int device = -1;
  int sms = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = true;
  cudaStream_t user_stream = nullptr;   // set by wxx_set_stream (capture/interop)
  cudaMemPool_t pool = nullptr;
  int* err_word = nullptr;              // device int, 0 = no error
  std::mutex mu;
  std::unordered_map<void*, size_t> live;
  int64_t active_bytes = 0;
  int64_t peak_bytes = 0;
  int64_t n_alloc = 0;
  int64_t n_free = 0;
};

State g;
thread_local char g_err[1024] = {0};
std::atomic<int64_t> g_launches{0};

}  // namespace

namespace wxx {

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int require_init() {
  if (!g.ready) {
    set_error("wxx_init(device) has not been called");
    return WXX_E_STATE;
  }
  return WXX_OK;
}

cudaStream_t stream() { return g.user_stream ? g.user_stream : g.stream; }
int num_sms() { return g.sms > 0 ? g.sms : 148; }
int* device_error_word() { return g.err_word; }

}  // namespace wxx

WXX_EXPORT const char* wxx_last_error(void) { return g_err; }

WXX_EXPORT const char* wxx_version(void) { return "wxx_b200 0.1 (sm_100a)"; }

// Number of kernels this library has launched since the process started.
WXX_EXPORT int wxx_launch_count(int64_t* out) {
  *out = g_launches.load(std::memory_order_relaxed);
  return WXX_OK;
}

WXX_EXPORT int wxx_device_count(int* count) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  *count = n;
  return WXX_OK;
}

WXX_EXPORT int wxx_init(int device) {
  if (g.ready) {
    if (device == g.device) return WXX_OK;
    wxx::set_error("wxx_init: already initialised on device %d (asked for %d); "
                   "the library drives one GPU per process", g.device, device);
    return WXX_E_STATE;
  }
  WXX_CUDA_CHECK(cudaSetDevice(device));
  cudaDeviceProp prop;
  WXX_CUDA_CHECK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) {
    wxx::set_error("wxx_init: device %d is sm_%d%d; this library is built for sm_100a (B200)",
                   device, prop.major, prop.minor);
    return WXX_E_UNSUPPORTED;
  }
  g.sms = prop.multiProcessorCount;
  WXX_CUDA_CHECK(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking));
  WXX_CUDA_CHECK(cudaDeviceGetDefaultMemPool(&g.pool, device));
  uint64_t threshold = UINT64_MAX;
  WXX_CUDA_CHECK(cudaMemPoolSetAttribute(g.pool, cudaMemPoolAttrReleaseThreshold, &threshold));
  WXX_CUDA_CHECK(cudaMalloc(&g.err_word, 256));
  WXX_CUDA_CHECK(cudaMemset(g.err_word, 0, 256));
  g.device = device;
  g.ready = true;
  return WXX_OK;
}

WXX_EXPORT int wxx_current_device(int* device) {
  WXX_REQUIRE_INIT();
  *device = g.device;
  return WXX_OK;
}

WXX_EXPORT int wxx_num_sms(int* sms) {
  WXX_REQUIRE_INIT();
  *sms = g.sms;
  return WXX_OK;
}

// ---------------------------------------------------------------- allocator

WXX_EXPORT int wxx_malloc(void** out, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(out != nullptr, "wxx_malloc: out is NULL");
  // Round to 256 B: every buffer starts 256-B aligned (TMA needs 16 B) and
  // the pool sees few distinct sizes.
  size_t sz = nbytes < 256 ? 256 : ((nbytes + 255) & ~size_t(255));
  void* p = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&p, sz, g.pool, wxx::stream());
  if (e != cudaSuccess) {
    cudaGetLastError();
    // Out of memory with blocks cached in the pool: give them back and retry.
    cudaStreamSynchronize(wxx::stream());
    cudaMemPoolTrimTo(g.pool, 0);
    e = cudaMallocFromPoolAsync(&p, sz, g.pool, wxx::stream());
    if (e != cudaSuccess) {
      wxx::set_error("wxx_malloc(%llu bytes) failed: %s", (unsigned long long)nbytes,
                     cudaGetErrorString(e));
      cudaGetLastError();
      return WXX_E_CUDA;
    }
  }
  {
    std::lock_guard<std::mutex> lk(g.mu);
    g.live[p] = sz;
    g.active_bytes += (int64_t)sz;
    if (g.active_bytes > g.peak_bytes) g.peak_bytes = g.active_bytes;
    g.n_alloc++;
  }
  *out = p;
  return WXX_OK;
}

WXX_EXPORT int wxx_free(void* p) {
  if (p == nullptr) return WXX_OK;
  WXX_REQUIRE_INIT();
  size_t sz = 0;
  {
    std::lock_guard<std::mutex> lk(g.mu);
    auto it = g.live.find(p);
    if (it == g.live.end()) {
      wxx::set_error("wxx_free: %p was not allocated by wxx_malloc (or freed twice)", p);
      return WXX_E_ARG;
    }
    sz = it->second;
    g.live.erase(it);
    g.active_bytes -= (int64_t)sz;
    g.n_free++;
  }
  WXX_CUDA_CHECK(cudaFreeAsync(p, wxx::stream()));
  return WXX_OK;
}

// out[0] active bytes, out[1] live blocks, out[2] bytes reserved by the pool,
// out[3] peak active bytes, out[4] total allocations, out[5] total frees.
WXX_EXPORT int wxx_mem_stats(int64_t* out) {
  WXX_REQUIRE_INIT();
  uint64_t reserved = 0;
  WXX_CUDA_CHECK(cudaMemPoolGetAttribute(g.pool, cudaMemPoolAttrReservedMemCurrent, &reserved));
  std::lock_guard<std::mutex> lk(g.mu);
  out[0] = g.active_bytes;
  out[1] = (int64_t)g.live.size();
  out[2] = (int64_t)reserved;
  out[3] = g.peak_bytes;
  out[4] = g.n_alloc;
  out[5] = g.n_free;
  return WXX_OK;
}

WXX_EXPORT int wxx_mem_trim(void) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaStreamSynchronize(wxx::stream()));
  WXX_CUDA_CHECK(cudaMemPoolTrimTo(g.pool, 0));
  return WXX_OK;
}

WXX_EXPORT int wxx_host_alloc(void** out, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaHostAlloc(out, nbytes ? nbytes : 1, cudaHostAllocDefault));
  return WXX_OK;
}

WXX_EXPORT int wxx_host_free(void* p) {
  if (!p) return WXX_OK;
  WXX_CUDA_CHECK(cudaFreeHost(p));
  return WXX_OK;
}

// ---------------------------------------------------------------- copies

WXX_EXPORT int wxx_memcpy_h2d(void* dst, const void* src, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  if (nbytes == 0) return WXX_OK;
  WXX_CUDA_CHECK(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, wxx::stream()));
  return WXX_OK;
}

// Device -> host; returns after the data has arrived (the stream is drained).
WXX_EXPORT int wxx_memcpy_d2h(void* dst, const void* src, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  if (nbytes) {
    WXX_CUDA_CHECK(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, wxx::stream()));
  }
  WXX_CUDA_CHECK(cudaStreamSynchronize(wxx::stream()));
  return WXX_OK;
}

// Device -> host without waiting (the caller synchronises before reading dst).
WXX_EXPORT int wxx_memcpy_d2h_async(void* dst, const void* src, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  if (nbytes == 0) return WXX_OK;
  WXX_CUDA_CHECK(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, wxx::stream()));
  return WXX_OK;
}

WXX_EXPORT int wxx_memcpy_d2d(void* dst, const void* src, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  if (nbytes == 0) return WXX_OK;
  WXX_CUDA_CHECK(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToDevice, wxx::stream()));
  return WXX_OK;
}

WXX_EXPORT int wxx_memset(void* dst, int value, uint64_t nbytes) {
  WXX_REQUIRE_INIT();
  if (nbytes == 0) return WXX_OK;
  WXX_CUDA_CHECK(cudaMemsetAsync(dst, value, nbytes, wxx::stream()));
  return WXX_OK;
}

WXX_EXPORT int wxx_sync(void) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaStreamSynchronize(wxx::stream()));
  return WXX_OK;
}

WXX_EXPORT void* wxx_get_stream(void) { return (void*)wxx::stream(); }

// Redirects all launches to `s` (NULL restores the library stream).  Used to
// capture a sequence of calls into a CUDA graph or to share a stream with an
// external runtime.
WXX_EXPORT int wxx_set_stream(void* s) {
  WXX_REQUIRE_INIT();
  g.user_stream = (cudaStream_t)s;
  return WXX_OK;
}

// ---------------------------------------------------------------- errors

// Reads the device error word (synchronising the stream first) and clears it.
// *code = 0 when no kernel reported an error.
WXX_EXPORT int wxx_device_status(int* code) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaStreamSynchronize(wxx::stream()));
  int v = 0;
  WXX_CUDA_CHECK(cudaMemcpy(&v, g.err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) WXX_CUDA_CHECK(cudaMemset(g.err_word, 0, sizeof(int)));
  *code = v;
  return WXX_OK;
}

// ---------------------------------------------------------------- events

WXX_EXPORT int wxx_event_create(void** ev) {
  WXX_REQUIRE_INIT();
  cudaEvent_t e;
  WXX_CUDA_CHECK(cudaEventCreate(&e));
  *ev = (void*)e;
  return WXX_OK;
}

WXX_EXPORT int wxx_event_destroy(void* ev) {
  if (!ev) return WXX_OK;
  WXX_CUDA_CHECK(cudaEventDestroy((cudaEvent_t)ev));
  return WXX_OK;
}

WXX_EXPORT int wxx_event_record(void* ev) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaEventRecord((cudaEvent_t)ev, wxx::stream()));
  return WXX_OK;
}

WXX_EXPORT int wxx_event_elapsed_ms(void* start, void* stop, float* ms) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaEventSynchronize((cudaEvent_t)stop));
  WXX_CUDA_CHECK(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)stop));
  return WXX_OK;
}
