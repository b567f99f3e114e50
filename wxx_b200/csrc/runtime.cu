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
#include <cstdlib>

#include "common.cuh"

#include <nvtx3/nvToolsExt.h>

#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <mutex>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

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

// Device memory a captured graph works in.  While a capture is open every
// wxx_malloc is served from the arena by a host-side best-fit allocator
// (stream order makes reuse of freed blocks safe), so the recorded kernels
// see addresses that stay valid for every replay.  Blocks freed after the
// capture stay reserved until the graph is destroyed.
struct Arena {
  char* base = nullptr;
  size_t size = 0;
  std::map<size_t, size_t> free_blocks;          // offset -> bytes
  std::unordered_map<void*, size_t> live;        // pointer -> bytes
  size_t used = 0, peak = 0;
  bool capturing = false;
  cudaGraphExec_t exec = nullptr;
  int64_t kernels = 0;                           // kernel launches recorded
  int64_t launches_at_begin = 0;
  // Pool blocks released while this capture was open: a cudaFreeAsync then
  // would be recorded into the graph (and is invalid for memory the graph did
  // not allocate), and kernels recorded before the release may still read the
  // block on every replay -- so they are freed when the graph is destroyed.
  std::vector<void*> deferred;
  // Destroyed while tensors allocated inside it were still alive: the arena
  // keeps its memory (in g_arenas, so their frees are recognised) until the
  // last of them is freed.  Releasing it earlier would let the pool hand the
  // range to new blocks, and a late free of an arena pointer could then
  // release a live block that happens to start at the same address.
  bool dead = false;
};
std::vector<Arena*> g_arenas;                    // arenas with memory (guarded by g.mu)
Arena* g_capture = nullptr;                      // arena of the open capture

bool arena_alloc(Arena* a, size_t sz, void** out) {
  auto best = a->free_blocks.end();
  for (auto it = a->free_blocks.begin(); it != a->free_blocks.end(); ++it)
    if (it->second >= sz && (best == a->free_blocks.end() || it->second < best->second)) best = it;
  if (best == a->free_blocks.end()) return false;
  size_t off = best->first, len = best->second;
  a->free_blocks.erase(best);
  if (len > sz) a->free_blocks[off + sz] = len - sz;
  void* p = a->base + off;
  a->live[p] = sz;
  a->used += sz;
  if (a->used > a->peak) a->peak = a->used;
  *out = p;
  return true;
}

void arena_release(Arena* a, void* p, size_t sz) {
  size_t off = (size_t)((char*)p - a->base);
  a->used -= sz;
  auto next = a->free_blocks.lower_bound(off);
  if (next != a->free_blocks.end() && next->first == off + sz) {
    sz += next->second;
    next = a->free_blocks.erase(next);
  }
  if (next != a->free_blocks.begin()) {
    auto prev = std::prev(next);
    if (prev->first + prev->second == off) {
      prev->second += sz;
      return;
    }
  }
  a->free_blocks[off] = sz;
}

Arena* arena_of(void* p) {
  for (Arena* a : g_arenas)
    if ((char*)p >= a->base && (char*)p < a->base + a->size) return a;
  return nullptr;
}

thread_local char g_err[1024] = {0};
std::atomic<int64_t> g_launches{0};
bool g_check_mode = false;

}  // namespace

namespace wxx {

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int after_launch(const char* file, int line) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(e), file, line);
    return WXX_E_CUDA;
  }
  if (!g_check_mode) return WXX_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream(), &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
    return WXX_OK;   // a recorded launch runs later, at replay
  e = cudaStreamSynchronize(stream());
  if (e != cudaSuccess) {
    set_error("kernel launched at %s:%d failed: %s", file, line, cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  int v = 0;
  e = cudaMemcpy(&v, g.err_word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    set_error("reading the device error word failed: %s", cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  if (v != 0) {
    cudaMemset(g.err_word, 0, sizeof(int));
    set_error("kernel launched at %s:%d reported device error %d (%s)", file, line, v,
              v == WXX_DEV_ERR_MBAR_TIMEOUT ? "a bounded wait expired"
              : v == WXX_DEV_ERR_BAD_INDEX  ? "an index outside its table"
                                            : "unknown");
    return v == WXX_DEV_ERR_MBAR_TIMEOUT ? WXX_E_TIMEOUT : WXX_E_ARG;
  }
  return WXX_OK;
}

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
  const char* chk = getenv("WXX_CHECK");
  g_check_mode = chk != nullptr && chk[0] == '1';
  // Constant tables of the kernels, filled once here (never inside a capture).
  int st = wxx::fft_init_tables();
  if (st != WXX_OK) return st;
  WXX_CUDA_CHECK(cudaStreamSynchronize(g.stream));
  return WXX_OK;
}

// Check mode on (1) or off (0); see wxx::after_launch.  Also set by the
// environment variable WXX_CHECK=1 at wxx_init.
WXX_EXPORT int wxx_set_check_mode(int on) {
  g_check_mode = on != 0;
  return WXX_OK;
}

WXX_EXPORT int wxx_get_check_mode(int* on) {
  *on = g_check_mode ? 1 : 0;
  return WXX_OK;
}

// NVTX ranges around functional calls (WXX_NVTX=1 on the Python side):
// visible in Nsight timelines, free when no tool is attached.
WXX_EXPORT int wxx_nvtx_push(const char* name) {
  nvtxRangePushA(name ? name : "wxx");
  return WXX_OK;
}

WXX_EXPORT int wxx_nvtx_pop(void) {
  nvtxRangePop();
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
  {
    std::lock_guard<std::mutex> lk(g.mu);
    if (g_capture != nullptr) {
      if (!arena_alloc(g_capture, sz, &p)) {
        wxx::set_error("wxx_malloc(%llu bytes): graph arena of %llu bytes exhausted "
                       "(%llu in use)", (unsigned long long)nbytes,
                       (unsigned long long)g_capture->size, (unsigned long long)g_capture->used);
        return WXX_E_STATE;
      }
      *out = p;
      return WXX_OK;
    }
  }
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
    if (Arena* a = arena_of(p)) {
      auto ia = a->live.find(p);
      if (ia == a->live.end()) {
        wxx::set_error("wxx_free: %p freed twice inside a graph arena", p);
        return WXX_E_ARG;
      }
      // Inside the capture the block is reused by later allocations; after
      // it, replays still write there, so it stays reserved (only no longer
      // counted as held by a tensor).
      if (a == g_capture) arena_release(a, p, ia->second);
      a->live.erase(ia);
      if (a->dead && a->live.empty()) {
        for (size_t i = 0; i < g_arenas.size(); ++i)
          if (g_arenas[i] == a) {
            g_arenas.erase(g_arenas.begin() + i);
            break;
          }
        cudaFreeAsync(a->base, wxx::stream());
        delete a;
      }
      return WXX_OK;
    }
    auto it = g.live.find(p);
    if (it == g.live.end()) {
      wxx::set_error("wxx_free: %p was not allocated by wxx_malloc (or freed twice)", p);
      return WXX_E_ARG;
    }
    sz = it->second;
    g.live.erase(it);
    g.active_bytes -= (int64_t)sz;
    g.n_free++;
    if (g_capture != nullptr) {
      g_capture->deferred.push_back(p);
      return WXX_OK;
    }
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

// Restarts peak tracking at the current active bytes.
WXX_EXPORT int wxx_mem_reset_peak(void) {
  WXX_REQUIRE_INIT();
  std::lock_guard<std::mutex> lk(g.mu);
  g.peak_bytes = g.active_bytes;
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

// Inside a graph capture the record becomes an external event node, so every
// replay stamps the event (timing of kernels inside a replayed graph).
WXX_EXPORT int wxx_event_record(void* ev) {
  WXX_REQUIRE_INIT();
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  WXX_CUDA_CHECK(cudaStreamIsCapturing(wxx::stream(), &cs));
  if (cs == cudaStreamCaptureStatusActive) {
    WXX_CUDA_CHECK(cudaEventRecordWithFlags((cudaEvent_t)ev, wxx::stream(),
                                            cudaEventRecordExternal));
  } else {
    WXX_CUDA_CHECK(cudaEventRecord((cudaEvent_t)ev, wxx::stream()));
  }
  return WXX_OK;
}

WXX_EXPORT int wxx_event_elapsed_ms(void* start, void* stop, float* ms) {
  WXX_REQUIRE_INIT();
  WXX_CUDA_CHECK(cudaEventSynchronize((cudaEvent_t)stop));
  WXX_CUDA_CHECK(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)stop));
  return WXX_OK;
}

// ---------------------------------------------------------------- CUDA graphs
//
// wxx_graph_begin opens a capture of the library stream with a fresh arena of
// arena_bytes; every library call until wxx_graph_end is recorded instead of
// run.  wxx_graph_launch replays the recorded kernels on the library stream
// with the same pointers (inputs are read from where they were at capture;
// outputs land in the arena).  Host synchronisation (wxx_sync, blocking
// copies, device_status) is invalid inside a capture and ends it with an error.

WXX_EXPORT int wxx_graph_begin(uint64_t arena_bytes, void** handle) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(handle != nullptr, "wxx_graph_begin: handle is NULL");
  {
    std::lock_guard<std::mutex> lk(g.mu);
    WXX_REQUIRE(g_capture == nullptr, "wxx_graph_begin: a capture is already open");
  }
  size_t sz = arena_bytes < 256 ? 256 : ((arena_bytes + 255) & ~size_t(255));
  Arena* a = new Arena();
  // From the stream-ordered pool like every other block (a plain cudaMalloc /
  // cudaFree pair synchronises the device, and was seen taking ~0.6 s now and
  // then between generation calls); it is ordered before the capture begins.
  cudaError_t e = cudaMallocFromPoolAsync((void**)&a->base, sz, g.pool, wxx::stream());
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaStreamSynchronize(wxx::stream());
    cudaMemPoolTrimTo(g.pool, 0);
    e = cudaMallocFromPoolAsync((void**)&a->base, sz, g.pool, wxx::stream());
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    delete a;
    wxx::set_error("wxx_graph_begin: arena of %llu bytes: %s", (unsigned long long)sz,
                   cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  a->size = sz;
  a->free_blocks[0] = sz;
  e = cudaStreamBeginCapture(wxx::stream(), cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaFreeAsync(a->base, wxx::stream());
    delete a;
    wxx::set_error("wxx_graph_begin: cudaStreamBeginCapture: %s", cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  a->capturing = true;
  a->launches_at_begin = g_launches.load();
  {
    std::lock_guard<std::mutex> lk(g.mu);
    g_arenas.push_back(a);
    g_capture = a;
  }
  *handle = a;
  return WXX_OK;
}

// Closes the capture opened by wxx_graph_begin and instantiates it.  On
// failure the handle is still valid and must be passed to wxx_graph_destroy.
WXX_EXPORT int wxx_graph_end(void* handle) {
  WXX_REQUIRE_INIT();
  Arena* a = (Arena*)handle;
  {
    std::lock_guard<std::mutex> lk(g.mu);
    WXX_REQUIRE(a != nullptr && a == g_capture, "wxx_graph_end: not the open capture");
    g_capture = nullptr;
  }
  a->capturing = false;
  const int64_t recorded = g_launches.load() - a->launches_at_begin;
  g_launches.fetch_sub(recorded);   // recorded, not run
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(wxx::stream(), &graph);
  if (e != cudaSuccess || graph == nullptr) {
    cudaGetLastError();
    wxx::set_error("wxx_graph_end: capture failed: %s (a call inside the capture "
                   "synchronised with the host or failed)", cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  e = cudaGraphInstantiate(&a->exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    cudaGetLastError();
    a->exec = nullptr;
    wxx::set_error("wxx_graph_end: cudaGraphInstantiate: %s", cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  a->kernels = recorded;
  return WXX_OK;
}

WXX_EXPORT int wxx_graph_launch(void* handle) {
  WXX_REQUIRE_INIT();
  Arena* a = (Arena*)handle;
  WXX_REQUIRE(a != nullptr && a->exec != nullptr, "wxx_graph_launch: no instantiated graph");
  WXX_CUDA_CHECK(cudaGraphLaunch(a->exec, wxx::stream()));
  g_launches.fetch_add(a->kernels);
  return WXX_OK;
}

// out[0] arena bytes, out[1] peak bytes used during capture, out[2] kernels recorded.
WXX_EXPORT int wxx_graph_stats(void* handle, int64_t* out) {
  Arena* a = (Arena*)handle;
  WXX_REQUIRE(a != nullptr && out != nullptr, "wxx_graph_stats: NULL argument");
  out[0] = (int64_t)a->size;
  out[1] = (int64_t)a->peak;
  out[2] = a->kernels;
  return WXX_OK;
}

// Ends an open capture if needed, waits for replays in flight, frees the arena.
WXX_EXPORT int wxx_graph_destroy(void* handle) {
  WXX_REQUIRE_INIT();
  Arena* a = (Arena*)handle;
  if (a == nullptr) return WXX_OK;
  bool open;
  {
    std::lock_guard<std::mutex> lk(g.mu);
    open = (a == g_capture);
    if (open) g_capture = nullptr;
  }
  if (open) {
    cudaGraph_t graph = nullptr;
    cudaStreamEndCapture(wxx::stream(), &graph);
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    g_launches.fetch_sub(g_launches.load() - a->launches_at_begin);
  }
  cudaError_t e = cudaStreamSynchronize(wxx::stream());
  if (a->exec) cudaGraphExecDestroy(a->exec);
  a->exec = nullptr;
  for (void* p : a->deferred) cudaFreeAsync(p, wxx::stream());
  a->deferred.clear();
  {
    std::lock_guard<std::mutex> lk(g.mu);
    if (!a->live.empty()) {
      a->dead = true;   // freed with the last of its tensors (wxx_free)
      a = nullptr;
    } else {
      for (size_t i = 0; i < g_arenas.size(); ++i)
        if (g_arenas[i] == a) {
          g_arenas.erase(g_arenas.begin() + i);
          break;
        }
    }
  }
  if (a != nullptr) {
    cudaFreeAsync(a->base, wxx::stream());
    delete a;
  }
  if (e != cudaSuccess) {
    wxx::set_error("wxx_graph_destroy: %s", cudaGetErrorString(e));
    return WXX_E_CUDA;
  }
  return WXX_OK;
}
