// tcgen05 / TMEM GEMM engine for sm_100a (TF32 tensor cores, fp32 accumulate).
//
// One persistent, warp-specialised kernel template computes
//   D[tile] = sum_k A[m, k] * B[n, k]
// for 128 x BN output tiles (BN = 64, 128 or 256) with a BK = 32 (128-byte)
// K-block pipeline:
//   warp 0        TMA producer: cp.async.bulk.tensor loads into 128B-swizzled
//                 shared memory (no multicast), expect-tx on the stage barrier
//   warp 1        TMEM allocator + single-thread tcgen05.mma issuer
//                 (kind::tf32, M = 128, N = BN, K = 8 per instruction),
//                 tcgen05.commit frees smem stages and publishes accumulators
//   warps 2..5    epilogue: tcgen05.ld 32x32b from TMEM -> registers ->
//                 bias / scale -> global memory
//   warps 6..9    gather producers for operands that TMA cannot address
//                 (rows not 16-byte aligned, im2col of a convolution):
//                 ld.global -> st.shared in the same swizzled layout, then
//                 fence.proxy.async and an mbarrier arrive
// Two TMEM accumulator buffers (2 x BN columns) let the epilogue of tile i
// overlap the main loop of tile i+1.
//
// Every mbarrier wait is bounded (wall-clock limit read from %globaltimer):
// on expiry the waiting role records WXX_DEV_ERR_MBAR_TIMEOUT in the device
// error word, raises a CTA-wide abort flag and leaves its loop; before the
// CTA exits the producer drains its outstanding TMA transactions and the MMA
// warp drains its outstanding tensor-core work, then TMEM is released.
#pragma once

#include "common.cuh"

#include <cuda.h>

namespace wxx_tc {

constexpr int BM = 128;          // tile rows (UMMA M, one TMEM lane per row)
constexpr int BK = 32;           // fp32 elements per K-block = one 128 B swizzle row
constexpr int UMMA_K = 8;        // K per tcgen05.mma kind::tf32
constexpr int NUM_THREADS = 320; // 10 warps
constexpr int EPI_WARP0 = 2;
constexpr int GATHER_WARP0 = 6;
constexpr int GATHER_THREADS = 128;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 4;                 // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;                 // 8/16/32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;   // 4 / 6 / 8
  static constexpr int TMEM_COLS = 2 * BN;                    // 128 / 256 / 512
  // Per epilogue warp: two 4 KB staging tiles (32 x 32 fp32, 128B-swizzled
  // for the TMA store); the padded-transpose fallback reuses the first 4.2 KB.
  static constexpr int EPI_WARP_BYTES = 8192;
  static constexpr int EPI_BYTES = 4 * EPI_WARP_BYTES;        // 32 KB
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024;
};

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false when the
// wall-clock limit (limit_ns of %globaltimer) expired -- recording
// WXX_DEV_ERR_MBAR_TIMEOUT and raising the abort flag -- or another role
// raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, int* err,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 255) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > limit_ns) {
        wxx_device_fail(err, WXX_DEV_ERR_MBAR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Shared -> global tensor store of one box (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed bulk groups still read their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (TMEM) (+)= A (TMEM: row i in lane i, one 32-bit column per K element,
// K-major) * B (shared memory descriptor).
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread t of the warp gets row
// (lane base + t), columns [col, col + 32).
// tcgen05.ld of 32 columns without the wait: issue several, then tmem_ld_wait().
__device__ __forceinline__ void tmem_ld_32x32_nowait(uint32_t taddr, float (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
        "=f"(v[7]), "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]),
        "=f"(v[14]), "=f"(v[15]), "=f"(v[16]), "=f"(v[17]), "=f"(v[18]), "=f"(v[19]),
        "=f"(v[20]), "=f"(v[21]), "=f"(v[22]), "=f"(v[23]), "=f"(v[24]), "=f"(v[25]),
        "=f"(v[26]), "=f"(v[27]), "=f"(v[28]), "=f"(v[29]), "=f"(v[30]), "=f"(v[31])
      : "r"(taddr));
}

// tcgen05.wait::ld that also ties v's registers to the wait, so no read of
// them can be scheduled before the load has landed.
__device__ __forceinline__ void tmem_ld_wait(float (&v)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]), "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15]), "+f"(v[16]), "+f"(v[17]), "+f"(v[18]), "+f"(v[19]), "+f"(v[20]), "+f"(v[21]), "+f"(v[22]), "+f"(v[23]), "+f"(v[24]), "+f"(v[25]), "+f"(v[26]), "+f"(v[27]), "+f"(v[28]), "+f"(v[29]), "+f"(v[30]), "+f"(v[31])
               :
               : "memory");
}

// Orders later reads of v after the preceding (volatile) wait.
__device__ __forceinline__ void reg_pin(float (&v)[32]) {
  asm volatile(""
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]), "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15]), "+f"(v[16]), "+f"(v[17]), "+f"(v[18]), "+f"(v[19]), "+f"(v[20]), "+f"(v[21]), "+f"(v[22]), "+f"(v[23]), "+f"(v[24]), "+f"(v[25]), "+f"(v[26]), "+f"(v[27]), "+f"(v[28]), "+f"(v[29]), "+f"(v[30]), "+f"(v[31]));
}

// tcgen05.st of 32 columns (one row per lane), then wait for it to land.
__device__ __forceinline__ void tmem_st_32x32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      :
      : "r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (sm100 layout): start>>4 [0,14),
// LBO>>4 [16,30), SBO>>4 [32,46), version 1 at [46,48), layout type at [61,64):
// 2 = SWIZZLE_128B (16-byte chunks), 1 = SWIZZLE_128B_BASE32B (32-byte chunks).
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW128Base32B = 1;

__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                          uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

// K-major tile: rows of 128 B (32 fp32 k-values), 8-row 1024 B swizzle atoms
// (SBO); one MMA K-step (8 values = 32 B) advances the start address.
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t tile, int kk) {
  return sdesc(tile + kk * 32, 16, 1024, kLayoutSW128);
}

// MN-major tile (tf32 must use the 32-byte-atom 128B swizzle): each 32-wide
// MN chunk is a TMA box of 32 k-rows x 128 B (4096 B apart: LBO); swizzle
// atoms are 4 k-rows (512 B: SBO); one MMA K-step covers 8 rows (1024 B).
__device__ __forceinline__ uint64_t sdesc_mnmajor(uint32_t tile, int kk) {
  return sdesc(tile + kk * 1024, 4096, 512, kLayoutSW128Base32B);
}

// Instruction descriptor for kind::tf32: D f32 [4,6), A/B tf32 [7,10)/[10,13),
// A/B major [15]/[16] (1 = MN-major), N>>3 [17,23), M>>4 [24,29).
__host__ __device__ constexpr uint32_t idesc_tf32_mn(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_tf32(int n, bool a_mn, bool b_mn) {
  return idesc_tf32_mn(BM, n, a_mn, b_mn);
}

// Byte offset of element (row, k) of a K-major 128B-swizzled tile
// (rows of 128 B = 32 fp32 k-values, 8-row atoms of 1024 B).
__device__ __forceinline__ uint32_t kmajor_offset(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 2) ^ (row & 7)) & 7) << 4) + ((k & 3) << 2));
}

// ------------------------------------------------------------ operand sources

// How one operand tile (rows x 32 k) reaches shared memory.
//   kind 0: TMA, K-major global (k contiguous): one box {32, rows}
//   kind 1: TMA, MN-major global (rows contiguous): rows/32 boxes {32, 32}
//   kind 2: gather, generic strided matrix
//   kind 3: gather, im2col of an NCHW convolution input (A operand only)
struct OperandSrc {
  int kind;
  int bcast_batch;        // TMA: batch coordinate always 0
  // gather (kind 2): element (row, k) of batch b at base + b*bs + row*s_row + k*s_k
  const float* base;
  int64_t bs, s_row, s_k;
  int rows_total;         // valid rows (M or N)
  int k_total;            // valid K
  // im2col (kind 3); kind 4 (NHWC convolution input, TMA) uses cin, kw,
  // strides, padding, dilation, ho, wo: K-block kc is 32 channels of one
  // filter tap (k = (fh * KW + fw) * cin + c) and a 128-row tile is one 4-D
  // box (32 channels, W, H, images) of the input at the tap's offset
  int cin, h, w, kh, kw, sh, sw, ph, pw, dh, dw, ho, wo;
};

// Convolution output post-ops, applied after alpha and the conv bias:
// eval-mode batchnorm of channel n with the batchnorm kernel's expression
// (x - mean) * rsqrt(var + eps) * gamma + beta, then + residual (laid out like
// the output, at the output's own index), then ReLU -- ResNet's conv -> bn
// (-> add) -> relu chain in the conv's epilogue, with the same fp32
// operations.  NCHW outputs (kind 1) and the split-K reduce read `res` here;
// row-major (NHWC) outputs stored by TMA read the residual from EpiParams.res.
struct ConvPost {
  const float* rm;        // running mean (NULL: no batchnorm)
  const float* rv;        // running variance
  const float* g;         // gamma
  const float* b;         // beta
  float eps;
  const float* res;       // residual (B, N, Ho, Wo) or NULL
  int relu;
};

__device__ __forceinline__ float conv_post(const ConvPost& c, float v, int n, int64_t idx) {
  if (c.rm != nullptr) {
    const float inv = rsqrtf(c.rv[n] + c.eps);
    v = (v - c.rm[n]) * inv * c.g[n] + c.b[n];
  }
  if (c.res != nullptr) v = v + c.res[idx];
  if (c.relu) v = fmaxf(0.0f, v);
  return v;
}

struct EpiParams {
  int kind;               // 0 = row-major matrix C, 1 = NCHW convolution output,
                          // 2 = short causal conv along rows, written (B, N, L) (pair kernel)
  float* C;
  int64_t c_bs;           // batch stride of C (elements)
  int ldc;                // row stride of C (elements), kind 0
  const float* bias;
  int bias_mode;          // 0 none, 1 (N,), 2 (M,N), 3 (batch,M,N); conv: 1 = per channel
  int64_t bias_bs;
  float alpha;
  int hw_out;             // conv: Ho*Wo
  int tma_store;          // kind 0 with bias_mode <= 1: C written by TMA stores
  // TMA-store path only: C = act(alpha * AB + bias) + res
  int act;                // 0 none, 1 GELU (tanh form), 2 paired GLU (C has N/2 columns)
  const float* res;       // residual (M, N) per batch, or NULL
  int64_t res_ld, res_bs;
  int raw;                // split-K: raw partial sums to the workspace map, z = batch * splits + slice
  int round_tf32;         // kind 0: store C rounded to the nearest TF32 value (tf32_rna)
  // SM-pair kernel, plain epilogue: instead of storing C, each row's maximum
  // over the tile's columns (values above -1e38; among equal values the
  // column with the smaller amax_key, the argmax kernels' tie order) goes to
  // amax[(bt * M + m) * tiles_n + tn] as (value, column within the tile as
  // int bits); C is not written.
  float2* amax;
  ConvPost post;          // kind 1 only
  // kind 2: rows are (sequence b, position n) = (row / conv_len, row % conv_len);
  // C[b, c, n] (c_bs = N * conv_len) = conv_b[c'] + sum_k conv_w[c', k] * Y[row - k, c]
  // over taps k < conv_k with n >= k, c' = c % conv_ch, Y = alpha * AB + bias.
  int conv_len, conv_k, conv_ch;
  const float* conv_w;
  const float* conv_b;
};

struct GemmParams {
  int M, N, K;
  int batch;
  int tiles_m, tiles_n;
  int group_m;            // row blocks per raster band (tiles_m: plain row-fastest order)
  int num_kb;             // K-blocks per pass
  int passes;             // 1 = TF32; 3 = 3xTF32 (hi*lo, lo*hi, hi*hi)
  int splits;             // K-slices per tile (split-K; 1 = whole K)
  int kb_per_split;       // K-blocks (over all passes) per slice
  // SM-pair kernel, stream-K: the pairs share the tile-major K-block
  // iterations evenly; a pair that does not reach a tile's last K-block
  // leaves its raw partial in sk_ws (slot = its pair index) and counts it in
  // sk_flags[tile]; the pair finishing the tile adds it.
  int sk;
  float* sk_ws;
  int* sk_flags;
  OperandSrc a, b;
  EpiParams epi;
  int* err;
};

// Tile order: batch-major; inside a batch, bands of `group_m` row blocks,
// row block fastest inside a band, then column block.  Concurrent tiles then
// share a band of A (kept in L2) and a few column blocks of B.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& bt, int& tm, int& tn) {
  const int per_batch = p.tiles_m * p.tiles_n;
  bt = t / per_batch;
  int r = t - bt * per_batch;
  const int band_tiles = p.group_m * p.tiles_n;
  int band = r / band_tiles;
  int in_band = r - band * band_tiles;
  int rows_left = p.tiles_m - band * p.group_m;
  int gm = rows_left < p.group_m ? rows_left : p.group_m;
  tm = band * p.group_m + in_band % gm;
  tn = in_band / gm;
}

// Work unit u -> output tile t and its K-block range [kb0, kb1) (split-K
// slices of one tile are consecutive units).
__device__ __forceinline__ void unit_range(const GemmParams& p, int u, int& t, int& sp, int& kb0,
                                           int& kb1) {
  t = u / p.splits;
  sp = u - t * p.splits;
  const int total = p.num_kb * p.passes;
  kb0 = sp * p.kb_per_split;
  kb1 = kb0 + p.kb_per_split < total ? kb0 + p.kb_per_split : total;
}

// 3xTF32 operand parts: the tensor core reads the top 19 bits of each fp32
// word, so x = hi + lo with hi = x with the low 13 mantissa bits cleared and
// lo = x - hi (exact in fp32); lo itself is then read to tf32 precision.
__device__ __forceinline__ float split_part(float x, int part) {
  if (part == 0) return x;
  float hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  return part == 1 ? hi : x - hi;
}

// Gather `rows` x 32 fp32 values into a K-major swizzled tile (rows % 8 == 0).
// Executed by the GATHER_THREADS producer threads.  part: 0 raw, 1 hi, 2 lo.
__device__ __forceinline__ void gather_tile(const OperandSrc& s, uint8_t* dst, int rows, int row0,
                                            int k0, int batch, int gtid, int part) {
  if (s.kind == 2) {
    const float* base = s.base + (int64_t)batch * s.bs;
    if (s.s_k == 1) {
      // lanes along k (coalesced), threads over rows, 8 loads in flight
      int k = gtid & 31;
      int kg = k0 + k;
      bool kvalid = kg < s.k_total;
      for (int r0 = gtid >> 5; r0 < rows; r0 += 8 * (GATHER_THREADS / 32)) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          int r = r0 + u * (GATHER_THREADS / 32);
          int row = row0 + r;
          v[u] = (r < rows && row < s.rows_total && kvalid)
                     ? __ldg(base + (int64_t)row * s.s_row + kg)
                     : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          int r = r0 + u * (GATHER_THREADS / 32);
          if (r < rows) *reinterpret_cast<float*>(dst + kmajor_offset(r, k)) = split_part(v[u], part);
        }
      }
    } else {
      // lanes along rows (coalesced when s_row == 1), 8 loads in flight
      const int total = rows * BK;
      for (int e0 = gtid; e0 < total; e0 += 8 * GATHER_THREADS) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          int e = e0 + u * GATHER_THREADS;
          int r = e % rows, k = e / rows;
          int row = row0 + r, kg = k0 + k;
          v[u] = (e < total && row < s.rows_total && kg < s.k_total)
                     ? __ldg(base + (int64_t)row * s.s_row + (int64_t)kg * s.s_k)
                     : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          int e = e0 + u * GATHER_THREADS;
          if (e < total) {
            int r = e % rows, k = e / rows;
            *reinterpret_cast<float*>(dst + kmajor_offset(r, k)) = split_part(v[u], part);
          }
        }
      }
    }
  } else {
    // im2col: row = output pixel (b, oh, ow); k = (c, fr, fq) over the filter.
    // The filter coordinate advances incrementally along k (no divisions in
    // the loop) and all 32 loads of a row are issued before any is stored.
    const int khw = s.kh * s.kw;
    for (int r = gtid; r < rows; r += GATHER_THREADS) {
      const int m = row0 + r;
      const bool mvalid = m < s.rows_total;
      int ow = 0, oh = 0, b = 0;
      if (mvalid) {
        ow = m % s.wo;
        const int t = m / s.wo;
        oh = t % s.ho;
        b = t / s.ho;
      }
      const int ih0 = oh * s.sh - s.ph, iw0 = ow * s.sw - s.pw;
      const float* xb = s.base + (int64_t)b * s.cin * s.h * s.w;
      int c = k0 / khw;
      int rem = k0 - c * khw;
      int fr = rem / s.kw, fq = rem - fr * s.kw;
      float v[BK];
#pragma unroll
      for (int k = 0; k < BK; ++k) {
        const int ih = ih0 + fr * s.dh, iw = iw0 + fq * s.dw;
        const bool ok = mvalid && (k0 + k) < s.k_total && ih >= 0 && ih < s.h && iw >= 0 &&
                        iw < s.w;
        v[k] = ok ? __ldg(xb + ((int64_t)c * s.h + ih) * s.w + iw) : 0.f;
        if (++fq == s.kw) {
          fq = 0;
          if (++fr == s.kh) { fr = 0; ++c; }
        }
      }
#pragma unroll
      for (int k = 0; k < BK; ++k)
        *reinterpret_cast<float*>(dst + kmajor_offset(r, k)) = split_part(v[k], part);
    }
  }
}

// Row-major epilogue for one warp's 32 x 32 chunk (rows m0..m0+31, columns
// n0..n0+31).  Thread t holds row m0+t in v[]; the chunk is transposed through
// a padded shared-memory tile so that each store instruction writes four
// full 128-byte row segments (lane l: row r0 + l/8, columns 4*(l%8)..+3).
__device__ __forceinline__ void epi_store_rows(const GemmParams& p, int bt, int m0, int n0,
                                               float (&v)[32], float* stage) {
  const EpiParams& e = p.epi;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 32; ++j) stage[lane * 33 + j] = v[j];
  __syncwarp();
  const int cq = (lane & 7) * 4;
  const int n = n0 + cq;
  float* cbase = e.C + (int64_t)bt * e.c_bs;
  const bool vec_ok = ((e.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(cbase) & 15) == 0);
  float bcol[4] = {0.f, 0.f, 0.f, 0.f};
  if (e.bias_mode == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) bcol[i] = (n + i < p.N) ? e.bias[n + i] : 0.f;
  }
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    const int m = m0 + r;
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = stage[r * 33 + cq + i] * e.alpha + bcol[i];
    if (m < p.M) {
      if (e.bias_mode >= 2) {
        const float* brow = e.bias + (e.bias_mode == 3 ? (int64_t)bt * e.bias_bs : 0) +
                            (int64_t)m * p.N;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (n + i < p.N) o[i] += brow[n + i];
      }
      if (e.round_tf32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = tf32_rna(o[i]);
      }
      float* crow = cbase + (int64_t)m * e.ldc;
      if (vec_ok && n + 3 < p.N) {
        *reinterpret_cast<float4*>(crow + n) = make_float4(o[0], o[1], o[2], o[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (n + i < p.N) crow[n + i] = o[i];
      }
    }
  }
  __syncwarp();
}

// Epilogue store of one thread's row segment: row m, columns n0..n0+31.
__device__ __forceinline__ void epi_store(const GemmParams& p, int bt, int m, int n0,
                                          float (&v)[32]) {
  const EpiParams& e = p.epi;
  if (m >= p.M) return;
  if (e.kind == 0) {
    float* crow = e.C + (int64_t)bt * e.c_bs + (int64_t)m * e.ldc;
    const float* brow = nullptr;
    if (e.bias_mode == 1) brow = e.bias;
    else if (e.bias_mode == 2) brow = e.bias + (int64_t)m * p.N;
    else if (e.bias_mode == 3) brow = e.bias + (int64_t)bt * e.bias_bs + (int64_t)m * p.N;
    bool full = (n0 + 32 <= p.N) && ((e.ldc & 3) == 0) &&
                ((reinterpret_cast<uintptr_t>(crow + n0) & 15) == 0);
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 o;
        o.x = v[j] * e.alpha;
        o.y = v[j + 1] * e.alpha;
        o.z = v[j + 2] * e.alpha;
        o.w = v[j + 3] * e.alpha;
        if (brow) {
          o.x += brow[n0 + j];
          o.y += brow[n0 + j + 1];
          o.z += brow[n0 + j + 2];
          o.w += brow[n0 + j + 3];
        }
        if (e.round_tf32) {
          o.x = tf32_rna(o.x);
          o.y = tf32_rna(o.y);
          o.z = tf32_rna(o.z);
          o.w = tf32_rna(o.w);
        }
        *reinterpret_cast<float4*>(crow + n0 + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        int n = n0 + j;
        if (n < p.N) {
          float o = v[j] * e.alpha;
          if (brow) o += brow[n];
          crow[n] = e.round_tf32 ? tf32_rna(o) : o;
        }
      }
    }
  } else {
    // NCHW: row m = (b, pixel), column n = output channel.
    int b = m / e.hw_out, pix = m - b * e.hw_out;
    const int64_t base = (int64_t)b * p.N * e.hw_out + pix;
    float* out = e.C + base;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      int n = n0 + j;
      if (n < p.N) {
        float o = v[j] * e.alpha;
        if (e.bias_mode == 1) o += e.bias[n];
        o = conv_post(e.post, o, n, base + (int64_t)n * e.hw_out);
        out[(int64_t)n * e.hw_out] = o;
      }
    }
  }
}

// ------------------------------------------------------------ SM-pair (cta_group::2) helpers
//
// Two CTAs of a cluster (one per SM of a TPC) compute one 256 x BN tile: each
// holds 128 rows of A and BN/2 rows of B in its own shared memory, the pair's
// leader (cluster rank 0) issues tcgen05.mma.cta_group::2 reading both, and
// each CTA's TMEM receives its own 128 accumulator rows.  Every tcgen05
// instruction of such a kernel uses cta_group::2.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Every thread of both CTAs; the non-.aligned form tolerates a warp whose
// lanes arrive from different branches.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\t"
               "barrier.cluster.wait.acquire;" ::: "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier that may live in the peer CTA (cluster address `bar_cl`).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_cl, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cl), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void umma2_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on the mbarrier at cluster address `bar_cl` when every
// tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma2_commit(uint32_t bar_cl) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cl)
               : "memory");
}

__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cl) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cl)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait with cluster-scope acquire (barriers that peers arrive on).
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag, int* err) {
  uint32_t addr = smem_u32(bar);
  if (mbar_try_wait_cluster(addr, parity)) return true;
  unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(addr, parity)) return true;
    if ((it & 255) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        wxx_device_fail(err, WXX_DEV_ERR_MBAR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Tie order of the argmax kernels (argminmax_warp_kernel) for a position r:
// slot = r mod 256 = lane + 32 j; the lane tree (shuffle strides 16 .. 1,
// lower lane kept on ties) prefers the lane whose bit-reversed index is
// smaller, and the in-lane tree over j (strides 4, 2, 1) likewise.  Among
// equal values the smaller key wins; equal keys (the same slot) go to the
// earlier position.
__host__ __device__ __forceinline__ int amax_key(int slot) {
  const int l = slot & 31, j = (slot >> 5) & 7;
  const int lr = ((l & 1) << 4) | ((l & 2) << 2) | (l & 4) | ((l & 8) >> 2) | ((l & 16) >> 4);
  const int jr = ((j & 1) << 2) | (j & 2) | ((j & 4) >> 2);
  return (lr << 3) | jr;
}

// Epilogue math of the TMA-store path for row m, columns n0..n0+31:
// v = act(alpha * v + bias[n]) + res[m, n].
// POST: apply the convolution post-ops (batchnorm, ReLU) when EpiParams.post
// asks for them; the SM-pair kernel, which never computes a convolution,
// compiles without them.
template <bool POST = true>
__device__ __forceinline__ void epi_apply(const GemmParams& p, int bt, int m, int n0,
                                          float (&v)[32], bool may_round = true) {
  const EpiParams& e = p.epi;
  const float alpha = e.alpha;
  if (e.bias_mode == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      v[j] = v[j] * alpha + ((n0 + j < p.N) ? __ldg(e.bias + n0 + j) : 0.f);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= alpha;
  }
  if (e.act == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  }
  if (POST && e.post.rm != nullptr) {
    // eval batchnorm of column n (the batchnorm kernel's expression)
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j < p.N ? n0 + j : p.N - 1;
      const float inv = rsqrtf(__ldg(e.post.rv + n) + e.post.eps);
      v[j] = (v[j] - __ldg(e.post.rm + n)) * inv * __ldg(e.post.g + n) + __ldg(e.post.b + n);
    }
  }
  if (e.res != nullptr && m < p.M) {
    const float* r = e.res + (int64_t)bt * e.res_bs + (int64_t)m * e.res_ld + n0;
    if (n0 + 32 <= p.N && !(reinterpret_cast<uintptr_t>(r) & 15)) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = __ldg(reinterpret_cast<const float4*>(r) + q);
        v[4 * q] += w.x;
        v[4 * q + 1] += w.y;
        v[4 * q + 2] += w.z;
        v[4 * q + 3] += w.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) v[j] += __ldg(r + j);
    }
  }
  if (POST && e.post.relu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = fmaxf(0.0f, v[j]);
  }
  if (may_round && e.round_tf32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = tf32_rna(v[j]);
  }
}

// act == 2 (paired GLU): product columns 2j and 2j+1 are the gate and the up
// projection of output column j, out[j] = silu(gate) * up.  Reads product
// columns n0 .. n0+63 of this thread's row from TMEM in two halves (alpha and
// bias applied) and leaves output columns n0/2 .. n0/2 + 31 in v.
template <bool POST>
__device__ __forceinline__ void epi_glu_load(const GemmParams& p, int bt, int m, int n0,
                                             uint32_t taddr, float (&v)[32]) {
  // TF32 rounding is skipped for the gate / up products and applied to the
  // GLU output that is stored.
  float w[32];
  tmem_ld_32x32(taddr, w);
  epi_apply<POST>(p, bt, m, n0, w, false);
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = silu_lib(w[2 * j]) * w[2 * j + 1];
  tmem_ld_32x32(taddr + 32u, w);
  epi_apply<POST>(p, bt, m, n0 + 32, w, false);
#pragma unroll
  for (int j = 0; j < 16; ++j) v[16 + j] = silu_lib(w[2 * j]) * w[2 * j + 1];
  if (p.epi.round_tf32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = tf32_rna(v[j]);
  }
}

// Short causal convolution epilogue (EpiParams kind 2).
//
// conv_stage_weights: once per tile, each epilogue warp copies the taps of
// the tile's BN columns into its own 8 KB of shared memory, column c at
// ws[8 c] = (w0, w1, w2, conv bias, w3, projection bias, 0, 0): the loads of
// all columns are in flight together, and the chunk loop below reads them as
// warp-uniform (broadcast) 16-byte shared loads -- one per column for up to
// three taps without a projection bias -- instead of waiting on a global
// load per column.
__device__ __forceinline__ void conv_stage_weights(const GemmParams& p, int c0, int cnt, int lane,
                                                   float* ws) {
  const EpiParams& e = p.epi;
  const int K = e.conv_k;
#pragma unroll 4
  for (int cl = lane; cl < cnt; cl += 32) {
    const int c = c0 + cl;
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f), t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < p.N) {
      const int cw = c % e.conv_ch;
      const float* wr = e.conv_w + (int64_t)cw * K;
      w.x = __ldg(wr);
      if (K > 1) w.y = __ldg(wr + 1);
      if (K > 2) w.z = __ldg(wr + 2);
      w.w = __ldg(e.conv_b + cw);
      if (K > 3) t.x = __ldg(wr + 3);
      if (e.bias_mode == 1) t.y = __ldg(e.bias + c);
    }
    reinterpret_cast<float4*>(ws)[2 * cl] = w;
    reinterpret_cast<float4*>(ws)[2 * cl + 1] = t;
  }
  __syncwarp();
}

// One 32-column chunk: lane i holds row `row` (= the warp's first row + i),
// v[j] its column n0 + j (local column cl0 + j of the tile).  Taps reach back
// up to three rows, which sit in lanes i-1 .. i-3 of the same warp (the tile
// rows overlap so that the first KT - 1 lanes of every warp are such halo
// rows; they are not stored).  Lanes hold consecutive positions, so each
// column's store is one coalesced run along n of the (B, N, L) output.  The
// tap order and the multiply-adds are those of the standalone causal conv.
// KT (the tap count) is a template parameter so that a group of 8 columns is
// one branch-free block the compiler interleaves; the group's tap loads come
// before its first global store (a load cannot move across a store it may
// alias), so one shared-memory latency covers 8 columns.
template <int KT>
__device__ __forceinline__ void epi_conv_tr(const GemmParams& p, int row, bool own, int n0,
                                            int cl0, const float* ws, const float (&v)[32]) {
  const EpiParams& e = p.epi;
  const int L = e.conv_len;
  own = own && row >= 0 && row < p.M;
  const int rr = row < 0 ? 0 : row;
  const int b = rr / L, n = rr - b * L;
  float* out = e.C + (int64_t)b * e.c_bs + n;
  const float4* wq = reinterpret_cast<const float4*>(ws) + 2 * cl0;
  const bool has_bias = e.bias_mode == 1;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float4 w[8], t[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) w[q] = wq[2 * (8 * g + q)];
    if (KT > 3 || has_bias) {
#pragma unroll
      for (int q = 0; q < 8; ++q) t[q] = wq[2 * (8 * g + q) + 1];
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) t[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float x[8], acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      x[q] = has_bias ? v[8 * g + q] * e.alpha + t[q].y : v[8 * g + q] * e.alpha;
      acc[q] = w[q].w;
      acc[q] = acc[q] + w[q].x * x[q];
    }
    if constexpr (KT > 1) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float x1 = __shfl_up_sync(0xffffffffu, x[q], 1);
        if (n >= 1) acc[q] = acc[q] + w[q].y * x1;
      }
    }
    if constexpr (KT > 2) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float x2 = __shfl_up_sync(0xffffffffu, x[q], 2);
        if (n >= 2) acc[q] = acc[q] + w[q].z * x2;
      }
    }
    if constexpr (KT > 3) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float x3 = __shfl_up_sync(0xffffffffu, x[q], 3);
        if (n >= 3) acc[q] = acc[q] + t[q].x * x3;
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int c = n0 + 8 * g + q;
      if (own && c < p.N) out[(int64_t)c * L] = acc[q];
    }
  }
}

// Columns [c0, c0 + cnt) of the tile (TMEM columns from row_addr on) for a
// warp whose first row is mc.
template <int KT>
__device__ __forceinline__ void epi_conv_tile(const GemmParams& p, int c0, int cnt, int mc,
                                              int lane, uint32_t row_addr, float* ws) {
  constexpr int hal = KT - 1;
#pragma unroll 1
  for (int c = 0; c < cnt; c += 32) {
    const int n0 = c0 + c;
    if (n0 >= p.N) break;
    float v[32];
    tmem_ld_32x32(row_addr + (uint32_t)c, v);
    epi_conv_tr<KT>(p, mc + lane, lane >= hal, n0, c, ws, v);
  }
}

// ------------------------------------------------------------ the kernel

template <int BN, bool GLU = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_a0,
                   const __grid_constant__ CUtensorMap tm_a1,
                   const __grid_constant__ CUtensorMap tm_b0,
                   const __grid_constant__ CUtensorMap tm_b1,
                   const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool a_gather = p.a.kind == 2 || p.a.kind == 3;
  const bool b_gather = p.b.kind == 2 || p.b.kind == 3;
  const bool any_gather = a_gather || b_gather;
  // Work units: output tiles, each cut into p.splits K-slices (split-K).
  const int total_units = p.batch * p.tiles_m * p.tiles_n * p.splits;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1 + (any_gather ? GATHER_THREADS : 0));
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], 4 * 32);
    }
    mbar_init(&drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    if (p.a.kind < 2) { prefetch_tmap(&tm_a0); if (p.passes > 1) prefetch_tmap(&tm_a1); }
    if (p.b.kind < 2) { prefetch_tmap(&tm_b0); if (p.passes > 1) prefetch_tmap(&tm_b1); }
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    // ---------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t tx_bytes = (a_gather ? 0 : C::A_BYTES) + (b_gather ? 0 : C::B_BYTES);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int t, sp, kb0, kb1, bt, tm, tn;
        unit_range(p, u, t, sp, kb0, kb1);
        tile_coords(p, t, bt, tm, tn);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, &abort_flag, p.err)) { ok = false; break; }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          int pass = kb / p.num_kb;
          int kc = (kb - pass * p.num_kb) * BK;
          // pass order for 3xTF32: (hi, lo), (lo, hi), (hi, hi)
          const CUtensorMap* ma = (p.passes > 1 && pass == 1) ? &tm_a1 : &tm_a0;
          const CUtensorMap* mb = (p.passes > 1 && pass == 0) ? &tm_b1 : &tm_b0;
          mbar_arrive_expect_tx(&full_bar[stage], tx_bytes);
          if (!a_gather) {
            int zb = p.a.bcast_batch ? 0 : bt;
            if (p.a.kind == 0) {
              tma_load_3d(smem_u32(sa), ma, &full_bar[stage], kc, tm * BM, zb);
            } else if (p.a.kind == 4) {
              const int tap = kc / p.a.cin, c0 = kc - tap * p.a.cin;
              const int fh = tap / p.a.kw, fw = tap - fh * p.a.kw;
              const int hw = p.a.ho * p.a.wo, m0 = tm * BM;
              const int b0 = m0 / hw, r = m0 - b0 * hw;
              const int ho0 = r / p.a.wo, wo0 = r - ho0 * p.a.wo;
              tma_load_4d(smem_u32(sa), ma, &full_bar[stage], c0,
                          wo0 * p.a.sw - p.a.pw + fw * p.a.dw, ho0 * p.a.sh - p.a.ph + fh * p.a.dh,
                          b0);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j)
                tma_load_3d(smem_u32(sa + j * 4096), ma, &full_bar[stage], tm * BM + j * 32, kc, zb);
            }
          }
          if (!b_gather) {
            int zb = p.b.bcast_batch ? 0 : bt;
            if (p.b.kind == 0) {
              tma_load_3d(smem_u32(sb), mb, &full_bar[stage], kc, tn * BN, zb);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tma_load_3d(smem_u32(sb + j * 4096), mb, &full_bar[stage], tn * BN + j * 32, kc, zb);
            }
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: every stage we issued must have completed before the CTA exits.
      volatile int dummy_abort = 0;
      for (int s = 0; s < C::STAGES; ++s)
        if (issued_mask & (1u << s))
          mbar_wait(&full_bar[s], (issued_parity >> s) & 1, &dummy_abort, p.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0) {
      const bool a_mn = (p.a.kind == 1);
      const bool b_mn = (p.b.kind == 1);
      const uint32_t idesc = idesc_tf32(BN, a_mn, b_mn);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++local) {
        int t, sp, kb0, kb1;
        unit_range(p, u, t, sp, kb0, kb1);
        int acc = local & 1;
        uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, &abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, &abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            uint64_t ad = a_mn ? sdesc_mnmajor(sa, kk) : sdesc_kmajor(sa, kk);
            uint64_t bd = b_mn ? sdesc_mnmajor(sb, kk) : sdesc_kmajor(sb, kk);
            umma_tf32(d_tmem, ad, bd, idesc, ((kb - kb0) | kk) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
      }
      // Drain all tensor-core work issued by this thread before TMEM is freed.
      umma_commit(&drain_bar);
      volatile int dummy_abort = 0;
      mbar_wait(&drain_bar, 0, &dummy_abort, p.err);
    }
  } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
    // ---------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    uint8_t* wstage = smem + C::STAGES * C::STAGE_BYTES + (warp - EPI_WARP0) * C::EPI_WARP_BYTES;
    const bool use_tma = p.epi.kind == 0 && p.epi.tma_store;
    int local = 0;
    int chunk_seq = 0;  // TMA-store staging buffer parity
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++local) {
      int t, sp, kb0, kb1, bt, tm, tn;
      unit_range(p, u, t, sp, kb0, kb1);
      tile_coords(p, t, bt, tm, tn);
      int acc = local & 1;
      uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, &abort_flag, p.err)) break;
      tc_fence_after();
      const int m0 = tm * BM + quarter * 32;
      uint32_t row_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      constexpr bool glu = GLU;   // host: GLU <=> p.epi.act == 2
#pragma unroll 1
      for (int c = 0; c < BN; c += glu ? 64 : 32) {
        float v[32];
        int n0 = tn * BN + c;
        int nc = n0;  // output column of v[0]
        if constexpr (glu) {
          if (n0 >= p.N) continue;
          epi_glu_load<true>(p, bt, m0 + lane, n0, row_addr + (uint32_t)c, v);
          nc = n0 / 2;
        } else {
          tmem_ld_32x32(row_addr + (uint32_t)c, v);
          if (n0 >= p.N) continue;
        }
        if (use_tma) {
          // alpha, bias, activation and residual in registers, row ->
          // swizzled staging tile, one TMA store per 32 x 32 chunk (clipped
          // at the edges).
          // (split-K: raw partial sums, slice index as the z coordinate)
          if (!p.epi.raw && !glu) epi_apply(p, bt, m0 + lane, n0, v);
          uint8_t* buf = wstage + (chunk_seq & 1) * 4096;
          if (lane == 0) bulk_wait_read<1>();  // the store that used `buf` has read it
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 w = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            *reinterpret_cast<float4*>(buf + lane * 128 + ((q ^ (lane & 7)) << 4)) = w;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tm_c, smem_u32(buf), nc, m0, p.epi.raw ? bt * p.splits + sp : bt);
            bulk_commit();
          }
          ++chunk_seq;
        } else if (p.epi.kind == 0) {
          epi_store_rows(p, bt, m0, n0, v, reinterpret_cast<float*>(wstage));
        } else {
          epi_store(p, bt, m0 + lane, n0, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
    if (use_tma && lane == 0) bulk_wait<0>();  // all stores complete before exit
  } else if (warp >= GATHER_WARP0 && any_gather) {
    // ---------------------------------------------------- gather producers
    const int gtid = threadIdx.x - GATHER_WARP0 * 32;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      int t, sp, kb0, kb1, bt, tm, tn;
      unit_range(p, u, t, sp, kb0, kb1);
      tile_coords(p, t, bt, tm, tn);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1, &abort_flag, p.err)) { ok = false; break; }
        uint8_t* sa = smem + stage * C::STAGE_BYTES;
        uint8_t* sb = sa + C::A_BYTES;
        int pass = kb / p.num_kb;
        int kc = (kb - pass * p.num_kb) * BK;
        // 3xTF32 pass order: (A hi, B lo), (A lo, B hi), (A hi, B hi)
        int pa = p.passes > 1 ? (pass == 1 ? 2 : 1) : 0;
        int pb = p.passes > 1 ? (pass == 0 ? 2 : 1) : 0;
        if (a_gather) gather_tile(p.a, sa, BM, tm * BM, kc, p.a.bcast_batch ? 0 : bt, gtid, pa);
        if (b_gather) gather_tile(p.b, sb, BN, tn * BN, kc, p.b.bcast_batch ? 0 : bt, gtid, pb);
        fence_proxy_async_smem();
        mbar_arrive(&full_bar[stage]);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------ SM-pair kernel
//
// 256 x BN output tiles on an SM pair (cluster of 2).  Per K-block each CTA
// loads 128 rows of A and BN/2 rows of B (32 KB at BN = 256), half the B
// traffic per SM of a 128 x 256 single-SM tile for the same tensor work.
// Operands must be TMA-fed (kind 0 or 1) and C written by TMA stores.
// Roles per CTA: warp 0 TMA producer, warp 1 TMEM allocator (+ MMA issuer in
// the leader), warps 2..5 epilogue of this CTA's 128 rows.
constexpr int PAIR_THREADS = 192;
// The short-conv epilogue (EpiParams kind 2) runs 8 epilogue warps: two per
// TMEM lane quarter, each on half of the tile's columns, so every SM
// sub-partition has a second warp to issue while one waits.
constexpr int PAIR_THREADS_CONV = 320;

// First K-block iteration of pair q when W iterations are shared by P pairs.
__device__ __forceinline__ int64_t sk_start(int q, int64_t W, int P) {
  return (int64_t)q * W / P;
}

// Number of work units of `pair`: strided whole tiles, or (stream-K) the
// tiles its iteration range touches.
__device__ __forceinline__ int pair_units(const GemmParams& p, int pair, int np, int tiles,
                                          int kb) {
  if (!p.sk) return pair < tiles ? (tiles - 1 - pair) / np + 1 : 0;
  const int64_t W = (int64_t)tiles * kb;
  const int64_t a = sk_start(pair, W, np), b = sk_start(pair + 1, W, np);
  if (a >= b) return 0;
  return (int)((b - 1) / kb - a / kb + 1);
}

// Unit i of `pair`: tile t and its K-block range [k0, k1).  Stream-K order:
// first the head of the pair's last tile (a contributor: never waits), then
// the tail of its first tile (the finisher: waits for the previous pair's
// first unit, and its epilogue overlaps the main loops that follow), then the
// whole tiles in between.
__device__ __forceinline__ void pair_unit(const GemmParams& p, int pair, int np, int tiles, int kb,
                                          int i, int& t, int& k0, int& k1) {
  if (!p.sk) {
    t = pair + i * np;
    k0 = 0;
    k1 = kb;
    return;
  }
  const int64_t W = (int64_t)tiles * kb;
  const int64_t a = sk_start(pair, W, np), b = sk_start(pair + 1, W, np);
  const int t_first = (int)(a / kb), t_last = (int)((b - 1) / kb);
  const int head = (int)(b - (int64_t)t_last * kb);    // K-blocks of the last tile
  const int tail0 = (int)(a - (int64_t)t_first * kb);  // first K-block in the first tile
  const bool has_con = head < kb;
  const bool has_fin = tail0 > 0;
  if (has_con) {
    if (i == 0) { t = t_last; k0 = 0; k1 = head; return; }
    --i;
  }
  if (has_fin) {
    if (i == 0) { t = t_first; k0 = tail0; k1 = kb; return; }
    --i;
  }
  t = t_first + (has_fin ? 1 : 0) + i;
  k0 = 0;
  k1 = kb;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add(int* ptr, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

template <int BN>
struct PairCfg {
  static constexpr int A_BYTES = BM * BK * 4;                 // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 4;           // 16 KB at BN = 256
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;   // 6
  static constexpr int TMEM_COLS = 2 * BN;                    // double-buffered accumulator
  static constexpr int EPI_WARP_BYTES = 8192;
  static constexpr int EPI_BYTES = 4 * EPI_WARP_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static_assert(TMEM_COLS <= 512, "TMEM");
  static_assert(BN * 32 <= EPI_WARP_BYTES, "short-conv taps of a tile fit a warp's staging");
};

// Epilogue forms of the SM-pair kernel (template parameter EPI).
constexpr int kPairEpiPlain = 0;   // TMA-store epilogue (bias, GELU, residual, stream-K)
constexpr int kPairEpiGlu = 1;     // paired GLU (act == 2)
constexpr int kPairEpiConv = 2;    // short causal conv written (B, N, L) (kind 2), 8 warps
constexpr int kPairEpiArgmax = 3;  // row maxima per tile into EpiParams.amax, C not written

template <int BN, int EPI = kPairEpiPlain>
__global__ void __cluster_dims__(2, 1, 1)
    __launch_bounds__(EPI == kPairEpiConv ? PAIR_THREADS_CONV : PAIR_THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a0,
                        const __grid_constant__ CUtensorMap tm_a1,
                        const __grid_constant__ CUtensorMap tm_b0,
                        const __grid_constant__ CUtensorMap tm_b1,
                        const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
  using C = PairCfg<BN>;
  constexpr bool GLU = EPI == kPairEpiGlu;
  constexpr int PM = 2 * BM;  // rows per pair tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];   // leader: both CTAs' loads landed
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];  // each CTA: its stage consumed
  __shared__ __align__(8) uint64_t tfull_bar[2];          // each CTA: accumulator ready
  __shared__ __align__(8) uint64_t tempty_bar[2];         // leader: both epilogues drained it
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int total_tiles = p.batch * p.tiles_m * p.tiles_n;
  const int total_kb = p.num_kb * p.passes;
  const int n_units = pair_units(p, pair, num_pairs, total_tiles, total_kb);
  const int n_epi = (int)(blockDim.x >> 5) - 2;   // 4, or 8 for the short-conv epilogue

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], 2 * n_epi);   // one arrive per epilogue warp of both CTAs
    }
    mbar_init(&drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a0);
    prefetch_tmap(&tm_b0);
    if (p.passes > 1) { prefetch_tmap(&tm_a1); prefetch_tmap(&tm_b1); }
  }
  if (warp == 1) tmem_alloc2(&tmem_base_sh, C::TMEM_COLS);
  tc_fence_before();
  // Both CTAs' barriers are initialised (and TMEM allocated) before any
  // load, commit or arrive targets the peer.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    // ---------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t tx_bytes = 2 * C::STAGE_BYTES;   // both CTAs' loads, counted by the leader
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = 0; u < n_units && ok; ++u) {
        int t, k0, k1, bt, tm, tn;
        pair_unit(p, pair, num_pairs, total_tiles, total_kb, u, t, k0, k1);
        tile_coords(p, t, bt, tm, tn);
        const int row_a = tm * PM + (int)rank * BM;
        const int row_b = tn * BN + (int)rank * (BN / 2);
        for (int kb = k0; kb < k1; ++kb) {
          if (!mbar_wait_cl(&empty_bar[stage], phase ^ 1, &abort_flag, p.err)) { ok = false; break; }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const int pass = kb / p.num_kb;
          const int kc = (kb - pass * p.num_kb) * BK;
          const CUtensorMap* ma = (p.passes > 1 && pass == 1) ? &tm_a1 : &tm_a0;
          const CUtensorMap* mb = (p.passes > 1 && pass == 0) ? &tm_b1 : &tm_b0;
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], tx_bytes);
          const int za = p.a.bcast_batch ? 0 : bt;
          if (EPI == kPairEpiConv) {
            // overlapping 32-row boxes: each warp's rows start conv_k - 1 early
            const int hal = p.epi.conv_k - 1, cu = 32 - hal;
            const int r0 = tm * 8 * cu + (int)rank * 4 * cu - hal;
#pragma unroll
            for (int j = 0; j < BM / 32; ++j)
              tma_load_3d_pair(smem_u32(sa + j * 4096), ma, fb, kc, r0 + j * cu, za);
          } else if (p.a.kind == 0) {
            tma_load_3d_pair(smem_u32(sa), ma, fb, kc, row_a, za);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 32; ++j)
              tma_load_3d_pair(smem_u32(sa + j * 4096), ma, fb, row_a + j * 32, kc, za);
          }
          const int zb = p.b.bcast_batch ? 0 : bt;
          if (p.b.kind == 0) {
            tma_load_3d_pair(smem_u32(sb), mb, fb, kc, row_b, zb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d_pair(smem_u32(sb + j * 4096), mb, fb, row_b + j * 32, kc, zb);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: the stages this CTA filled last are consumed (their empty
      // barrier completes only after the leader's MMAs read them), so no load
      // is still landing when the CTA leaves.
      volatile int no_abort = 0;
      for (int i = 0; i < C::STAGES && total_kb > 0; ++i) {
        if (--stage < 0) { stage = C::STAGES - 1; phase ^= 1; }
        // A stage never filled in the last lap was drained by an earlier lap.
        mbar_wait_cl(&empty_bar[stage], phase, &no_abort, p.err);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer (leader only)
    if (leader && lane == 0) {
      const bool a_mn = (p.a.kind == 1);
      const bool b_mn = (p.b.kind == 1);
      const uint32_t idesc = idesc_tf32_mn(PM, BN, a_mn, b_mn);
      const uint32_t peer = 1;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = 0; u < n_units && ok; ++u, ++local) {
        int t, k0, k1;
        pair_unit(p, pair, num_pairs, total_tiles, total_kb, u, t, k0, k1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_cl(&tempty_bar[acc], acc_phase ^ 1, &abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = k0; kb < k1; ++kb) {
          if (!mbar_wait_cl(&full_bar[stage], phase, &abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            uint64_t ad = a_mn ? sdesc_mnmajor(sa, kk) : sdesc_kmajor(sa, kk);
            uint64_t bd = b_mn ? sdesc_mnmajor(sb, kk) : sdesc_kmajor(sb, kk);
            umma2_tf32(d_tmem, ad, bd, idesc, ((kb - k0) | kk) ? 1u : 0u);
          }
          const uint32_t eb = smem_u32(&empty_bar[stage]);
          umma2_commit(eb);
          umma2_commit(mapa_shared(eb, peer));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        const uint32_t fb = smem_u32(&tfull_bar[acc]);
        umma2_commit(fb);
        umma2_commit(mapa_shared(fb, peer));
      }
      // All tensor-core work (which also writes the peer's TMEM) completes
      // before either CTA frees TMEM.
      umma2_commit(smem_u32(&drain_bar));
      volatile int no_abort = 0;
      mbar_wait_cl(&drain_bar, 0, &no_abort, p.err);
    }
  } else {
    // ---------------------------------------------------- epilogue (both CTAs)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int ew = warp - 2;       // epilogue warp index: 0..3, or 0..7 (kind 2)
    uint8_t* wstage = smem + C::STAGES * C::STAGE_BYTES + ew * (C::EPI_BYTES / n_epi);
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
    int local = 0;
    int chunk_seq = 0;
    for (int u = 0; u < n_units; ++u, ++local) {
      int t, k0, k1, bt, tm, tn;
      pair_unit(p, pair, num_pairs, total_tiles, total_kb, u, t, k0, k1);
      tile_coords(p, t, bt, tm, tn);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_cl(&tfull_bar[acc], acc_phase, &abort_flag, p.err)))
        break;
      tc_fence_after();
      const int m0 = tm * PM + (int)rank * BM + quarter * 32;
      const uint32_t row_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      // Stream-K roles.  A warp's share of a tile's partial (its 32 rows x BN
      // columns) is stored in register order, [chunk][quad][lane] float4s, so
      // every store and load of the warp covers 512 contiguous bytes; slot =
      // the contributing pair, then its CTA rank and the warp's quarter.
      const bool contributor = k1 < total_kb;
      const bool finisher = k0 > 0;
      if (contributor) {
        float4* wq = reinterpret_cast<float4*>(
            p.sk_ws + (((int64_t)pair * 2 + rank) * 4 + quarter) * (32 * BN));
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld_32x32(row_addr + (uint32_t)c, v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            wq[((c >> 5) * 8 + q) * 32 + lane] =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_add(p.sk_flags + t, 1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        continue;
      }
      const float* prow = nullptr;
      if (finisher) {
        // The head of this tile was computed by the previous pair (whose
        // range holds at least one whole tile); its 8 epilogue warps each
        // count their rows in sk_flags[t].
        bool ready = true;
        if (lane == 0) {
          unsigned long long t_start = globaltimer();
          while (ld_acquire_gpu(p.sk_flags + t) < 8) {
            if (abort_flag || globaltimer() - t_start > kWaitLimitNs) {
              if (!abort_flag) wxx_device_fail(p.err, WXX_DEV_ERR_MBAR_TIMEOUT);
              abort_flag = 1;
              ready = false;
              break;
            }
          }
        }
        ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
        if (!ready) break;
        prow = p.sk_ws + (((int64_t)(pair - 1) * 2 + rank) * 4 + quarter) * (32 * BN);
      }
      if constexpr (EPI == kPairEpiConv) {
        const int hal = p.epi.conv_k - 1, cu = 32 - hal;
        const int mc = tm * 8 * cu + (int)rank * 4 * cu + quarter * cu - hal;
        // this warp's columns [c_lo, c_lo + c_cnt) of the tile and its share of
        // the staging area (32 bytes of taps per column)
        const int c_cnt = BN * 4 / n_epi;
        const int c_lo = (ew >> 2) * c_cnt;
        float* ws = reinterpret_cast<float*>(wstage);
        if (mc + hal < p.M) {
          conv_stage_weights(p, tn * BN + c_lo, c_cnt, lane, ws);
          switch (p.epi.conv_k) {
            case 1: epi_conv_tile<1>(p, tn * BN + c_lo, c_cnt, mc, lane, row_addr + c_lo, ws); break;
            case 2: epi_conv_tile<2>(p, tn * BN + c_lo, c_cnt, mc, lane, row_addr + c_lo, ws); break;
            case 3: epi_conv_tile<3>(p, tn * BN + c_lo, c_cnt, mc, lane, row_addr + c_lo, ws); break;
            default: epi_conv_tile<4>(p, tn * BN + c_lo, c_cnt, mc, lane, row_addr + c_lo, ws); break;
          }
        }
        __syncwarp();   // the next tile restages ws
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        continue;
      }
      constexpr bool glu = GLU;  // host: GLU <=> p.epi.act == 2, never with stream-K partials
      constexpr bool amax = EPI == kPairEpiArgmax;
      float best_v = -1e38f;
      int best_c = 0;
#pragma unroll 1
      for (int c = 0; c < BN && m0 < p.M; c += glu ? 64 : 32) {
        const int n0 = tn * BN + c;
        if (n0 >= p.N) break;
        float v[32];
        int nc = n0;
        if constexpr (glu) {
          epi_glu_load<false>(p, bt, m0 + lane, n0, row_addr + (uint32_t)c, v);
          nc = n0 / 2;
        } else {
          tmem_ld_32x32(row_addr + (uint32_t)c, v);
        }
        if (prow != nullptr) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 w = __ldcg(reinterpret_cast<const float4*>(prow) + ((c >> 5) * 8 + q) * 32 + lane);
            v[4 * q] += w.x;
            v[4 * q + 1] += w.y;
            v[4 * q + 2] += w.z;
            v[4 * q + 3] += w.w;
          }
        }
        if (!glu) epi_apply<false>(p, bt, m0 + lane, n0, v);
        if constexpr (amax) {
          // the chunk's maximum by a tree (independent fmaxf: NaN loses);
          // the ordered scan with the tie keys only when it can change the
          // row's best (kept rolled: a compact epilogue leaves the MMA and
          // producer warps' instructions in the cache)
          float t16[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            t16[j] = fmaxf(n0 + j < p.N ? v[j] : -INFINITY, n0 + j + 16 < p.N ? v[j + 16] : -INFINITY);
#pragma unroll
          for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
            for (int j = 0; j < w; ++j) t16[j] = fmaxf(t16[j], t16[j + w]);
          const float cm = t16[0];
          if (cm > best_v || (cm == best_v && best_v > -1e38f)) {
            // the chunk's columns holding its maximum, the smallest tie key
            // among them, merged with the row's best so far
            unsigned eq = 0u;
#pragma unroll
            for (int j = 0; j < 32; ++j) eq |= (n0 + j < p.N && v[j] == cm) ? (1u << j) : 0u;
            int kc = c, kk = 0x7fffffff;
            for (unsigned m = eq; m != 0u; m &= m - 1u) {
              const int col = c + __ffs(m) - 1, k = amax_key(col);
              if (k < kk) {
                kk = k;
                kc = col;
              }
            }
            if (cm > best_v) {
              best_v = cm;
              best_c = kc;
            } else if (kk < amax_key(best_c)) {
              best_c = kc;
            }
          }
          continue;
        }
        uint8_t* buf = wstage + (chunk_seq & 1) * 4096;
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(buf + lane * 128 + ((q ^ (lane & 7)) << 4)) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tm_c, smem_u32(buf), nc, m0, bt);
          bulk_commit();
        }
        ++chunk_seq;
      }
      if (amax && m0 + lane < p.M)   // (constexpr: only the argmax form stores here)
        p.epi.amax[((int64_t)bt * p.M + m0 + lane) * p.tiles_n + tn] =
            make_float2(best_v, __int_as_float(best_c));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  // Neither CTA frees TMEM or exits while the leader's MMAs or the peer's
  // arrivals may still touch it.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace wxx_tc
