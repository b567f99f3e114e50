// Matmul and conv2d entry points on the tcgen05 GEMM engine (tc_gemm.cuh),
// plus an exact-fp32 SIMT kernel (mode 2) used as a cross-check and for
// callers that ask for full fp32 products.
//
// Reference: functional.matmul_add (functional/utils.py:378-499, matmul.wgsl)
//   C[b] = op(A[b]) @ op(B[b]) (+ bias), bias modes 0 none, 1 (N,), 2 (M,N),
//   3 (batch,M,N); an unbatched operand broadcasts (batch stride 0).
// Reference: functional.conv2d (functional/convolution.py:658-729, conv2d.wgsl)
//   NCHW cross-correlation as an implicit GEMM: rows = B*Ho*Wo output pixels,
//   columns = Cout, K = Cin*KH*KW.
#include "tc_gemm.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

extern "C" int wxx_memset(void* dst, int value, uint64_t nbytes);
extern "C" int wxx_malloc(void** out, uint64_t nbytes);
extern "C" int wxx_free(void* p);

using namespace wxx_tc;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// Encodes a 3-D fp32 tensor map {inner, outer, batch} with a {32, box_outer, 1}
// box.  K-major operands use the 128-byte swizzle with 16-byte chunks;
// MN-major operands (mn_major) the 128-byte swizzle with 32-byte chunks, the
// only shared-memory layout tcgen05 accepts for MN-major tf32.  Returns false
// when TMA cannot address the operand (alignment), so the caller gathers it.
bool encode_map(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                uint64_t batch, uint64_t ld_elems, uint64_t bs_elems, uint32_t box_outer,
                bool mn_major) {
  auto enc = get_encode();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_elems * 4) % 16) return false;
  if (batch > 1 && (bs_elems * 4) % 16) return false;
  if (inner == 0 || outer == 0 || batch == 0) return false;
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {ld_elems * 4, (batch > 1 ? bs_elems : ld_elems * outer) * 4};
  cuuint32_t box[3] = {32, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Describes a GEMM operand: `mn` rows (M for A, N for B) by K, batch-strided.
// k_contig: element (row, k) at row*ld + k; otherwise at k*ld + row.
struct OperandDesc {
  const float* base;
  int64_t rows, K, batch, ld, bs;
  bool k_contig;
  bool bcast;
};

// Fills `src` (and the tensor map when TMA can be used).
void setup_operand(const OperandDesc& d, int box_rows, bool allow_tma, OperandSrc& src,
                   CUtensorMap* map) {
  memset(&src, 0, sizeof(src));
  src.bcast_batch = d.bcast ? 1 : 0;
  int64_t nb = d.bcast ? 1 : d.batch;
  bool tma = false;
  if (allow_tma) {
    if (d.k_contig) {
      tma = encode_map(map, d.base, (uint64_t)d.K, (uint64_t)d.rows, (uint64_t)nb, (uint64_t)d.ld,
                       (uint64_t)d.bs, (uint32_t)box_rows, false);
      src.kind = 0;
    } else {
      tma = encode_map(map, d.base, (uint64_t)d.rows, (uint64_t)d.K, (uint64_t)nb, (uint64_t)d.ld,
                       (uint64_t)d.bs, 32u, true);
      src.kind = 1;
    }
  }
  if (!tma) {
    src.kind = 2;
    src.base = d.base;
    src.bs = d.bcast ? 0 : d.bs;
    src.s_row = d.k_contig ? d.ld : 1;
    src.s_k = d.k_contig ? 1 : d.ld;
    src.rows_total = (int)d.rows;
    src.k_total = (int)d.K;
  }
}

// Tensor map of the row-major output C [batch, M, N] for the TMA-store
// epilogue (32 x 32 boxes, 128-byte swizzle).  False when C is not
// 16-byte addressable; the epilogue then stores from registers.
bool encode_c_map(CUtensorMap* map, const GemmParams& p) {
  auto enc = get_encode();
  if (!enc || p.epi.kind != 0 || p.epi.bias_mode > 1) return false;
  if ((reinterpret_cast<uintptr_t>(p.epi.C) & 15) || ((int64_t)p.epi.ldc * 4) % 16) return false;
  // split-K partials: z runs over (batch, K-slice) of the workspace
  const int zdim = p.epi.raw ? p.batch * p.splits : p.batch;
  if (zdim > 1 && (p.epi.c_bs * 4) % 16) return false;
  const int64_t ncols = p.epi.act == 2 ? p.N / 2 : p.N;   // paired GLU halves the width
  cuuint64_t dims[3] = {(cuuint64_t)ncols, (cuuint64_t)p.M, (cuuint64_t)zdim};
  cuuint64_t strides[2] = {(cuuint64_t)p.epi.ldc * 4,
                           (cuuint64_t)(zdim > 1 ? p.epi.c_bs : (int64_t)p.epi.ldc * p.M) * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.epi.C, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
int launch_tc(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
              const CUtensorMap& b1, GemmParams& p) {
  using C = Cfg<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_kernel<BN, false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    WXX_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_kernel<BN, true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    attr_set = true;
  }
  p.tiles_m = (p.M + BM - 1) / BM;
  p.tiles_n = (p.N + BN - 1) / BN;
  // When A (per batch) fits comfortably in L2, stream B once with all row
  // blocks live; otherwise raster in bands of 16 row blocks so that a band of
  // A stays L2-resident while B is swept.
  int64_t a_bytes = (int64_t)p.M * p.K * 4;
  p.group_m = (a_bytes <= (48ll << 20) || p.tiles_m <= 16) ? p.tiles_m : 16;
  int64_t tiles = (int64_t)p.batch * p.tiles_m * p.tiles_n * p.splits;   // work units
  WXX_REQUIRE(tiles < (int64_t(1) << 31), "gemm: too many tiles");
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  p.epi.tma_store = encode_c_map(&mc, p) ? 1 : 0;
  WXX_REQUIRE(p.epi.act != 2 || p.epi.tma_store,
              "gemm: the paired GLU epilogue needs a TMA-storable output");
  WXX_REQUIRE(p.epi.tma_store || !p.epi.raw, "gemm: split-K workspace is not TMA-storable");
  WXX_REQUIRE(p.epi.tma_store || (p.epi.act == 0 && p.epi.res == nullptr),
              "gemm: a fused activation/residual needs a TMA-storable C");
  int grid = (int)(tiles < wxx::num_sms() ? tiles : wxx::num_sms());
  if (p.epi.act == 2)
    tc_gemm_kernel<BN, true><<<grid, NUM_THREADS, C::SMEM_BYTES, wxx::stream()>>>(a0, a1, b0, b1,
                                                                                mc, p);
  else
    tc_gemm_kernel<BN, false><<<grid, NUM_THREADS, C::SMEM_BYTES, wxx::stream()>>>(a0, a1, b0,
                                                                                 b1, mc, p);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// 256 x BN tiles on SM pairs (both operands TMA-fed, C stored by TMA).
template <int BN>
int launch_pair(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
                const CUtensorMap& b1, const CUtensorMap& mc, GemmParams& p) {
  using C = PairCfg<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_pair_kernel<BN, kPairEpiPlain>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    WXX_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_pair_kernel<BN, kPairEpiGlu>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    WXX_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_pair_kernel<BN, kPairEpiConv>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    WXX_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_pair_kernel<BN, kPairEpiArgmax>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    attr_set = true;
  }
  // Rows per pair tile: 256, or for the short-conv epilogue 8 warps of 32 rows
  // whose first conv_k - 1 rows overlap the previous warp's.
  const int tile_rows = p.epi.kind == 2 ? 8 * (32 - (p.epi.conv_k - 1)) : 2 * BM;
  p.tiles_m = (p.M + tile_rows - 1) / tile_rows;
  p.tiles_n = (p.N + BN - 1) / BN;
  int64_t a_bytes = (int64_t)p.M * p.K * 4;
  p.group_m = (a_bytes <= (48ll << 20) || p.tiles_m <= 8) ? p.tiles_m : 8;
  int64_t tiles = (int64_t)p.batch * p.tiles_m * p.tiles_n;
  WXX_REQUIRE(tiles < (int64_t(1) << 31), "gemm: too many tiles");
  // Persistent grid: as many SM pairs as can be co-resident (a GPC with an
  // odd number of free SMs leaves one out).
  static int max_pairs = -1;
  if (max_pairs < 0) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)(2 * (wxx::num_sms() / 2)));
    cfg.blockDim = dim3(PAIR_THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = wxx::stream();
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)tc_gemm_pair_kernel<BN, kPairEpiPlain>, &cfg) !=
            cudaSuccess ||
        n <= 0) {
      cudaGetLastError();
      n = wxx::num_sms() / 2;
    }
    max_pairs = n < wxx::num_sms() / 2 ? n : wxx::num_sms() / 2;
  }
  int pairs = max_pairs;
  if (tiles < pairs) pairs = (int)tiles;
  // Stream-K (opt-in, WXX_GEMM_STREAMK=1) when whole waves would leave many
  // pairs idle in the last one (> 5 % of the pair-time lost) and every pair
  // still covers >= 1 tile.  Off by default: inside the captured GPT2 step it
  // measured slower than whole tiles (the partial-tile traffic and the extra
  // memset outweigh the balanced last wave), although a lone K = 4096 product
  // gained 8 %.
  const char* sk_env = getenv("WXX_GEMM_STREAMK");
  const int64_t waves = (tiles + pairs - 1) / pairs;
  const bool sk = sk_env != nullptr && sk_env[0] == '1' && p.epi.act != 2 && p.epi.kind == 0 &&
                  p.epi.amax == nullptr &&
                  tiles >= pairs &&
                  (double)tiles / (double)(waves * pairs) < 0.95;
  void* ws = nullptr;
  void* flags = nullptr;
  p.sk = 0;
  p.sk_ws = nullptr;
  p.sk_flags = nullptr;
  if (sk) {
    int st = wxx_malloc(&ws, (uint64_t)pairs * 2 * BM * BN * sizeof(float));
    if (st == WXX_OK) st = wxx_malloc(&flags, (uint64_t)tiles * sizeof(int));
    if (st == WXX_OK) st = wxx_memset(flags, 0, (uint64_t)tiles * sizeof(int));
    if (st != WXX_OK) {
      wxx_free(ws);
      wxx_free(flags);
      return st;
    }
    p.sk = 1;
    p.sk_ws = (float*)ws;
    p.sk_flags = (int*)flags;
  }
  if (p.epi.kind == 2)
    tc_gemm_pair_kernel<BN, kPairEpiConv>
        <<<2 * pairs, PAIR_THREADS_CONV, C::SMEM_BYTES, wxx::stream()>>>(a0, a1, b0, b1, mc, p);
  else if (p.epi.act == 2)
    tc_gemm_pair_kernel<BN, kPairEpiGlu>
        <<<2 * pairs, PAIR_THREADS, C::SMEM_BYTES, wxx::stream()>>>(a0, a1, b0, b1, mc, p);
  else if (p.epi.amax != nullptr)
    tc_gemm_pair_kernel<BN, kPairEpiArgmax>
        <<<2 * pairs, PAIR_THREADS, C::SMEM_BYTES, wxx::stream()>>>(a0, a1, b0, b1, mc, p);
  else
    tc_gemm_pair_kernel<BN, kPairEpiPlain>
        <<<2 * pairs, PAIR_THREADS, C::SMEM_BYTES, wxx::stream()>>>(a0, a1, b0, b1, mc, p);
  const int st_launch = wxx::after_launch(__FILE__, __LINE__);
  int st_ws = wxx_free(ws);       // stream-ordered: valid for the kernel just enqueued
  int st_fl = wxx_free(flags);
  if (st_launch != WXX_OK) return st_launch;
  return st_ws ? st_ws : st_fl;
}

// SM-pair tiles are used for large TMA-fed products (enough 256 x 256 tiles
// to give every SM pair one); WXX_GEMM_PAIR=0 keeps single-SM tiles.
bool pair_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("WXX_GEMM_PAIR");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

int pick_bn(int64_t M, int64_t N, int64_t batch) {
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  // Prefer 256-wide tiles (lower shared-memory traffic per MMA) unless that
  // leaves most SMs idle.
  int64_t t256 = batch * ((M + 127) / 128) * ((N + 255) / 256);
  if (t256 >= wxx::num_sms() / 2) return 256;
  return 128;
}

// ------------------------------------------------------------ split-K

// K-slices for a product with few output tiles: enough units to cover the
// SMs once, at least 4 K-blocks per slice, at most 32 slices.
int choose_splits(int64_t tiles, int total_kb) {
  const int sms = wxx::num_sms();
  if (tiles >= sms / 2 || total_kb < 8) return 1;
  int64_t sp = sms / tiles;
  if (sp > total_kb / 4) sp = total_kb / 4;
  if (sp > 32) sp = 32;
  return sp < 2 ? 1 : (int)sp;
}

// out = alpha * (ws[0] + ws[1] + ... ) + bias, the K-slices of each batch
// entry added in index order (deterministic); ws is [batch][slice][M][N].
// kind 0: row-major C[b*c_bs + m*ldc + n] with bias_mode 1 (n), 2 (m, n) or
// 3 (b, m, n); kind 1 (batch 1): NCHW C[(img*N + n)*hw + pix] with
// m = img*hw + pix (m fastest there: coalesced writes).
__global__ void splitk_reduce_kernel(float* __restrict__ C, const float* __restrict__ ws,
                                     int splits, int batch, int M, int N, float alpha,
                                     const float* __restrict__ bias, int bias_mode, int kind,
                                     int64_t ldc, int64_t c_bs, int hw, ConvPost post,
                                     int round_tf32) {
  const int64_t MN = (int64_t)M * N;
  const int64_t total = MN * batch;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / MN;
    const int64_t r = i - b * MN;
    int64_t m, n;
    if (kind == 0) {
      m = r / N;
      n = r - m * N;
    } else {
      n = r / M;
      m = r - n * M;
    }
    const int64_t src = m * N + n;
    const float* w = ws + b * splits * MN;
    float acc = w[src];
    for (int k = 1; k < splits; ++k) acc += w[(int64_t)k * MN + src];
    float v = acc * alpha;
    if (bias != nullptr) {
      if (bias_mode == 1) v += bias[n];
      else if (bias_mode == 2) v += bias[src];
      else v += bias[b * MN + src];
    }
    if (kind == 0) {
      const int64_t o = b * c_bs + m * ldc + n;
      v = conv_post(post, v, (int)n, o);
      C[o] = round_tf32 ? tf32_rna(v) : v;
    } else {
      const int64_t img = m / hw, pix = m - img * hw;
      const int64_t o = (img * N + n) * hw + pix;
      C[o] = conv_post(post, v, (int)n, o);
    }
  }
}

// splitk_reduce_kernel for one row-major matrix (kind 0, batch 1) with N and
// ldc multiples of 4, 16-byte aligned C / ws / bias and splits * M * N below
// 2^31: four consecutive columns per thread with 16-byte loads and stores
// and 32-bit index arithmetic (the general kernel spends most of its
// instructions on 64-bit divisions).  Per element the same sum order and
// epilogue as splitk_reduce_kernel, so the same bits.
__global__ void splitk_reduce4_kernel(float* __restrict__ C, const float* __restrict__ ws,
                                      int splits, int M, int N, float alpha,
                                      const float* __restrict__ bias, int bias_mode, int ldc,
                                      ConvPost post, int round_tf32) {
  const int N4 = N >> 2;
  const int total4 = M * N4;
  const int MN = M * N;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += gridDim.x * blockDim.x) {
    const int m = i / N4;
    const int n = (i - m * N4) * 4;
    const int src = m * N + n;
    float4 acc = __ldg(reinterpret_cast<const float4*>(ws + src));
    for (int k = 1; k < splits; ++k) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(ws + k * MN + src));
      acc.x += w.x;
      acc.y += w.y;
      acc.z += w.z;
      acc.w += w.w;
    }
    float v[4] = {acc.x * alpha, acc.y * alpha, acc.z * alpha, acc.w * alpha};
    if (bias != nullptr) {
      const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + (bias_mode == 1 ? n : src)));
      v[0] += bb.x;
      v[1] += bb.y;
      v[2] += bb.z;
      v[3] += bb.w;
    }
    const int o = m * ldc + n;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = conv_post(post, v[j], n + j, (int64_t)(o + j));
      if (round_tf32) v[j] = tf32_rna(v[j]);
    }
    *reinterpret_cast<float4*>(C + o) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

int run_tc(int bn, const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
           const CUtensorMap& b1, GemmParams& p);

// Longest tensor-core accumulation chain (K-blocks over all passes) allowed in
// 3xTF32 mode.  The TMEM accumulator loses precision along a chain (measured:
// 3xTF32 max error 2.7e-6 at K = 1024, 1.1e-5 at 4096, 3.7e-5 at 16384 with
// whole-K accumulation; 0.7e-6 to 3.9e-6 when 512-deep slices are summed in
// fp32 on the CUDA cores), so fp32-faithful products are cut into slices.
constexpr int kMaxChainKb3x = 96;

// Sets p.splits / p.kb_per_split for BN-wide tiles; true when split-K applies:
// few output tiles (batch 1), or a 3xTF32 product longer than kMaxChainKb3x.
bool plan_splits(GemmParams& p, int bn) {
  const int total_kb = p.num_kb * p.passes;
  if (p.N % 4) return false;   // the workspace is written by TMA stores
  int sp = 1;
  if (p.passes > 1 && total_kb > kMaxChainKb3x) {
    sp = (total_kb + kMaxChainKb3x - 1) / kMaxChainKb3x;
  } else if (p.batch == 1) {
    const int64_t tiles = ((p.M + BM - 1) / BM) * (int64_t)((p.N + bn - 1) / bn);
    sp = choose_splits(tiles, total_kb);
  }
  if (sp <= 1) return false;
  p.kb_per_split = (total_kb + sp - 1) / sp;
  p.splits = (total_kb + p.kb_per_split - 1) / p.kb_per_split;   // no empty slice
  return p.splits > 1;
}

// Runs the GEMM of `p` (batch 1, epilogue kind 0 or 1 with at most a column
// bias) as p.splits K-slices into a workspace, then reduces into the real
// output.  p.epi holds the real output description on entry.
int run_splitk(int bn, const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
               const CUtensorMap& b1, GemmParams& p) {
  const EpiParams real = p.epi;
  const int64_t MN = (int64_t)p.M * p.N;
  void* ws = nullptr;
  int st = wxx_malloc(&ws, (uint64_t)p.batch * p.splits * MN * sizeof(float));
  if (st) return st;
  p.epi.kind = 0;
  p.epi.C = (float*)ws;
  p.epi.ldc = p.N;
  p.epi.c_bs = MN;
  p.epi.bias = nullptr;
  p.epi.bias_mode = 0;
  p.epi.alpha = 1.0f;
  p.epi.raw = 1;
  p.epi.round_tf32 = 0;
  p.epi.act = 0;
  p.epi.res = nullptr;
  memset(&p.epi.post, 0, sizeof(p.epi.post));
  st = run_tc(bn, a0, a1, b0, b1, p);
  const bool vec4 =
      real.kind == 0 && p.batch == 1 && p.N % 4 == 0 && real.ldc % 4 == 0 &&
      (int64_t)p.splits * MN < (int64_t(1) << 31) &&
      (int64_t)(p.M - 1) * real.ldc + p.N < (int64_t(1) << 31) &&
      (real.bias_mode == 0 || real.bias_mode == 1 || real.bias_mode == 2) &&
      !((reinterpret_cast<uintptr_t>(real.C) | reinterpret_cast<uintptr_t>(ws) |
         reinterpret_cast<uintptr_t>(real.bias_mode ? real.bias : nullptr)) & 15);
  if (st == WXX_OK && vec4) {
    splitk_reduce4_kernel<<<wxx::grid_for(MN / 4, 256), 256, 0, wxx::stream()>>>(
        real.C, (const float*)ws, p.splits, p.M, p.N, real.alpha,
        real.bias_mode ? real.bias : nullptr, real.bias_mode, real.ldc, real.post,
        real.round_tf32);
    st = wxx::after_launch(__FILE__, __LINE__);
  } else if (st == WXX_OK) {
    splitk_reduce_kernel<<<wxx::grid_for(MN * p.batch, 256), 256, 0, wxx::stream()>>>(
        real.C, (const float*)ws, p.splits, p.batch, p.M, p.N, real.alpha,
        real.bias_mode ? real.bias : nullptr, real.bias_mode, real.kind,
        real.kind == 0 ? (int64_t)real.ldc : 0, real.kind == 0 ? real.c_bs : 0, real.hw_out,
        real.post, real.kind == 0 ? real.round_tf32 : 0);
    st = wxx::after_launch(__FILE__, __LINE__);
  }
  int st2 = wxx_free(ws);   // stream-ordered: valid for the kernels just enqueued
  p.epi = real;
  return st ? st : st2;
}

int run_tc(int bn, const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
           const CUtensorMap& b1, GemmParams& p) {
  switch (bn) {
    case 64: return launch_tc<64>(a0, a1, b0, b1, p);
    case 128: return launch_tc<128>(a0, a1, b0, b1, p);
    default: return launch_tc<256>(a0, a1, b0, b1, p);
  }
}

// ------------------------------------------------------------ 3xTF32 residuals

// lo[i] = x[i] - tf32(x[i]) where tf32() clears the 13 low mantissa bits --
// exactly what the tensor core reads from an fp32 word (it truncates), so the
// raw operand serves as the "hi" part and only the residual needs storage.
__global__ void tf32_residual_kernel(float* __restrict__ lo, const float* __restrict__ x,
                                     int64_t n) {
  const bool vec = !((reinterpret_cast<uintptr_t>(lo) | reinterpret_cast<uintptr_t>(x)) & 15);
  int64_t n4 = vec ? n / 4 : 0;
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n4; i += step) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    float4 r;
    r.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    r.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    r.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    r.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    reinterpret_cast<float4*>(lo)[i] = r;
  }
  for (int64_t i = n4 * 4 + tid; i < n; i += step) {
    float v = x[i];
    lo[i] = v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  }
}

// Elements spanned by an operand (from its base pointer).
int64_t operand_extent(const OperandDesc& d) {
  int64_t nb = d.bcast ? 1 : d.batch;
  int64_t inner_last = d.k_contig ? (d.rows - 1) * d.ld + d.K : (d.K - 1) * d.ld + d.rows;
  return (nb - 1) * d.bs + inner_last;
}

// For a TMA-fed operand in 3xTF32 mode: writes its residual into `*scratch`
// (allocated here, released by the caller after the GEMM is enqueued) and
// encodes the residual's tensor map.
int make_residual(const OperandDesc& d, const OperandSrc& src, int box_rows, CUtensorMap* map_lo,
                  void** scratch) {
  *scratch = nullptr;
  if (src.kind >= 2) return WXX_OK;  // gathered operands are split on the fly
  int64_t n = operand_extent(d);
  int st = wxx_malloc(scratch, (uint64_t)n * sizeof(float));
  if (st) return st;
  tf32_residual_kernel<<<wxx::grid_for(n / 4 + 1, 256), 256, 0, wxx::stream()>>>(
      (float*)*scratch, d.base, n);
  WXX_LAUNCH_CHECK();
  OperandDesc dl = d;
  dl.base = (const float*)*scratch;
  OperandSrc tmp;
  setup_operand(dl, box_rows, true, tmp, map_lo);
  if (tmp.kind != src.kind) {
    wxx::set_error("gemm: residual operand lost TMA addressability");
    return WXX_E_STATE;
  }
  return WXX_OK;
}

// ------------------------------------------------------------ exact fp32 SIMT

// C[b] (M x N, N <= kSkinnyN) = alpha * op(A[b]) op(B[b]) + bias: one warp per
// output row, lanes striding K, the N partial sums combined by shuffles in a
// fixed order (deterministic).
constexpr int kSkinnyN = 16;

__global__ void __launch_bounds__(256) skinny_gemm_kernel(
    float* __restrict__ C, const float* __restrict__ A, const float* __restrict__ B,
    const float* __restrict__ bias, int64_t batch, int M, int N, int K, int64_t a_bs,
    int64_t b_bs, int64_t lda, int64_t ldb, int trans_a, int trans_b, int bias_mode, float alpha) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = (((int64_t)blockIdx.x * blockDim.x) + threadIdx.x) >> 5; row < batch * M;
       row += warps) {
    const int64_t bt = row / M;
    const int m = (int)(row - bt * M);
    const float* Ab = A + bt * a_bs;
    const float* Bb = B + bt * b_bs;
    float acc[kSkinnyN];
#pragma unroll
    for (int n = 0; n < kSkinnyN; ++n) acc[n] = 0.f;
    for (int k = lane; k < K; k += 32) {
      const float a = trans_a ? Ab[(int64_t)k * lda + m] : Ab[(int64_t)m * lda + k];
#pragma unroll
      for (int n = 0; n < kSkinnyN; ++n)
        if (n < N)
          acc[n] = fmaf(a, trans_b ? Bb[(int64_t)n * ldb + k] : Bb[(int64_t)k * ldb + n], acc[n]);
    }
#pragma unroll
    for (int n = 0; n < kSkinnyN; ++n) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[n] += __shfl_xor_sync(0xffffffffu, acc[n], off);
    }
    if (lane < N) {
      float v = 0.f;
#pragma unroll
      for (int n = 0; n < kSkinnyN; ++n) v = (n == lane) ? acc[n] : v;
      v *= alpha;
      if (bias_mode == 1) v += bias[lane];
      C[bt * M * N + (int64_t)m * N + lane] = v;
    }
  }
}

// ------------------------------------------------------------ few rows (decode)

// C (M <= 32 rows) = act(alpha * A' @ W^T + bias) + res for a K-major weight W
// (N, K): the decode step's products, where the weight is read once and each
// of its values meets only M activations, so the time is the weight stream.
// A tile-based GEMM gives such a product N / 256 CTAs; here a CTA takes
// kGemvCols columns and its 8 warps split K, so N = 1024 spreads over 256
// CTAs with every warp's weight loads in flight at once.  Per warp:
// kGemvCols weight rows and 8 activation rows as float4 loads along K, 32
// fp32 accumulators (column c, row r at index 8c + r), reduced across the
// lanes by a halving exchange (31 shuffles; lane l ends with the sum for
// index l), then over the K-split warps in fixed order through shared
// memory.  Exact fp32 products; the epilogue is the tensor-core path's
// (alpha, bias, GELU, residual, TF32 rounding of the stored value).
// LN: A' = LayerNorm(A) over its K entries (gamma, beta; the LayerNorm
// kernel's two-pass statistics and expression), computed by every CTA for
// the rows it needs -- the block's norm and the next product in one launch.
constexpr int kGemvCols = 4;
constexpr int kGemvWarps = 8;
constexpr int kGemvMaxRows = 32;

template <bool LN>
__global__ void __launch_bounds__(kGemvWarps * 32, 2) rows_gemv_kernel(
    float* __restrict__ C, const float* __restrict__ A, int64_t lda, const float* __restrict__ W,
    int64_t ldw, const float* __restrict__ bias, int M, int N, int K, float alpha, int act,
    const float* __restrict__ res, int round_out, const float* __restrict__ ln_g,
    const float* __restrict__ ln_b, float ln_eps) {
  __shared__ float part[kGemvWarps][32];
  __shared__ float s_mu[kGemvMaxRows], s_inv[kGemvMaxRows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kq = ((K + kGemvWarps * 128 - 1) / (kGemvWarps * 128)) * 128;
  const int kb = warp * kq, ke = min(K, kb + kq);
  if (LN) {
    for (int m = warp; m < M; m += kGemvWarps) {
      const float* ar = A + (int64_t)m * lda;
      // float4 loads, eight in flight per lane (K % 4 == 0)
      float sum = 0.f;
      for (int k0 = lane * 4; k0 < K; k0 += 32 * 4 * 8) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = k0 + i * 128;
          v[i] = k < K ? __ldg(reinterpret_cast<const float4*>(ar + k))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float mean = sum / (float)K;
      float ss = 0.f;
      for (int k0 = lane * 4; k0 < K; k0 += 32 * 4 * 8) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = k0 + i * 128;
          v[i] = k < K ? __ldg(reinterpret_cast<const float4*>(ar + k))
                       : make_float4(mean, mean, mean, mean);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
          ss += (a * a + b * b) + (c * c + d * d);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float var = fmaxf(0.f, ss / (float)K);
      if (lane == 0) {
        s_mu[m] = mean;
        s_inv[m] = var > 0.f ? rsqrtf(var + ln_eps) : 0.f;
      }
    }
    __syncthreads();
  }
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  // column groups handed out grid-stride: the row statistics above are made
  // once per CTA, not once per group.  (Loading the next group's weights
  // while this group's products, reduction and stores ran was measured
  // slower: 1.20 against 1.07 ms a GPT2-scaled decode step.)
  const int groups = (N + kGemvCols - 1) / kGemvCols;
  for (int grp = blockIdx.x; grp < groups; grp += gridDim.x) {
  const int n0 = grp * kGemvCols;
  const float* wr[kGemvCols];
  bool wv[kGemvCols];
#pragma unroll
  for (int c = 0; c < kGemvCols; ++c) {
    wv[c] = n0 + c < N;
    wr[c] = W + (int64_t)(wv[c] ? n0 + c : 0) * ldw;
  }
  for (int m0 = 0; m0 < M; m0 += 8) {
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    for (int k = kb + lane * 4; k < ke; k += 128) {
      float4 w4[kGemvCols];
#pragma unroll
      for (int c = 0; c < kGemvCols; ++c)
        w4[c] = wv[c] ? __ldg(reinterpret_cast<const float4*>(wr[c] + k)) : zero;
      float4 g4 = zero, b4 = zero;
      if (LN) {
        g4 = __ldg(reinterpret_cast<const float4*>(ln_g + k));
        b4 = __ldg(reinterpret_cast<const float4*>(ln_b + k));
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        float4 a = (m0 + r < M)
            ? __ldg(reinterpret_cast<const float4*>(A + (int64_t)(m0 + r) * lda + k)) : zero;
        if (LN && m0 + r < M) {
          const float mu = s_mu[m0 + r], inv = s_inv[m0 + r];
          a.x = (a.x - mu) * inv * g4.x + b4.x;
          a.y = (a.y - mu) * inv * g4.y + b4.y;
          a.z = (a.z - mu) * inv * g4.z + b4.z;
          a.w = (a.w - mu) * inv * g4.w + b4.w;
        }
#pragma unroll
        for (int c = 0; c < kGemvCols; ++c) {
          float t = acc[8 * c + r];
          t = fmaf(a.x, w4[c].x, t);
          t = fmaf(a.y, w4[c].y, t);
          t = fmaf(a.z, w4[c].z, t);
          t = fmaf(a.w, w4[c].w, t);
          acc[8 * c + r] = t;
        }
      }
    }
    // halving exchange: after the step with distance s a lane keeps the half
    // of its indices selected by its lane bit s, summed with its partner's
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
      const bool upper = (lane & s) != 0;
#pragma unroll
      for (int i = 0; i < s; ++i) {
        const float send = upper ? acc[i] : acc[i + s];
        const float keep = upper ? acc[i + s] : acc[i];
        acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
      }
    }
    part[warp][lane] = acc[0];
    __syncthreads();
    if (warp == 0) {
      float v = part[0][lane];
#pragma unroll
      for (int q = 1; q < kGemvWarps; ++q) v += part[q][lane];
      const int n = n0 + (lane >> 3), m = m0 + (lane & 7);
      if (n < N && m < M) {
        v = bias != nullptr ? v * alpha + __ldg(bias + n) : v * alpha;
        if (act == 1) v = gelu_tanh(v);
        if (res != nullptr) v += __ldg(res + (int64_t)m * N + n);
        if (round_out) v = tf32_rna(v);
        C[(int64_t)m * N + n] = v;
      }
    }
    __syncthreads();
  }
  }
}

// The same products for K <= 2048 with the weight streamed through shared
// memory: cp.async copies (16 bytes each, tracked by commit groups, no
// registers held while in flight) fill kGvStages stages of 16 columns x 256
// K-values ahead of the math, so a CTA keeps ~48 KB of weight loads in
// flight instead of one float4 per column per lane.  The (LayerNorm-ed)
// activation rows are staged in shared memory once per CTA and pass of 8
// rows.  Thread t takes column t / 16 of a tile and K-values 4 (t % 16) + 64 j
// of each chunk, 8 row accumulators; the 16 lanes of a column are summed by
// shuffles (fixed order) when its tile's last chunk is done.
constexpr int kGvCols = 16;
constexpr int kGvKc = 256;
constexpr int kGvStages = 4;
constexpr int kGvMaxK = 2048;
constexpr int kGvStageFloats = kGvCols * kGvKc;

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gptr, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr), "l"(gptr),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <bool LN>
__global__ void __launch_bounds__(256, 2) rows_gemv_async_kernel(
    float* __restrict__ C, const float* __restrict__ A, int64_t lda, const float* __restrict__ W,
    int64_t ldw, const float* __restrict__ bias, int M, int N, int K, float alpha, int act,
    const float* __restrict__ res, int round_out, const float* __restrict__ ln_g,
    const float* __restrict__ ln_b, float ln_eps) {
  extern __shared__ __align__(16) float gsm[];
  float* ws = gsm;                                   // kGvStages x (16 cols x 256)
  float* as = gsm + kGvStages * kGvStageFloats;      // 8 rows x K
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int col = t >> 4, kl = t & 15;
  const int nkc = (K + kGvKc - 1) / kGvKc;
  const int tiles = (N + kGvCols - 1) / kGvCols;
  const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int chunks = my_tiles * nkc;
  const uint32_t ws_addr = smem_u32(ws);
  // copy chunk q (tile blockIdx.x + (q / nkc) * gridDim.x, K-chunk q % nkc) into its stage
  auto issue = [&](int q) {
    if (q < chunks) {
      const int tile = blockIdx.x + (q / nkc) * gridDim.x, kc = q - (q / nkc) * nkc;
      const int stage = q % kGvStages;
#pragma unroll
      for (int i = 0; i < kGvStageFloats / 4 / 256; ++i) {
        const int e = t + i * 256;                 // float4 index in the stage
        const int c = e / (kGvKc / 4), k4 = e - c * (kGvKc / 4);
        const int n = tile * kGvCols + c, k = kc * kGvKc + k4 * 4;
        const bool ok = n < N && k < K;
        const float* src = W + (ok ? (int64_t)n * ldw + k : 0);
        cp_async16(ws_addr + (uint32_t)((stage * kGvStageFloats + c * kGvKc + k4 * 4) * 4), src,
                   ok ? 16 : 0);
      }
    }
    cp_async_commit();   // one group per chunk slot, empty past the end
  };
  for (int m0 = 0; m0 < M; m0 += 8) {
    for (int q = 0; q < kGvStages - 1; ++q) issue(q);
    // activation rows m0 .. m0+7 (LayerNorm-ed) into shared memory, zero past
    // M and K: warp r holds row m0 + r in registers (all its float4 loads in
    // flight at once), takes the two-pass statistics from them and stores
    // the normalised row
    {
      const int r = warp, m = m0 + r;
      const int kp = nkc * kGvKc;                 // padded row length, <= kGvMaxK
      const float* ar = A + (int64_t)(m < M ? m : 0) * lda;
      float4 v[kGvMaxK / 128];
#pragma unroll
      for (int i = 0; i < kGvMaxK / 128; ++i) {
        const int k = (i * 32 + lane) * 4;
        v[i] = (m < M && k < K) ? __ldg(reinterpret_cast<const float4*>(ar + k))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float mean = 0.f, inv = 1.f;
      if (LN) {
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kGvMaxK / 128; ++i) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mean = sum / (float)K;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kGvMaxK / 128; ++i) {
          const int k = (i * 32 + lane) * 4;
          if (k < K) {
            const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean,
                        d = v[i].w - mean;
            ss += (a * a + b * b) + (c * c + d * d);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float var = fmaxf(0.f, ss / (float)K);
        inv = var > 0.f ? rsqrtf(var + ln_eps) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kGvMaxK / 128; ++i) {
        const int k = (i * 32 + lane) * 4;
        if (k < kp) {
          float4 o = v[i];
          if (LN && m < M && k < K) {
            const float4 g4 = __ldg(reinterpret_cast<const float4*>(ln_g + k));
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(ln_b + k));
            o.x = (o.x - mean) * inv * g4.x + b4.x;
            o.y = (o.y - mean) * inv * g4.y + b4.y;
            o.z = (o.z - mean) * inv * g4.z + b4.z;
            o.w = (o.w - mean) * inv * g4.w + b4.w;
          }
          *reinterpret_cast<float4*>(as + r * kp + k) = o;
        }
      }
    }
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = 0.f;
    for (int q = 0; q < chunks; ++q) {
      cp_async_wait<kGvStages - 2>();
      __syncthreads();   // chunk q landed for every thread; chunk q - 1's math is done
      issue(q + kGvStages - 1);
      const int kc = q % nkc, stage = q % kGvStages;
      const float* wc = ws + stage * kGvStageFloats + col * kGvKc;
      const float* ac = as + kc * kGvKc;
#pragma unroll
      for (int j = 0; j < kGvKc / 64; ++j) {
        const int k = kl * 4 + j * 64;
        const float4 w4 = *reinterpret_cast<const float4*>(wc + k);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float4 a4 = *reinterpret_cast<const float4*>(ac + r * (nkc * kGvKc) + k);
          float tt = acc[r];
          tt = fmaf(a4.x, w4.x, tt);
          tt = fmaf(a4.y, w4.y, tt);
          tt = fmaf(a4.z, w4.z, tt);
          tt = fmaf(a4.w, w4.w, tt);
          acc[r] = tt;
        }
      }
      if (kc == nkc - 1) {
        // the tile's 16 K-lanes of each column summed in a fixed order
#pragma unroll
        for (int r = 0; r < 8; ++r) {
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        }
        const int tile = blockIdx.x + (q / nkc) * gridDim.x;
        const int n = tile * kGvCols + col, m = m0 + kl;
        float v = acc[0];
#pragma unroll
        for (int r = 1; r < 8; ++r) v = (kl == r) ? acc[r] : v;
        if (kl < 8 && n < N && m < M) {
          v = bias != nullptr ? v * alpha + __ldg(bias + n) : v * alpha;
          if (act == 1) v = gelu_tanh(v);
          if (res != nullptr) v += __ldg(res + (int64_t)m * N + n);
          if (round_out) v = tf32_rna(v);
          C[(int64_t)m * N + n] = v;
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r] = 0.f;
      }
    }
    cp_async_wait<0>();
    __syncthreads();   // the stages and the rows are reused by the next pass
  }
}

// Few rows, K <= 1024, wide N (the decode step's q/k/v, fc1 and LM head):
// every warp owns 2 weight rows (output columns) whole, so all 2 x K / 4
// float4 loads of a lane are in flight at once; the (LayerNorm-ed) activation
// rows sit in shared memory, staged once per CTA and pass of 8 rows, and the
// CTA walks column blocks of 16 grid-stride with no barrier between them.
// The 16 accumulators (column c, row r at 8c + r) are summed across the
// lanes by a halving exchange over lane bits 3..0 and one shuffle across the
// half-warps; exact fp32, the epilogue of rows_gemv_kernel.
constexpr int kG3Cols = 2;
constexpr int kG3MaxK = 1024;

template <bool LN>
__global__ void __launch_bounds__(256, 2) rows_gemv_k1k_kernel(
    float* __restrict__ C, const float* __restrict__ A, int64_t lda, const float* __restrict__ W,
    int64_t ldw, const float* __restrict__ bias, int M, int N, int K, float alpha, int act,
    const float* __restrict__ res, int round_out, const float* __restrict__ ln_g,
    const float* __restrict__ ln_b, float ln_eps) {
  __shared__ __align__(16) float as[8 * kG3MaxK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cols_per_cta = 8 * kG3Cols;
  const int blocks = (N + cols_per_cta - 1) / cols_per_cta;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w[kG3Cols][kG3MaxK / 128];
  auto load_w = [&](int blk) {
    const int n0 = blk * cols_per_cta + warp * kG3Cols;
#pragma unroll
    for (int c = 0; c < kG3Cols; ++c) {
      const float* wr = W + (int64_t)(n0 + c < N ? n0 + c : 0) * ldw;
#pragma unroll
      for (int i = 0; i < kG3MaxK / 128; ++i) {
        const int k = (i * 32 + lane) * 4;
        w[c][i] = (n0 + c < N && k < K) ? __ldg(reinterpret_cast<const float4*>(wr + k)) : zero;
      }
    }
  };
  for (int m0 = 0; m0 < M; m0 += 8) {
    if (m0 > 0) __syncthreads();   // the previous pass is done with the rows
    {
      // warp r stages row m0 + r: its float4s in registers, two-pass
      // statistics from them (LN), then the normalised row
      const int r = warp, m = m0 + r;
      const float* ar = A + (int64_t)(m < M ? m : 0) * lda;
      float4 v[kG3MaxK / 128];
#pragma unroll
      for (int i = 0; i < kG3MaxK / 128; ++i) {
        const int k = (i * 32 + lane) * 4;
        v[i] = (m < M && k < K) ? __ldg(reinterpret_cast<const float4*>(ar + k)) : zero;
      }
      float mean = 0.f, inv = 1.f;
      if (LN) {
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kG3MaxK / 128; ++i) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mean = sum / (float)K;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kG3MaxK / 128; ++i) {
          const int k = (i * 32 + lane) * 4;
          if (k < K) {
            const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean,
                        d = v[i].w - mean;
            ss += (a * a + b * b) + (c * c + d * d);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float var = fmaxf(0.f, ss / (float)K);
        inv = var > 0.f ? rsqrtf(var + ln_eps) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kG3MaxK / 128; ++i) {
        const int k = (i * 32 + lane) * 4;
        float4 o = v[i];
        if (LN && m < M && k < K) {
          const float4 g4 = __ldg(reinterpret_cast<const float4*>(ln_g + k));
          const float4 b4 = __ldg(reinterpret_cast<const float4*>(ln_b + k));
          o.x = (o.x - mean) * inv * g4.x + b4.x;
          o.y = (o.y - mean) * inv * g4.y + b4.y;
          o.z = (o.z - mean) * inv * g4.z + b4.z;
          o.w = (o.w - mean) * inv * g4.w + b4.w;
        }
        *reinterpret_cast<float4*>(as + r * kG3MaxK + k) = o;
      }
    }
    __syncthreads();
    for (int blk = blockIdx.x; blk < blocks; blk += gridDim.x) {
      const int n0 = blk * cols_per_cta + warp * kG3Cols;
      load_w(blk);   // (issuing the first block's loads before the row staging measured slower)
      float acc[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) acc[q] = 0.f;
#pragma unroll
      for (int i = 0; i < kG3MaxK / 128; ++i) {
        const int k = (i * 32 + lane) * 4;
        if (k < K) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const float4 a = *reinterpret_cast<const float4*>(as + r * kG3MaxK + k);
#pragma unroll
            for (int c = 0; c < kG3Cols; ++c) {
              float t = acc[8 * c + r];
              t = fmaf(a.x, w[c][i].x, t);
              t = fmaf(a.y, w[c][i].y, t);
              t = fmaf(a.z, w[c][i].z, t);
              t = fmaf(a.w, w[c][i].w, t);
              acc[8 * c + r] = t;
            }
          }
        }
      }
      // halving exchange over lane bits 3..0 (lane l keeps index l & 15),
      // then the two half-warps added
#pragma unroll
      for (int sft = 8; sft >= 1; sft >>= 1) {
        const bool upper = (lane & sft) != 0;
#pragma unroll
        for (int q = 0; q < sft; ++q) {
          const float send = upper ? acc[q] : acc[q + sft];
          const float keep = upper ? acc[q + sft] : acc[q];
          acc[q] = keep + __shfl_xor_sync(0xffffffffu, send, sft);
        }
      }
      float v = acc[0] + __shfl_xor_sync(0xffffffffu, acc[0], 16);
      const int n = n0 + ((lane & 15) >> 3), m = m0 + (lane & 7);
      if (lane < 16 && n < N && m < M) {
        v = bias != nullptr ? v * alpha + __ldg(bias + n) : v * alpha;
        if (act == 1) v = gelu_tanh(v);
        if (res != nullptr) v += __ldg(res + (int64_t)m * N + n);
        if (round_out) v = tf32_rna(v);
        C[(int64_t)m * N + n] = v;
      }
    }
  }
}

// WXX_GEMV_ASYNC=1 selects the shared-memory-streamed form for K <= kGvMaxK
// (read once); by default the register form runs: 1.07 against 1.25-1.27 ms
// per GPT2-scaled decode step (batch 8) when measured side by side.
bool gemv_async_enabled() {
  static int on = [] {
    const char* e = std::getenv("WXX_GEMV_ASYNC");
    return (e != nullptr && e[0] == '1') ? 1 : 0;
  }();
  return on != 0;
}

// True when rows_gemv_kernel takes the product (see its comment).
bool gemv_fits(int64_t rows, int64_t N, int64_t K, int64_t lda, int64_t ldb, const void* A,
               const void* B) {
  return rows >= 1 && rows <= kGemvMaxRows && N >= 64 && K >= 128 && K % 4 == 0 &&
         lda % 4 == 0 && ldb % 4 == 0 && (lda >= K || rows == 1) &&
         !(reinterpret_cast<uintptr_t>(A) & 15) && !(reinterpret_cast<uintptr_t>(B) & 15) &&
         N < (int64_t(1) << 31) / kGemvCols;
}

int launch_gemv(float* C, const float* A, int64_t lda, const float* W, int64_t ldw,
                const float* bias, int rows, int N, int K, float alpha, int act, const float* res,
                int round_out, const float* ln_g, const float* ln_b, float ln_eps) {
  if (K <= kG3MaxK && N >= 2048 && !gemv_async_enabled()) {
    const int64_t blocks = (N + 8 * kG3Cols - 1) / (8 * kG3Cols);
    const unsigned grid = (unsigned)std::min<int64_t>(blocks, 2 * (int64_t)wxx::num_sms());
    if (ln_g != nullptr)
      rows_gemv_k1k_kernel<true><<<grid, 256, 0, wxx::stream()>>>(
          C, A, lda, W, ldw, bias, rows, N, K, alpha, act, res, round_out, ln_g, ln_b, ln_eps);
    else
      rows_gemv_k1k_kernel<false><<<grid, 256, 0, wxx::stream()>>>(
          C, A, lda, W, ldw, bias, rows, N, K, alpha, act, res, round_out, nullptr, nullptr, 0.f);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  if (K <= kGvMaxK && gemv_async_enabled()) {
    const int nkc = (K + kGvKc - 1) / kGvKc;
    const size_t smem = (size_t)(kGvStages * kGvStageFloats + 8 * nkc * kGvKc) * sizeof(float);
    static bool attr = false;
    if (!attr) {
      WXX_CUDA_CHECK(cudaFuncSetAttribute(rows_gemv_async_kernel<true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)((kGvStages * kGvStageFloats + 8 * kGvMaxK) * 4)));
      WXX_CUDA_CHECK(cudaFuncSetAttribute(rows_gemv_async_kernel<false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)((kGvStages * kGvStageFloats + 8 * kGvMaxK) * 4)));
      attr = true;
    }
    const int64_t tiles = (N + kGvCols - 1) / kGvCols;
    const unsigned grid = (unsigned)std::min<int64_t>(tiles, 2 * (int64_t)wxx::num_sms());
    if (ln_g != nullptr)
      rows_gemv_async_kernel<true><<<grid, 256, smem, wxx::stream()>>>(
          C, A, lda, W, ldw, bias, rows, N, K, alpha, act, res, round_out, ln_g, ln_b, ln_eps);
    else
      rows_gemv_async_kernel<false><<<grid, 256, smem, wxx::stream()>>>(
          C, A, lda, W, ldw, bias, rows, N, K, alpha, act, res, round_out, nullptr, nullptr, 0.f);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  const int64_t groups = (N + kGemvCols - 1) / kGemvCols;
  const unsigned grid = (unsigned)std::min<int64_t>(groups, 2 * (int64_t)wxx::num_sms());
  if (ln_g != nullptr)
    rows_gemv_kernel<true><<<grid, kGemvWarps * 32, 0, wxx::stream()>>>(
        C, A, lda, W, ldw, bias, rows, N, K, alpha, act, res, round_out, ln_g, ln_b, ln_eps);
  else
    rows_gemv_kernel<false><<<grid, kGemvWarps * 32, 0, wxx::stream()>>>(
        C, A, lda, W, ldw, bias, rows, N, K, alpha, act, res, round_out, nullptr, nullptr, 0.f);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// 64x64 output tile, K-step 16, 4x4 outputs per thread, fp32 FMA.
__global__ void __launch_bounds__(256) simt_gemm_kernel(
    float* __restrict__ C, const float* __restrict__ A, const float* __restrict__ B,
    const float* __restrict__ bias, int M, int N, int K, int64_t a_bs, int64_t b_bs, int64_t lda,
    int64_t ldb, int trans_a, int trans_b, int bias_mode, float alpha) {
  __shared__ float As[16][68];
  __shared__ float Bs[16][68];
  int bt = blockIdx.z;
  const float* Ab = A + (int64_t)bt * a_bs;
  const float* Bb = B + (int64_t)bt * b_bs;
  int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      int kk = e / 64, mm = e % 64;
      int m = m0 + mm, k = k0 + kk;
      float v = 0.f;
      if (m < M && k < K) v = trans_a ? Ab[(int64_t)k * lda + m] : Ab[(int64_t)m * lda + k];
      As[kk][mm] = v;
      int n = n0 + mm;
      float w = 0.f;
      if (n < N && k < K) w = trans_b ? Bb[(int64_t)n * ldb + k] : Bb[(int64_t)k * ldb + n];
      Bs[kk][mm] = w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    int m = m0 + ty * 4 + i;
    if (m >= M) continue;
    for (int j = 0; j < 4; ++j) {
      int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float o = acc[i][j] * alpha;
      if (bias_mode == 1) o += bias[n];
      else if (bias_mode == 2) o += bias[(int64_t)m * N + n];
      else if (bias_mode == 3) o += bias[(int64_t)bt * M * N + (int64_t)m * N + n];
      C[(int64_t)bt * M * N + (int64_t)m * N + n] = o;
    }
  }
}

}  // namespace

// C (dense [batch, M, N]) = alpha * op(A) @ op(B) (+ bias).
//   A: trans_a = 0 -> element (m, k) at A[b*a_bs + m*lda + k]; 1 -> A[b*a_bs + k*lda + m]
//   B: trans_b = 0 -> element (k, n) at B[b*b_bs + k*ldb + n]; 1 -> B[b*b_bs + n*ldb + k]
//   a_bs / b_bs = 0 broadcasts that operand over the batch.
//   bias_mode: 0 none, 1 bias[n], 2 bias[m*N + n], 3 bias[b*M*N + m*N + n]
//   mode: 0 TF32 tensor cores, 1 3xTF32 tensor cores (fp32-faithful), 2 fp32 SIMT.
namespace {

// wxx_matmul with the TMA-store epilogue's optional GELU (act = 1) and
// residual matrix (res, dense [batch, M, N]); act/res need mode 0/1 and a
// 16-byte addressable C (checked by wxx_linear).
int matmul_impl(float* C, const float* A, const float* B, const float* bias, int64_t batch,
                int64_t M, int64_t N, int64_t K, int64_t a_bs, int64_t b_bs, int64_t lda,
                int64_t ldb, int trans_a, int trans_b, int bias_mode, float alpha, int mode,
                int act, const float* res, float2* amax_ws = nullptr) {
  WXX_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "wxx_matmul: negative size");
  WXX_REQUIRE(mode >= 0 && mode <= 3, "wxx_matmul: mode %d not in 0..3", mode);
  // mode 3: TF32 products with the stored result rounded to the nearest TF32
  // value, for outputs that are read only as operands of TF32 products.
  const int round_out = mode == 3 ? 1 : 0;
  if (round_out) mode = 0;
  WXX_REQUIRE(bias_mode >= 0 && bias_mode <= 3, "wxx_matmul: bias_mode %d not in 0..3", bias_mode);
  WXX_REQUIRE(bias_mode == 0 || bias != nullptr, "wxx_matmul: bias_mode %d needs a bias", bias_mode);
  WXX_REQUIRE(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31),
              "wxx_matmul: dimension exceeds 2^31");
  if (batch * M * N == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  if (K == 0) {
    // Empty reduction: C = bias (or 0).
    WXX_CUDA_CHECK(cudaMemsetAsync(C, 0, batch * M * N * sizeof(float), s));
    if (bias_mode == 0) return WXX_OK;
    mode = 2;  // the SIMT kernel adds the bias to the zero product
  }
  // Row maxima instead of C (wxx_matmul_argmax) only from the SM-pair
  // kernel's epilogue; other shapes are the caller's to handle.
  if (amax_ws != nullptr && (K == 0 || mode == 2 || act != 0 || res != nullptr || bias_mode != 0)) {
    wxx::set_error("wxx_matmul: the row-maximum epilogue needs a plain tensor-core product");
    return WXX_E_UNSUPPORTED;
  }
  // A few rows against a K-major weight (generation's decode step): the
  // weight-streaming kernel.  Batches whose A rows are consecutive and share
  // the weight fold into rows.
  const int64_t rows_all = batch * M;
  if (amax_ws == nullptr && trans_a == 0 && trans_b != 0 && act <= 1 && bias_mode <= 1 &&
      (batch == 1 || (a_bs == M * lda && b_bs == 0)) &&
      gemv_fits(rows_all, N, K, lda, ldb, A, B)) {
    return launch_gemv(C, A, lda, B, ldb, bias_mode == 1 ? bias : nullptr, (int)rows_all, (int)N,
                       (int)K, alpha, act, res, round_out, nullptr, nullptr, 0.f);
  }
  // Skinny products with a long K (ResNet's 256 x 10 x 512 classifier: two
  // gathered tensor-core tiles walking 16 K-blocks) run one warp per output
  // row in exact fp32; the fused epilogues (act / residual) stay on the
  // tensor cores.
  if (amax_ws == nullptr && !round_out && act == 0 && res == nullptr && N <= kSkinnyN && K >= 256 &&
      batch * M * N * K <= (int64_t(1) << 24) && bias_mode <= 1) {
    const int64_t rows = batch * M;
    skinny_gemm_kernel<<<wxx::grid_for(rows * 32, 256), 256, 0, s>>>(
        C, A, B, bias, batch, (int)M, (int)N, (int)K, a_bs, b_bs, lda, ldb, trans_a, trans_b,
        bias_mode, alpha);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  if (mode == 2) {
    WXX_REQUIRE(batch <= 65535, "wxx_matmul: SIMT path supports batch <= 65535");
    dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64), (unsigned)batch);
    simt_gemm_kernel<<<grid, 256, 0, s>>>(C, A, B, bias, (int)M, (int)N, (int)K, a_bs, b_bs, lda,
                                         ldb, trans_a, trans_b, bias_mode, alpha);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)batch;
  p.num_kb = (int)((K + BK - 1) / BK);
  p.passes = mode == 1 ? 3 : 1;
  p.splits = 1;
  p.kb_per_split = p.num_kb * p.passes;
  p.err = wxx::device_error_word();
  int bn = pick_bn(M, N, batch);
  CUtensorMap ma0, ma1, mb0, mb1;
  memset(&ma0, 0, sizeof(ma0));
  memset(&mb0, 0, sizeof(mb0));
  // TMA wherever the operand is 16-byte addressable, gather producers
  // otherwise.  3xTF32 adds the residual operands (scratch, TMA-fed) or
  // splits gathered operands on the fly.
  OperandDesc da{A, M, K, batch, lda, a_bs, trans_a == 0, a_bs == 0 && batch > 1};
  OperandDesc db{B, N, K, batch, ldb, b_bs, trans_b != 0, b_bs == 0 && batch > 1};
  const int64_t n_out = act == 2 ? N / 2 : N;
  p.epi.kind = 0;
  p.epi.C = C;
  p.epi.c_bs = M * n_out;
  p.epi.ldc = (int)n_out;
  p.epi.bias = bias;
  p.epi.bias_mode = bias_mode;
  p.epi.bias_bs = M * N;
  p.epi.alpha = alpha;
  p.epi.act = act;
  p.epi.res = res;
  p.epi.res_ld = N;
  p.epi.res_bs = M * N;
  p.epi.round_tf32 = round_out;
  p.epi.amax = amax_ws;
  if (amax_ws != nullptr) p.epi.C = reinterpret_cast<float*>(amax_ws);  // map only: no stores
  // SM-pair tiles when the product is large and every operand is TMA-fed;
  // each CTA then loads 128-row boxes of both A and B.
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  int64_t pair_tiles = batch * ((M + 2 * BM - 1) / (2 * BM)) * ((N + 255) / 256);
  // 3xTF32 products longer than one accumulation chain go to split-K instead.
  const bool long_3x = p.passes > 1 && p.num_kb * p.passes > kMaxChainKb3x;
  bool pair = bn == 256 && pair_enabled() && !long_3x && pair_tiles >= wxx::num_sms() / 2 &&
              encode_c_map(&mc, p);
  setup_operand(da, BM, true, p.a, &ma0);
  setup_operand(db, pair ? BM : bn, true, p.b, &mb0);
  if (pair && (p.a.kind >= 2 || p.b.kind >= 2)) {
    pair = false;
    setup_operand(db, bn, true, p.b, &mb0);
  }
  if (amax_ws != nullptr && !pair) {
    wxx::set_error("wxx_matmul: the row-maximum epilogue needs the SM-pair kernel");
    return WXX_E_UNSUPPORTED;
  }
  const int b_box = pair ? BM : bn;
  ma1 = ma0;
  mb1 = mb0;
  void* lo_a = nullptr;
  void* lo_b = nullptr;
  if (mode == 1) {
    int st = make_residual(da, p.a, BM, &ma1, &lo_a);
    if (st == WXX_OK) st = make_residual(db, p.b, b_box, &mb1, &lo_b);
    if (st != WXX_OK) {
      wxx_free(lo_a);
      wxx_free(lo_b);
      return st;
    }
  }
  int st;
  if (pair) {
    st = launch_pair<256>(ma0, ma1, mb0, mb1, mc, p);
  } else if (act == 0 && res == nullptr && plan_splits(p, bn)) {
    st = run_splitk(bn, ma0, ma1, mb0, mb1, p);
  } else {
    st = run_tc(bn, ma0, ma1, mb0, mb1, p);
  }
  // Stream-ordered frees: the residuals stay valid for the GEMM just enqueued.
  int st_a = wxx_free(lo_a);
  int st_b = wxx_free(lo_b);
  return st ? st : (st_a ? st_a : st_b);
}

}  // namespace

namespace {

// The bounded mbarrier wait of the tensor-core kernels (mbar_wait, the same
// function) on a barrier whose only expected arrival is made when `arrive` is
// set.  Without it nothing arrives and the wait ends after limit_ns with the
// device error word set, as a stalled producer would leave a GEMM.
__global__ void wait_probe_kernel(int arrive, unsigned long long limit_ns, int* err,
                                  int* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && arrive) mbar_arrive(&bar);
  const bool ok = mbar_wait(&bar, 0, &abort_flag, err, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) *result = ok ? 1 : 0;
}

}  // namespace

// Self-test of the device-side failure path (no reference counterpart): one
// CTA waits on an mbarrier with the tensor-core kernels' bounded wait and a
// limit of limit_ns nanoseconds.  arrive = 1 completes the barrier (the wait
// succeeds, *result_dev = 1); arrive = 0 leaves it pending, so the wait gives
// up after the limit, *result_dev = 0 and wxx_device_status reports
// WXX_DEV_ERR_MBAR_TIMEOUT (1) -- the context stays usable.  limit_ns in
// (0, 10 s].  result_dev: one device int.
WXX_EXPORT int wxx_wait_probe(int arrive, int64_t limit_ns, int* result_dev) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(limit_ns > 0 && limit_ns <= 10000000000ll,
              "wxx_wait_probe: limit %lld ns outside (0, 10 s]", (long long)limit_ns);
  WXX_REQUIRE(result_dev != nullptr, "wxx_wait_probe: result pointer is NULL");
  wait_probe_kernel<<<1, 32, 0, wxx::stream()>>>(arrive ? 1 : 0, (unsigned long long)limit_ns,
                                                 wxx::device_error_word(), result_dev);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

WXX_EXPORT int wxx_matmul(float* C, const float* A, const float* B, const float* bias,
                          int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_bs,
                          int64_t b_bs, int64_t lda, int64_t ldb, int trans_a, int trans_b,
                          int bias_mode, float alpha, int mode) {
  WXX_REQUIRE_INIT();
  return matmul_impl(C, A, B, bias, batch, M, N, K, a_bs, b_bs, lda, ldb, trans_a, trans_b,
                     bias_mode, alpha, mode, 0, nullptr);
}

// Batched form of wxx_linear for an A operand given as a strided view:
//   C[b] (M, N dense) = act(alpha * op(A[b]) @ op(B) + bias) + residual[b]
// A[b] at A + b*a_bs with row stride lda, op(A) = A or A^T (trans_a: A[b] is
// stored (K, M) -- a (B, K, M) activation read as (B, M, K) without a copy);
// B (K, N) or (N, K) with trans_b, shared by the batch; residual (batch, M,
// N) dense or NULL.  Same requirements as wxx_linear.
WXX_EXPORT int wxx_linear_batched(float* C, const float* A, const float* B, const float* bias,
                                  const float* residual, int64_t batch, int64_t M, int64_t N,
                                  int64_t K, int64_t a_bs, int64_t lda, int trans_a, int64_t ldb,
                                  int trans_b, int act, float alpha, int mode) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(batch >= 1 && M >= 0 && N >= 0 && K > 0, "wxx_linear_batched: bad sizes");
  WXX_REQUIRE(mode == 0 || mode == 1 || mode == 3,
              "wxx_linear_batched: mode %d not in {0, 1, 3}", mode);
  WXX_REQUIRE(act == 0 || act == 1, "wxx_linear_batched: act %d not in {0, 1}", act);
  WXX_REQUIRE(!(reinterpret_cast<uintptr_t>(C) & 15) && N % 4 == 0,
              "wxx_linear_batched: C must be 16-byte aligned with N a multiple of 4");
  if (batch * M * N == 0) return WXX_OK;
  return matmul_impl(C, A, B, bias, batch, M, N, K, a_bs, 0, lda, ldb, trans_a, trans_b,
                     bias ? 1 : 0, alpha, mode, act, residual);
}

// Linear layer with its follow-up fused into the GEMM epilogue:
//   C (M, N dense) = act(alpha * A @ op(B) + bias) + residual
// A (M, K) row stride lda; B (K, N) row stride ldb, or (N, K) with trans_b = 1;
// bias (N) or NULL; residual (M, N dense) or NULL; act 0 none, 1 GELU (tanh),
// 2 paired GLU: product columns 2j, 2j+1 are (gate, up) of output column j,
// C (M, N/2) = silu(gate) * up (no residual; N a multiple of 8).
// mode 0 TF32, 1 3xTF32, 3 TF32 with C rounded to the nearest TF32 value
// (for outputs read only by TF32 products).  C must be 16-byte aligned and N
// a multiple of 4.
WXX_EXPORT int wxx_linear(float* C, const float* A, const float* B, const float* bias,
                          const float* residual, int64_t M, int64_t N, int64_t K, int64_t lda,
                          int64_t ldb, int trans_b, int act, float alpha, int mode) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(M >= 0 && N >= 0 && K > 0, "wxx_linear: bad sizes (K must be positive)");
  WXX_REQUIRE(mode == 0 || mode == 1 || mode == 3, "wxx_linear: mode %d not in {0, 1, 3}", mode);
  WXX_REQUIRE(act >= 0 && act <= 2, "wxx_linear: act %d not in {0, 1, 2}", act);
  WXX_REQUIRE(act != 2 || (residual == nullptr && N % 8 == 0),
              "wxx_linear: the paired GLU takes no residual and needs N a multiple of 8");
  WXX_REQUIRE(!(reinterpret_cast<uintptr_t>(C) & 15) && N % 4 == 0,
              "wxx_linear: C must be 16-byte aligned with N a multiple of 4");
  if (M * N == 0) return WXX_OK;
  return matmul_impl(C, A, B, bias, 1, M, N, K, 0, 0, lda, ldb, 0, trans_b, bias ? 1 : 0, alpha,
                     mode, act, residual);
}

namespace {

// Per row: the tiles' (maximum, column within the tile) pairs merged in tile
// order -- larger value wins, equal values go to the smaller amax_key of the
// column within the tile (= the index mod 256 for 256-wide tiles), then to
// the earlier tile -- the argmax kernels' choice among the positions holding
// the row maximum.  A row with no value above -1e38 gets index 0.
__global__ void amax_merge_kernel(uint32_t* __restrict__ idx, float* __restrict__ vals,
                                  const float2* __restrict__ ws, int64_t rows, int tiles) {
  // one warp per row: the lanes read the row's tile entries 32 at a time
  // (coalesced) and the candidates are reduced by shuffles; the order
  // (value, then smaller key, then earlier tile) is total, so the reduction
  // order does not matter
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const float2* w = ws + r * tiles;
    bool ok = false;
    float bv = -1e38f;
    int bk = 0, bt = 0, bc = 0;
    for (int t = lane; t < tiles; t += 32) {
      const float2 e = w[t];
      if (e.x > -1e38f) {
        const int c = __float_as_int(e.y), k = amax_key(c);
        if (!ok || e.x > bv || (e.x == bv && (k < bk || (k == bk && t < bt)))) {
          ok = true;
          bv = e.x;
          bk = k;
          bt = t;
          bc = c;
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const bool ook = __shfl_xor_sync(0xffffffffu, ok ? 1 : 0, off) != 0;
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int ok_ = __shfl_xor_sync(0xffffffffu, bk, off);
      const int ot = __shfl_xor_sync(0xffffffffu, bt, off);
      const int oc = __shfl_xor_sync(0xffffffffu, bc, off);
      if (ook && (!ok || ov > bv || (ov == bv && (ok_ < bk || (ok_ == bk && ot < bt))))) {
        ok = true;
        bv = ov;
        bk = ok_;
        bt = ot;
        bc = oc;
      }
    }
    if (lane == 0) {
      idx[r] = ok ? (uint32_t)(bt * 256 + bc) : 0u;
      if (vals != nullptr) vals[r] = ok ? bv : -1e38f;
    }
  }
}

}  // namespace

// Row-wise argmax of a product without storing it (the GPT2 forward whose
// output is the next-token id of every position): idx[b*M + m] = argmax over n
// of (op(A[b]) @ op(B))[m, n], vals (or NULL) the maxima; the index rule of
// wxx_argminmax (op 0).  Arguments as wxx_matmul (no bias, alpha 1).  The
// SM-pair GEMM's epilogue keeps each row's maximum per 256-column tile and a
// small kernel merges the tiles.  Products that kernel does not take (too
// few tiles, operands TMA cannot address, fp32 SIMT mode, K = 0) return
// WXX_E_UNSUPPORTED with nothing enqueued: store the product and run
// wxx_argminmax instead.
WXX_EXPORT int wxx_matmul_argmax(uint32_t* idx, float* vals, const float* A, const float* B,
                                 int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_bs,
                                 int64_t b_bs, int64_t lda, int64_t ldb, int trans_a, int trans_b,
                                 int mode) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(batch >= 0 && M >= 0 && N > 0 && K >= 0, "wxx_matmul_argmax: bad sizes");
  WXX_REQUIRE(idx != nullptr, "wxx_matmul_argmax: idx is NULL");
  WXX_REQUIRE(mode >= 0 && mode <= 2, "wxx_matmul_argmax: mode %d not in 0..2", mode);
  const int64_t rows = batch * M;
  if (rows == 0) return WXX_OK;
  const int64_t tiles = (N + 255) / 256;
  void* ws = nullptr;
  int st = wxx_malloc(&ws, (uint64_t)rows * tiles * sizeof(float2));
  if (st) return st;
  st = K > 0 ? matmul_impl(nullptr, A, B, nullptr, batch, M, N, K, a_bs, b_bs, lda, ldb, trans_a,
                           trans_b, 0, 1.0f, mode, 0, nullptr, reinterpret_cast<float2*>(ws))
             : WXX_E_UNSUPPORTED;
  if (st == WXX_OK) {
    amax_merge_kernel<<<wxx::grid_for(rows * 32, 256), 256, 0, wxx::stream()>>>(
        idx, vals, reinterpret_cast<const float2*>(ws), rows, (int)tiles);
    st = wxx::after_launch(__FILE__, __LINE__);
  }
  const int st2 = wxx_free(ws);
  return st ? st : st2;
}

// A few rows through LayerNorm and a linear layer in one launch (the decode
// step's ln -> q/k/v, ln2 -> fc1 and ln_f -> LM head):
//   C (M, N dense) = act(LayerNorm(A) @ W^T + bias) + residual
// LayerNorm over A's K entries per row (row stride lda) with gamma / beta (K)
// and eps; W (N, K) K-major (row stride ldw); bias (N) or NULL; residual
// (M, N) or NULL; act 0 or 1 (GELU); round_out = 1 stores C rounded to the
// nearest TF32 value.  Exact fp32.  Returns WXX_E_UNSUPPORTED (nothing
// enqueued) unless 1 <= M <= 32, N >= 64, K >= 128 with K, lda, ldw multiples
// of 4 and A, W, gamma, beta 16-byte aligned.
WXX_EXPORT int wxx_ln_linear(float* C, const float* A, int64_t lda, const float* gamma,
                             const float* beta, float eps, const float* W, int64_t ldw,
                             const float* bias, const float* residual, int64_t M, int64_t N,
                             int64_t K, int act, int round_out) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(gamma != nullptr && beta != nullptr && act >= 0 && act <= 1,
              "wxx_ln_linear: gamma / beta missing or act %d not in {0, 1}", act);
  if (!gemv_fits(M, N, K, lda, ldw, A, W) || (reinterpret_cast<uintptr_t>(gamma) & 15) ||
      (reinterpret_cast<uintptr_t>(beta) & 15)) {
    wxx::set_error("wxx_ln_linear: shape or alignment outside the few-rows kernel");
    return WXX_E_UNSUPPORTED;
  }
  return launch_gemv(C, A, lda, W, ldw, bias, (int)M, (int)N, (int)K, 1.0f, act, residual,
                     round_out ? 1 : 0, gamma, beta, eps);
}

// Linear projection followed by a depthwise short causal convolution along
// the sequence, written channels-first: Hyena's projection, transpose and
// short conv (hyena.py: proj_v / proj_x, transpose(1, 2), short_conv) in one
// tcgen05 GEMM whose epilogue applies the taps.
//   Y (M, N) = alpha * A @ op(B) + bias, row = b * seq_len + n
//   out[b, c, n] (M / seq_len, N, seq_len dense) = conv_b[c']
//       + sum over k < conv_k with k <= n of conv_w[c', k] * Y[row - k, c],  c' = c % conv_ch
// A (M, K) with row stride lda, B (K, N) row stride ldb or (N, K) with
// trans_b, bias (N) or NULL, conv_w (conv_ch, conv_k), conv_b (conv_ch);
// conv_k in 1..4; mode 0 TF32, 1 3xTF32 (K <= 1024).  Returns
// WXX_E_UNSUPPORTED (nothing enqueued) when A or B is not TMA-addressable.
WXX_EXPORT int wxx_linear_short_conv(float* out, const float* A, const float* B, const float* bias,
                                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                     int trans_b, int64_t seq_len, const float* conv_w,
                                     const float* conv_b, int conv_ch, int conv_k, int mode) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(M >= 0 && N >= 0 && K > 0 && seq_len > 0,
              "wxx_linear_short_conv: bad sizes (K and seq_len must be positive)");
  WXX_REQUIRE(M % seq_len == 0, "wxx_linear_short_conv: M = %lld is not a multiple of seq_len %lld",
              (long long)M, (long long)seq_len);
  WXX_REQUIRE(conv_k >= 1 && conv_k <= 4, "wxx_linear_short_conv: conv_k %d not in 1..4", conv_k);
  WXX_REQUIRE(conv_ch >= 1 && conv_w != nullptr && conv_b != nullptr,
              "wxx_linear_short_conv: conv weights missing");
  WXX_REQUIRE(mode == 0 || mode == 1, "wxx_linear_short_conv: mode %d not in {0, 1}", mode);
  WXX_REQUIRE(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31),
              "wxx_linear_short_conv: dimension exceeds 2^31");
  if (M * N == 0) return WXX_OK;
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = 1;
  p.num_kb = (int)((K + BK - 1) / BK);
  p.passes = mode == 1 ? 3 : 1;
  p.splits = 1;
  p.kb_per_split = p.num_kb * p.passes;
  p.err = wxx::device_error_word();
  if (p.passes > 1 && p.num_kb * p.passes > kMaxChainKb3x) {
    wxx::set_error("wxx_linear_short_conv: 3xTF32 with K = %lld > 1024 is not fused",
                   (long long)K);
    return WXX_E_UNSUPPORTED;
  }
  p.epi.kind = 2;
  p.epi.C = out;
  p.epi.c_bs = N * seq_len;
  p.epi.ldc = (int)N;
  p.epi.bias = bias;
  p.epi.bias_mode = bias ? 1 : 0;
  p.epi.alpha = 1.0f;
  p.epi.conv_len = (int)seq_len;
  p.epi.conv_k = conv_k;
  p.epi.conv_ch = conv_ch;
  p.epi.conv_w = conv_w;
  p.epi.conv_b = conv_b;
  CUtensorMap ma0, ma1, mb0, mb1, mc;
  memset(&ma0, 0, sizeof(ma0));
  memset(&mb0, 0, sizeof(mb0));
  memset(&mc, 0, sizeof(mc));
  OperandDesc da{A, M, K, 1, lda, 0, true, false};
  OperandDesc db{B, N, K, 1, ldb, 0, trans_b != 0, false};
  setup_operand(da, 32, true, p.a, &ma0);   // 32-row boxes, one per epilogue warp
  setup_operand(db, BM, true, p.b, &mb0);
  if (p.a.kind != 0 || p.b.kind >= 2) {
    wxx::set_error("wxx_linear_short_conv: operands are not TMA-addressable (16-byte aligned "
                   "rows needed)");
    return WXX_E_UNSUPPORTED;
  }
  ma1 = ma0;
  mb1 = mb0;
  void* lo_a = nullptr;
  void* lo_b = nullptr;
  if (mode == 1) {
    int st = make_residual(da, p.a, 32, &ma1, &lo_a);
    if (st == WXX_OK) st = make_residual(db, p.b, BM, &mb1, &lo_b);
    if (st != WXX_OK) {
      wxx_free(lo_a);
      wxx_free(lo_b);
      return st;
    }
  }
  int st = launch_pair<256>(ma0, ma1, mb0, mb1, mc, p);
  int st_a = wxx_free(lo_a);
  int st_b = wxx_free(lo_b);
  return st ? st : (st_a ? st_a : st_b);
}

// Y (NCHW [B, Cout, Ho, Wo]) = conv2d(X [B, Cin, H, W], Wt [Cout, Cin, KH, KW]) (+ bias[Cout])
// with stride (sh, sw), padding (ph, pw), dilation (dh, dw);
// Ho = (H + 2ph - dh(KH-1) - 1)/sh + 1.  mode: 0 TF32, 1 3xTF32, 2 fp32 (3xTF32 path).
namespace {
int conv2d_impl(float* Y, const float* X, const float* Wt, const float* bias, int B, int Cin, int H,
                int W, int Cout, int KH, int KW, int sh, int sw, int ph, int pw, int dh, int dw,
                int mode, const ConvPost& post);

// W (Cout, Cin, KH*KW) -> Wr (Cout, KH*KW, Cin): the NHWC convolution's K order.
// One CTA per output channel transposes its (Cin x taps) block through shared
// memory, so both the reads and the writes are contiguous.
__global__ void __launch_bounds__(256) conv_weight_reorder_kernel(float* __restrict__ wr,
                                                                  const float* __restrict__ w,
                                                                  int cout, int cin, int taps) {
  extern __shared__ float blk[];   // cin * taps
  const int n = cin * taps;
  for (int o = blockIdx.x; o < cout; o += gridDim.x) {
    const float* src = w + (int64_t)o * n;
    float* dst = wr + (int64_t)o * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) blk[i] = src[i];
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int t = i / cin, c = i - t * cin;
      dst[i] = blk[c * taps + t];
    }
    __syncthreads();
  }
}

// The same reorder for up to kPackMax filters in one launch (blockIdx.y =
// filter): a network's convolutions pack their weights together instead of
// each paying a small launch of its own.
constexpr int kPackMax = 24;
struct PackArgs {
  float* dst[kPackMax];
  const float* src[kPackMax];
  int cout[kPackMax], cin[kPackMax], taps[kPackMax];
};

__global__ void __launch_bounds__(256) conv_weight_pack_kernel(PackArgs a) {
  extern __shared__ float blk[];
  const int f = blockIdx.y;
  const int cin = a.cin[f], taps = a.taps[f], n = cin * taps;
  for (int o = blockIdx.x; o < a.cout[f]; o += gridDim.x) {
    const float* src = a.src[f] + (int64_t)o * n;
    float* dst = a.dst[f] + (int64_t)o * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) blk[i] = src[i];
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int t = i / cin, c = i - t * cin;
      dst[i] = blk[c * taps + t];
    }
    __syncthreads();
  }
}

// 128-pixel output tiles as one TMA box (W, H, images) of output positions;
// false when the output geometry does not split that way.
bool nhwc_box(int Ho, int Wo, int* bw, int* bh, int* bb) {
  if (Wo >= BM) {
    if (Wo % BM) return false;
    *bw = BM; *bh = 1; *bb = 1;
    return true;
  }
  if (BM % Wo) return false;
  const int rows = BM / Wo;
  *bw = Wo;
  if (Ho >= rows) {
    if (Ho % rows) return false;
    *bh = rows; *bb = 1;
    return true;
  }
  if (rows % Ho) return false;
  *bh = Ho; *bb = rows / Ho;
  return true;
}

// 4-D map of an NHWC tensor (C, W, H, B) for the conv operand: boxes of 32
// channels x bw x bh x bb positions, W and H traversed with the conv stride.
bool encode_nhwc_map(CUtensorMap* map, const float* base, int C, int W, int H, int B, int bw,
                     int bh, int bb, int sw, int sh) {
  auto enc = get_encode();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || C % 32) return false;
  cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)C * 4, (cuuint64_t)W * C * 4, (cuuint64_t)H * W * C * 4};
  cuuint32_t box[4] = {32, (cuuint32_t)(bw * sw), (cuuint32_t)(bh * sh), (cuuint32_t)bb};
  cuuint32_t estr[4] = {1, (cuuint32_t)sw, (cuuint32_t)sh, 1};
  if (box[1] > 256 || box[2] > 256 || box[3] > 256 || sw > 8 || sh > 8) return false;
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

// NHWC convolution with the same follow-up ops as wxx_conv2d_bn:
//   Y (B, Ho, Wo, Cout) = relu?(bn(conv(X) + bias) + residual)
// X (B, H, W, Cin) NHWC, W (Cout, Cin, KH, KW) as in the reference, residual
// NHWC like Y or NULL.  An implicit GEMM whose A operand is fetched by TMA:
// each K-block is 32 channels of one filter tap and each 128-row tile one 4-D
// box of X (padding read as zeros, the stride as the box's traversal
// stride), so nothing is gathered by threads.  Requires Cin % 32 == 0,
// Cout % 4 == 0, 16-byte aligned X and Y, and an output geometry whose
// 128-pixel tiles are boxes (Wo a multiple of 128, or Wo dividing 128 and Ho
// a multiple or a divisor of 128 / Wo); else WXX_E_ARG.
namespace {
int conv2d_nhwc_impl(float* Y, const float* X, const float* Wt, bool packed, const float* bias,
                     int B, int Cin, int H, int W, int Cout, int KH, int KW, int sh, int sw,
                     int ph, int pw, int dh, int dw, int mode, const float* rm, const float* rv,
                     const float* gamma, const float* beta, float eps, const float* residual,
                     int relu) {
  WXX_REQUIRE(B >= 0 && Cin > 0 && H > 0 && W > 0 && Cout > 0 && KH > 0 && KW > 0,
              "wxx_conv2d_nhwc: bad sizes");
  WXX_REQUIRE(sh > 0 && sw > 0 && dh > 0 && dw > 0 && ph >= 0 && pw >= 0,
              "wxx_conv2d_nhwc: bad stride/padding/dilation");
  WXX_REQUIRE(rm == nullptr || (rv && gamma && beta),
              "wxx_conv2d_nhwc: batchnorm needs mean, variance, gamma and beta");
  const int Ho = (H + 2 * ph - dh * (KH - 1) - 1) / sh + 1;
  const int Wo = (W + 2 * pw - dw * (KW - 1) - 1) / sw + 1;
  WXX_REQUIRE(Ho > 0 && Wo > 0, "wxx_conv2d_nhwc: empty output");
  int bw = 0, bh = 0, bb = 0;
  WXX_REQUIRE(Cin % 32 == 0 && Cout % 4 == 0 && nhwc_box(Ho, Wo, &bw, &bh, &bb) &&
                  !(reinterpret_cast<uintptr_t>(X) & 15) && !(reinterpret_cast<uintptr_t>(Y) & 15),
              "wxx_conv2d_nhwc: unsupported geometry (Cin %% 32, Cout %% 4, 128-pixel boxes, "
              "alignment)");
  const int64_t Mrows = (int64_t)B * Ho * Wo;
  const int64_t K = (int64_t)Cin * KH * KW;
  WXX_REQUIRE(Mrows < (int64_t(1) << 31) && K < (int64_t(1) << 31), "wxx_conv2d_nhwc: too large");
  if (Mrows == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = (int)Mrows;
  p.N = Cout;
  p.K = (int)K;
  p.batch = 1;
  p.num_kb = (int)(K / BK);
  p.passes = mode == 0 ? 1 : 3;
  p.splits = 1;
  p.kb_per_split = p.num_kb * p.passes;
  p.err = wxx::device_error_word();
  const int bn = pick_bn(Mrows, Cout, 1);
  // B: the weights reordered to (Cout, tap, Cin), K-major
  void* wr = nullptr;
  void* lo_x = nullptr;
  void* lo_w = nullptr;
  int st = WXX_OK;
  if (packed) {
    wr = const_cast<float*>(Wt);   // already (Cout, tap, Cin); not freed below
  } else {
    st = wxx_malloc(&wr, (uint64_t)Cout * K * sizeof(float));
    if (st) return st;
  }
  if (!packed) {
    const size_t smem = (size_t)K * sizeof(float);
    static size_t smem_set = 48 * 1024;
    if (smem > smem_set) {
      WXX_CUDA_CHECK(cudaFuncSetAttribute(conv_weight_reorder_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
      smem_set = smem;
    }
    WXX_REQUIRE(smem <= 200 * 1024, "wxx_conv2d_nhwc: filter too large (Cin*KH*KW)");
    conv_weight_reorder_kernel<<<Cout < 1184 ? Cout : 1184, 256, smem, s>>>((float*)wr, Wt, Cout,
                                                                           Cin, KH * KW);
    st = wxx::after_launch(__FILE__, __LINE__);
    if (st != WXX_OK) {
      wxx_free(wr);
      return st;
    }
  }
  CUtensorMap ma0, ma1, mb0, mb1;
  memset(&ma0, 0, sizeof(ma0));
  memset(&mb0, 0, sizeof(mb0));
  OperandDesc db{(const float*)wr, Cout, K, 1, K, 0, true, false};
  setup_operand(db, bn, true, p.b, &mb0);
  // A: the NHWC input through 4-D boxes
  memset(&p.a, 0, sizeof(p.a));
  p.a.kind = 4;
  p.a.cin = Cin; p.a.h = H; p.a.w = W; p.a.kh = KH; p.a.kw = KW;
  p.a.sh = sh; p.a.sw = sw; p.a.ph = ph; p.a.pw = pw; p.a.dh = dh; p.a.dw = dw;
  p.a.ho = Ho; p.a.wo = Wo;
  bool ok = p.b.kind == 0 && encode_nhwc_map(&ma0, X, Cin, W, H, B, bw, bh, bb, sw, sh);
  ma1 = ma0;
  mb1 = mb0;
  if (ok && mode != 0) {
    // 3xTF32: the low parts of both operands, precomputed
    const int64_t nx = (int64_t)B * H * W * Cin;
    st = wxx_malloc(&lo_x, (uint64_t)nx * sizeof(float));
    if (st == WXX_OK) {
      tf32_residual_kernel<<<wxx::grid_for(nx / 4 + 1, 256), 256, 0, s>>>((float*)lo_x, X, nx);
      st = wxx::after_launch(__FILE__, __LINE__);
      ok = encode_nhwc_map(&ma1, (const float*)lo_x, Cin, W, H, B, bw, bh, bb, sw, sh);
      if (ok) st = make_residual(db, p.b, bn, &mb1, &lo_w);
    }
  }
  if (st == WXX_OK && !ok) {
    wxx::set_error("wxx_conv2d_nhwc: tensor maps could not be encoded");
    st = WXX_E_ARG;
  }
  if (st == WXX_OK) {
    p.epi.kind = 0;
    p.epi.C = Y;
    p.epi.ldc = Cout;
    p.epi.c_bs = Mrows * Cout;
    p.epi.bias = bias;
    p.epi.bias_mode = bias ? 1 : 0;
    p.epi.alpha = 1.0f;
    p.epi.res = residual;
    p.epi.res_ld = Cout;
    p.epi.res_bs = Mrows * Cout;
    p.epi.post.rm = rm;
    p.epi.post.rv = rv;
    p.epi.post.g = gamma;
    p.epi.post.b = beta;
    p.epi.post.eps = eps;
    p.epi.post.res = residual;   // read by the split-K reduce
    p.epi.post.relu = relu ? 1 : 0;
    st = plan_splits(p, bn) ? run_splitk(bn, ma0, ma1, mb0, mb1, p)
                            : run_tc(bn, ma0, ma1, mb0, mb1, p);
  }
  // stream-ordered frees: valid for the kernels just enqueued
  const int s1 = packed ? WXX_OK : wxx_free(wr), s2 = wxx_free(lo_x), s3 = wxx_free(lo_w);
  return st ? st : (s1 ? s1 : (s2 ? s2 : s3));
}
}  // namespace

WXX_EXPORT int wxx_conv2d_nhwc(float* Y, const float* X, const float* Wt, const float* bias, int B,
                               int Cin, int H, int W, int Cout, int KH, int KW, int sh, int sw,
                               int ph, int pw, int dh, int dw, int mode, const float* rm,
                               const float* rv, const float* gamma, const float* beta, float eps,
                               const float* residual, int relu) {
  WXX_REQUIRE_INIT();
  return conv2d_nhwc_impl(Y, X, Wt, false, bias, B, Cin, H, W, Cout, KH, KW, sh, sw, ph, pw, dh,
                          dw, mode, rm, rv, gamma, beta, eps, residual, relu);
}

// wxx_conv2d_nhwc with the weights already in the NHWC convolution's K order,
// Wp (Cout, KH*KW, Cin) as written by wxx_conv_weight_pack: no reorder launch
// and no scratch for it.
WXX_EXPORT int wxx_conv2d_nhwc_packed(float* Y, const float* X, const float* Wp, const float* bias,
                                      int B, int Cin, int H, int W, int Cout, int KH, int KW,
                                      int sh, int sw, int ph, int pw, int dh, int dw, int mode,
                                      const float* rm, const float* rv, const float* gamma,
                                      const float* beta, float eps, const float* residual,
                                      int relu) {
  WXX_REQUIRE_INIT();
  return conv2d_nhwc_impl(Y, X, Wp, true, bias, B, Cin, H, W, Cout, KH, KW, sh, sw, ph, pw, dh,
                          dw, mode, rm, rv, gamma, beta, eps, residual, relu);
}

// Reorders n <= 24 convolution weights W_i (cout[i], cin[i], taps[i]) to
// (cout[i], taps[i], cin[i]) in one launch; dst/src are host arrays of device
// pointers; cin[i] * taps[i] <= 51200.
WXX_EXPORT int wxx_conv_weight_pack(float* const* dst, const float* const* src, const int* cout,
                                    const int* cin, const int* taps, int n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n >= 0 && n <= kPackMax && (n == 0 || (dst && src && cout && cin && taps)),
              "wxx_conv_weight_pack: n %d not in 0..%d or NULL arrays", n, kPackMax);
  if (n == 0) return WXX_OK;
  PackArgs a;
  memset(&a, 0, sizeof(a));
  int max_n = 1, max_cout = 1;
  for (int i = 0; i < n; ++i) {
    WXX_REQUIRE(dst[i] && src[i] && cout[i] >= 0 && cin[i] > 0 && taps[i] > 0 &&
                    (int64_t)cin[i] * taps[i] <= 51200,
                "wxx_conv_weight_pack: filter %d has bad sizes", i);
    a.dst[i] = dst[i];
    a.src[i] = src[i];
    a.cout[i] = cout[i];
    a.cin[i] = cin[i];
    a.taps[i] = taps[i];
    if (cin[i] * taps[i] > max_n) max_n = cin[i] * taps[i];
    if (cout[i] > max_cout) max_cout = cout[i];
  }
  const size_t smem = (size_t)max_n * sizeof(float);
  static size_t smem_set = 48 * 1024;
  if (smem > smem_set) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(conv_weight_pack_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set = smem;
  }
  dim3 grid((unsigned)(max_cout < 512 ? max_cout : 512), (unsigned)n);
  conv_weight_pack_kernel<<<grid, 256, smem, wxx::stream()>>>(a);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

WXX_EXPORT int wxx_conv2d(float* Y, const float* X, const float* Wt, const float* bias, int B,
                          int Cin, int H, int W, int Cout, int KH, int KW, int sh, int sw, int ph,
                          int pw, int dh, int dw, int mode) {
  ConvPost post;
  memset(&post, 0, sizeof(post));
  return conv2d_impl(Y, X, Wt, bias, B, Cin, H, W, Cout, KH, KW, sh, sw, ph, pw, dh, dw, mode,
                     post);
}

// wxx_conv2d with ResNet's follow-up ops in the epilogue (or the split-K
// reduce): y = relu?(bn(conv(x) + bias) + residual) where bn is eval-mode
// batchnorm with running mean / variance rm, rv and affine gamma, beta
// (NULL rm: none; the batchnorm kernel's expression), residual NCHW like Y
// or NULL, relu 0/1.  Values equal the separate conv2d / batchnorm / add /
// relu kernels' (same fp32 operations in the same order).
WXX_EXPORT int wxx_conv2d_bn(float* Y, const float* X, const float* Wt, const float* bias, int B,
                             int Cin, int H, int W, int Cout, int KH, int KW, int sh, int sw,
                             int ph, int pw, int dh, int dw, int mode, const float* rm,
                             const float* rv, const float* gamma, const float* beta, float eps,
                             const float* residual, int relu) {
  WXX_REQUIRE(rm == nullptr || (rv && gamma && beta),
              "wxx_conv2d_bn: batchnorm needs mean, variance, gamma and beta");
  ConvPost post;
  post.rm = rm;
  post.rv = rv;
  post.g = gamma;
  post.b = beta;
  post.eps = eps;
  post.res = residual;
  post.relu = relu ? 1 : 0;
  return conv2d_impl(Y, X, Wt, bias, B, Cin, H, W, Cout, KH, KW, sh, sw, ph, pw, dh, dw, mode,
                     post);
}

namespace {
// Direct convolution for inputs with few channels (ResNet's 3-channel stem,
// K = 147): an implicit GEMM would gather 147-wide rows for little tensor
// work.  One CTA per (image, group of 16 output channels) holds the
// zero-padded image and the group's filters in shared memory; each thread
// accumulates 16 channels of its output pixels in exact fp32 (taps in the
// reference's (c, kh, kw) order) and applies bias and the post-ops.
constexpr int kDirectCG = 16;

template <int KWT>   // filter width (0: any, read from kw_rt)
__global__ void __launch_bounds__(256) conv_direct_kernel(
    float* __restrict__ Y, const float* __restrict__ X, const float* __restrict__ Wt,
    const float* __restrict__ bias, int Cin, int H, int W, int Cout, int KH, int kw_rt, int sh,
    int sw, int ph, int pw, int dh, int dw, int Ho, int Wo, ConvPost post) {
  const int KW = KWT > 0 ? KWT : kw_rt;
  extern __shared__ float dsm[];
  const int Hp = H + 2 * ph, Wp = W + 2 * pw;
  float* img = dsm;                              // Cin x Hp x Wp
  // taps x kDirectCG (channel fastest), read as float4: the image size is
  // rounded up to 4 floats so the weights start 16-byte aligned
  float* wts = dsm + ((Cin * Hp * Wp + 3) & ~3);
  const int groups = (Cout + kDirectCG - 1) / kDirectCG;
  const int b = blockIdx.x / groups, n0 = (blockIdx.x - b * groups) * kDirectCG;
  const int taps = Cin * KH * KW;
  const float* xb = X + (int64_t)b * Cin * H * W;
  // padded image: one padded row per iteration, no divisions per element
  for (int r = threadIdx.x >> 5; r < Cin * Hp; r += blockDim.x >> 5) {
    const int c = r / Hp, y = r - c * Hp - ph;
    float* dst = img + r * Wp;
    const bool rowin = y >= 0 && y < H;
    const float* src = xb + ((int64_t)c * H + y) * W;
    for (int x = (threadIdx.x & 31); x < Wp; x += 32) {
      const int xs = x - pw;
      dst[x] = (rowin && xs >= 0 && xs < W) ? src[xs] : 0.f;
    }
  }
  for (int i = threadIdx.x; i < taps * kDirectCG; i += blockDim.x) {
    const int t = i >> 4, j = i & (kDirectCG - 1);
    wts[i] = n0 + j < Cout ? Wt[(int64_t)(n0 + j) * taps + t] : 0.f;
  }
  __syncthreads();
  // two output pixels per thread (pix and pix + half): every weight load
  // feeds 32 FMAs
  const int hw = Ho * Wo, half = (hw + 1) / 2;
  for (int pix = threadIdx.x; pix < half; pix += blockDim.x) {
    const int pix2 = pix + half;
    const bool two = pix2 < hw;
    const int ho = pix / Wo, wo = pix - ho * Wo;
    const int ho2 = two ? pix2 / Wo : ho, wo2 = two ? pix2 - ho2 * Wo : wo;
    float acc[kDirectCG], acc2[kDirectCG];
#pragma unroll
    for (int j = 0; j < kDirectCG; ++j) acc[j] = acc2[j] = 0.f;
    const float4* wv = reinterpret_cast<const float4*>(wts);
    for (int c = 0; c < Cin; ++c) {
      for (int kh = 0; kh < KH; ++kh) {
        const float* row = img + (c * Hp + ho * sh + kh * dh) * Wp + wo * sw;
        const float* row2 = img + (c * Hp + ho2 * sh + kh * dh) * Wp + wo2 * sw;
#pragma unroll
        for (int kw = 0; kw < (KWT > 0 ? KWT : 1); ++kw) {
          for (int kk = 0; kk < (KWT > 0 ? 1 : KW); ++kk) {
            const int k = KWT > 0 ? kw : kk;
            const float xv = row[k * dw], xv2 = row2[k * dw];
#pragma unroll
            for (int q = 0; q < kDirectCG / 4; ++q) {
              const float4 w4 = wv[q];
              acc[4 * q] = fmaf(xv, w4.x, acc[4 * q]);
              acc[4 * q + 1] = fmaf(xv, w4.y, acc[4 * q + 1]);
              acc[4 * q + 2] = fmaf(xv, w4.z, acc[4 * q + 2]);
              acc[4 * q + 3] = fmaf(xv, w4.w, acc[4 * q + 3]);
              acc2[4 * q] = fmaf(xv2, w4.x, acc2[4 * q]);
              acc2[4 * q + 1] = fmaf(xv2, w4.y, acc2[4 * q + 1]);
              acc2[4 * q + 2] = fmaf(xv2, w4.z, acc2[4 * q + 2]);
              acc2[4 * q + 3] = fmaf(xv2, w4.w, acc2[4 * q + 3]);
            }
            wv += kDirectCG / 4;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kDirectCG; ++j) {
      const int n = n0 + j;
      if (n < Cout) {
        const float bv = bias != nullptr ? bias[n] : 0.f;
        const int64_t base = ((int64_t)b * Cout + n) * hw;
        float o = acc[j];
        if (bias != nullptr) o += bv;
        Y[base + pix] = conv_post(post, o, n, base + pix);
        if (two) {
          float o2 = acc2[j];
          if (bias != nullptr) o2 += bv;
          Y[base + pix2] = conv_post(post, o2, n, base + pix2);
        }
      }
    }
  }
}

int conv2d_impl(float* Y, const float* X, const float* Wt, const float* bias, int B, int Cin, int H,
                int W, int Cout, int KH, int KW, int sh, int sw, int ph, int pw, int dh, int dw,
                int mode, const ConvPost& post) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B >= 0 && Cin > 0 && H > 0 && W > 0 && Cout > 0 && KH > 0 && KW > 0,
              "wxx_conv2d: bad sizes");
  WXX_REQUIRE(sh > 0 && sw > 0 && dh > 0 && dw > 0 && ph >= 0 && pw >= 0,
              "wxx_conv2d: bad stride/padding/dilation");
  int Ho = (H + 2 * ph - dh * (KH - 1) - 1) / sh + 1;
  int Wo = (W + 2 * pw - dw * (KW - 1) - 1) / sw + 1;
  WXX_REQUIRE(Ho > 0 && Wo > 0, "wxx_conv2d: empty output");
  int64_t Mrows = (int64_t)B * Ho * Wo;
  int64_t K = (int64_t)Cin * KH * KW;
  WXX_REQUIRE(Mrows < (int64_t(1) << 31) && K < (int64_t(1) << 31), "wxx_conv2d: too large");
  if (Mrows == 0) return WXX_OK;
  {
    const size_t smem =
        ((((size_t)Cin * (H + 2 * ph) * (W + 2 * pw) + 3) & ~size_t(3)) + (size_t)K * kDirectCG) * 4;
    if (Cin <= 4 && smem <= 96 * 1024 && B <= 65535 * 8) {
      static bool attr = false;
      if (!attr) {
        WXX_CUDA_CHECK(cudaFuncSetAttribute(conv_direct_kernel<7>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            96 * 1024));
        WXX_CUDA_CHECK(cudaFuncSetAttribute(conv_direct_kernel<3>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            96 * 1024));
        WXX_CUDA_CHECK(cudaFuncSetAttribute(conv_direct_kernel<0>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            96 * 1024));
        attr = true;
      }
      const unsigned blocks = (unsigned)((int64_t)B * ((Cout + kDirectCG - 1) / kDirectCG));
      // one thread per pair of output pixels, up to 256
      const int pairs = (Ho * Wo + 1) / 2;
      const int threads = pairs >= 256 ? 256 : ((pairs + 31) / 32) * 32;
      cudaStream_t st = wxx::stream();
      if (KW == 7)
        conv_direct_kernel<7><<<blocks, threads, smem, st>>>(Y, X, Wt, bias, Cin, H, W, Cout, KH,
                                                             KW, sh, sw, ph, pw, dh, dw, Ho, Wo,
                                                             post);
      else if (KW == 3)
        conv_direct_kernel<3><<<blocks, threads, smem, st>>>(Y, X, Wt, bias, Cin, H, W, Cout, KH,
                                                             KW, sh, sw, ph, pw, dh, dw, Ho, Wo,
                                                             post);
      else
        conv_direct_kernel<0><<<blocks, threads, smem, st>>>(Y, X, Wt, bias, Cin, H, W, Cout, KH,
                                                             KW, sh, sw, ph, pw, dh, dw, Ho, Wo,
                                                             post);
      WXX_LAUNCH_CHECK();
      return WXX_OK;
    }
  }
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = (int)Mrows;
  p.N = Cout;
  p.K = (int)K;
  p.batch = 1;
  p.num_kb = (int)((K + BK - 1) / BK);
  p.passes = mode == 0 ? 1 : 3;
  p.splits = 1;
  p.kb_per_split = p.num_kb * p.passes;
  p.err = wxx::device_error_word();
  int bn = pick_bn(Mrows, Cout, 1);
  CUtensorMap ma, mb;
  memset(&ma, 0, sizeof(ma));
  memset(&mb, 0, sizeof(mb));
  // A: im2col gather.
  p.a.kind = 3;
  p.a.base = X;
  p.a.rows_total = (int)Mrows;
  p.a.k_total = (int)K;
  p.a.cin = Cin; p.a.h = H; p.a.w = W; p.a.kh = KH; p.a.kw = KW;
  p.a.sh = sh; p.a.sw = sw; p.a.ph = ph; p.a.pw = pw; p.a.dh = dh; p.a.dw = dw;
  p.a.ho = Ho; p.a.wo = Wo;
  // B: weights as [Cout, K] K-major.
  OperandDesc db{Wt, Cout, K, 1, K, 0, true, false};
  setup_operand(db, bn, mode == 0, p.b, &mb);
  p.epi.kind = 1;
  p.epi.C = Y;
  p.epi.bias = bias;
  p.epi.bias_mode = bias ? 1 : 0;
  p.epi.alpha = 1.0f;
  p.epi.hw_out = Ho * Wo;
  p.epi.post = post;
  if (plan_splits(p, bn)) return run_splitk(bn, ma, ma, mb, mb, p);
  return run_tc(bn, ma, ma, mb, mb, p);
}
}  // namespace
