// Fused multi-head attention on tcgen05 (TF32), forward only.
//
// Computes, per (batch b, head h), the reference's MultiHeadAttention core
// (nn/module.py:460-495):
//     scores = (Q K^T) * scale  (+ mask)      softmax over keys      O = P V
// without materialising the (B*H, S, S) score tensor.  Q, K, V are read in
// place from the projection outputs laid out (B, S, H, hd) (the reshape /
// permute / reshape head split of the reference becomes 4-D TMA boxes), and
// O is written in the merged (B, S, H*hd) layout the output projection reads,
// so the four head split/merge copies disappear too.
//
// A CTA owns one 128-row query tile of one (b, h) (the default: three CTAs
// per SM) or two tiles sharing each K / V block (WXX_ATTN_TILES=2, one CTA
// per SM); keys / values come in blocks of 64:
//   warp 0      TMA producer (Q once; K_j and V_j in stages with separate
//               barriers, so K_{j+1} loads as soon as S_j has read K_j)
//   warp 1      (and warp 10 for a second tile) one tcgen05.mma-issuing
//               thread per tile (warp 1 also owns the TMEM allocation): per
//               block j S_t(j) = Q_t K_j^T (M=128, N=64, K=hd) and
//               O_t += P_t(j) V_j (M=128, N=hd, K=64; P from TMEM, V MN-major
//               with the 32B-atom swizzle), O_t accumulated in TMEM
//   warps 2..5  (6..9 for a second tile) softmax: one query row per thread,
//               tcgen05.ld S, online softmax in the log2 domain on packed
//               fp32 pairs, P written back into TMEM over S (tcgen05.st; the
//               P V product reads its A operand from TMEM), final O / l
//               through a TMA store
// Every SM sub-partition runs a softmax warp of each resident tile, so one
// tile's exponentials overlap another's S and P V products.
// The running max used for P is only raised (and O in TMEM rescaled) when a
// row's max grows by more than 2^8 in probability units; P and the row sum l
// always use the same max, so O / l is unchanged by the laziness.
// Masked scores (causal: key > query; keys >= Sk) contribute exactly zero
// probability, as exp(score - 1e9 - max) underflows to 0 in the reference; an
// additive mask is added to the scaled scores.  With `causal`, key blocks above
// a tile's diagonal are skipped.  All waits are bounded (see tc_gemm.cuh).
#include "tc_gemm.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

using namespace wxx_tc;

namespace {

constexpr int BQ = 128;   // query rows per tile (UMMA M)
constexpr int BKV = 64;   // keys per block (UMMA N of S, K of PV)
// NT query tiles per CTA: 2 (one CTA per SM, K / V blocks shared by both
// tiles) or 1 (three CTAs per SM: one CTA's setup, loads, waits for S and
// output drain overlap the others' work).  Warps: producer, tile 0's MMA
// thread, 4 softmax warps per tile, then (NT = 2) tile 1's MMA thread.
__host__ __device__ constexpr int att_threads(int nt) { return 64 + nt * 128 + (nt - 1) * 32; }
__host__ __device__ constexpr int mma_warp1(int nt) { return 2 + nt * 4; }   // tile 1's MMA warp (NT = 2)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;   // raise the max used for P only past 2^8

// X3: the fp32-faithful 3xTF32 form (one tile per CTA, one CTA per SM).
// Each product x*y becomes hi(x)hi(y) + lo(x)hi(y) + hi(x)lo(y) where hi is
// the operand as the tensor core reads it (the low 13 mantissa bits
// dropped) and lo = x - hi(x): S = Q K^T + Qlo K^T + Q Klo^T and
// O += P V + Plo V + P Vlo.  Klo / Vlo are made in shared memory by a split
// warp as each block lands, Qlo (once) and Plo (per block) in TMEM by the
// softmax warps, which also keep P unrounded.
template <int HD, int NT, bool X3 = false>
struct ACfg {
  // One TF32 tile per CTA runs three CTAs per SM: one S / P buffer and one
  // K / V stage each (64 KB of shared memory, 128 TMEM columns), so while one
  // CTA's softmax waits for its next S, the other two keep the tensor core
  // and the SFU busy (measured faster than two CTAs with three S buffers and
  // two stages each, which spend the wait inside one CTA).
  static constexpr bool THREE = NT == 1 && !X3;
  static constexpr int Q_BYTES = BQ * HD * 4;          // per tile: 32 KB (hd 64)
  static constexpr int K_BYTES = BKV * HD * 4;         // 16 KB
  static constexpr int V_BYTES = BKV * HD * 4;         // 16 KB
  static constexpr int KVS = (NT == 2 && !X3) ? 4 : (THREE ? 1 : 2); // K / V pipeline stages
  static constexpr int STAGE_O_BYTES = 4 * 4096;       // per tile: O staging for the TMA store
  static constexpr int OFF_K = NT * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KVS * K_BYTES;
  static constexpr int OFF_KLO = OFF_V + KVS * V_BYTES;             // X3 only
  static constexpr int OFF_VLO = OFF_KLO + (X3 ? KVS * K_BYTES : 0);
  static constexpr int OFF_O = OFF_VLO + (X3 ? KVS * V_BYTES : 0);
  // NT = 1 stages O in its Q buffer (every S product has completed by then)
  static constexpr int SMEM = OFF_O + (NT == 2 ? NT * STAGE_O_BYTES : 0) + 1024;
  // TMEM per tile: SB S / P buffers of 64 columns then O (hd columns); X3
  // adds the Plo double buffer and Qlo.  With two tiles per CTA (one CTA per
  // SM) three S buffers let the MMA thread issue S(j + 1) right after
  // P(j - 1) V(j - 1) without waiting for that product to finish (it
  // overwrites P(j - 2)); the 3xTF32 form keeps two, which also orders its
  // Plo writes after the product that read them.
  static constexpr int SB = X3 ? 2 : (THREE ? 1 : 3);
  static constexpr int TMEM_TILE = SB * BKV + HD;
  static constexpr int PLO_COL = TMEM_TILE;
  static constexpr int QLO_COL = TMEM_TILE + 2 * BKV;
  static constexpr int TMEM_COLS = (NT == 2 || X3) ? 512 : (THREE ? 128 : 256);
  static constexpr bool ONE_PER_SM = NT == 2 || X3;
  static constexpr int PER_SM = ONE_PER_SM ? 1 : (THREE ? 3 : 2);
  static_assert(NT == 1 || NT == 2, "one or two query tiles per CTA");
  static_assert(!X3 || NT == 1, "the 3xTF32 form runs one tile per CTA");
  static_assert(NT * TMEM_TILE <= TMEM_COLS, "TMEM layout");
  static_assert(!X3 || QLO_COL + HD <= TMEM_COLS, "TMEM layout (3xTF32)");
  static_assert(NT == 2 || Q_BYTES >= STAGE_O_BYTES, "O staging in the Q buffer");
  static_assert(SMEM <= (ONE_PER_SM ? 227 * 1024 : (THREE ? 74 : 112) * 1024), "shared memory layout");
};

__device__ __forceinline__ float tf32_low(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// dst = lo(src) elementwise over a shared-memory tile (any layout: the
// descriptors that read src read dst the same way), one warp.
__device__ __forceinline__ void split_low_tile(const uint8_t* src, uint8_t* dst, int bytes,
                                               int lane) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int i = lane; i < bytes / 16; i += 32) {
    float4 v = s4[i];
    v.x = tf32_low(v.x);
    v.y = tf32_low(v.y);
    v.z = tf32_low(v.z);
    v.w = tf32_low(v.w);
    d4[i] = v;
  }
}

struct AttnParams {
  int B, H, Sq, Sk;
  int n_qpairs;
  float scale;
  int causal;
  int out_tf32;           // O stored rounded to the nearest TF32 value
  const float* mask;      // additive (Sq, Sk) mask, row stride mask_ld, or NULL
  int64_t mask_ld;
  int* err;
};

template <int HD, bool HAS_MASK, int NT, bool X3 = false>
__global__ void __launch_bounds__(att_threads(NT) + (X3 ? 32 : 0), ACfg<HD, NT, X3>::PER_SM)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_o, const AttnParams p) {
  using C = ACfg<HD, NT, X3>;
  constexpr int MMA_WARP1 = mma_warp1(NT);
  constexpr int SPLIT_WARP = att_threads(NT) / 32;   // X3: makes Klo / Vlo
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t k_full[C::KVS], k_empty[C::KVS], v_full[C::KVS], v_empty[C::KVS];
  __shared__ __align__(8) uint64_t s_full[NT][C::SB], p_full[NT][C::SB], p_empty[NT][C::SB];
  __shared__ __align__(8) uint64_t drain_bar[NT];
  __shared__ __align__(8) uint64_t klo_full[C::KVS], vlo_full[C::KVS], qlo_full;   // X3
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Heaviest query pairs first (causal work grows with the pair index).
  const int bh = blockIdx.x % (p.B * p.H);
  const int qp = p.n_qpairs - 1 - blockIdx.x / (p.B * p.H);
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qp * (NT * BQ);
  const int n_kv_all = (p.Sk + BKV - 1) / BKV;
  // Key blocks each tile visits (0 for a tile entirely past Sq).
  auto blocks_of = [&](int t) {
    const int qt = q0 + t * BQ;
    int n = qt < p.Sq ? n_kv_all : 0;
    if (p.causal && n) n = min(n, (qt + BQ - 1) / BKV + 1);
    return n;
  };
  const int n_t0 = blocks_of(0), n_t1 = NT == 2 ? blocks_of(1) : 0;
  const int n_kv = max(n_t0, n_t1);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_o);
    abort_flag = 0;
    mbar_init(&q_full, 1);
    for (int s = 0; s < C::KVS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], NT);   // one commit from each tile's MMA thread
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], NT);
    }
    for (int t = 0; t < NT; ++t)
      for (int sb = 0; sb < C::SB; ++sb) {
        mbar_init(&s_full[t][sb], 1);
        mbar_init(&p_full[t][sb], 128);
        mbar_init(&p_empty[t][sb], 1);
      }
    for (int t = 0; t < NT; ++t) mbar_init(&drain_bar[t], 1);
    if (X3) {
      for (int s = 0; s < C::KVS; ++s) {
        mbar_init(&klo_full[s], 1);
        mbar_init(&vlo_full[s], 1);
      }
      mbar_init(&qlo_full, 128);
    }
    fence_barrier_init();
    // The query tiles and the first K / V stages start loading before the
    // TMEM allocation and the block barrier (thread 0 is the TMA producer and
    // initialised the barriers; the first fill of a stage waits for nothing).
    mbar_arrive_expect_tx(&q_full, NT * C::Q_BYTES);
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int a = 0; a < HD / 32; ++a)
        tma_load_4d(smem_u32(smem + t * C::Q_BYTES + a * (BQ * 128)), &tm_q, &q_full, a * 32, h,
                    q0 + t * BQ, b);
    for (int j = 0; j < min(C::KVS, n_kv); ++j) {
      mbar_arrive_expect_tx(&k_full[j], C::K_BYTES);
#pragma unroll
      for (int a = 0; a < HD / 32; ++a)
        tma_load_4d(smem_u32(smem + C::OFF_K + j * C::K_BYTES + a * (BKV * 128)), &tm_k,
                    &k_full[j], a * 32, h, j * BKV, b);
      mbar_arrive_expect_tx(&v_full[j], C::V_BYTES);
#pragma unroll
      for (int a = 0; a < HD / 32; ++a)
        tma_load_4d(smem_u32(smem + C::OFF_V + j * C::V_BYTES + a * (BKV * 128)), &tm_v,
                    &v_full[j], a * 32, h, j * BKV, b);
    }
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      const int pre = min(C::KVS, n_kv);   // stages filled before the block barrier
      int last_k[C::KVS], last_v[C::KVS];
#pragma unroll
      for (int s = 0; s < C::KVS; ++s) last_k[s] = last_v[s] = s < pre ? s : -1;
      for (int j = pre; j < n_kv && ok; ++j) {
        const int s = j % C::KVS;
        const uint32_t par = ((j / C::KVS) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], par, &abort_flag, p.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[s], C::K_BYTES);
#pragma unroll
        for (int a = 0; a < HD / 32; ++a)
          tma_load_4d(smem_u32(smem + C::OFF_K + s * C::K_BYTES + a * (BKV * 128)), &tm_k,
                      &k_full[s], a * 32, h, j * BKV, b);
        last_k[s] = j;
        if (!mbar_wait(&v_empty[s], par, &abort_flag, p.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[s], C::V_BYTES);
#pragma unroll
        for (int a = 0; a < HD / 32; ++a)
          tma_load_4d(smem_u32(smem + C::OFF_V + s * C::V_BYTES + a * (BKV * 128)), &tm_v,
                      &v_full[s], a * 32, h, j * BKV, b);
        last_v[s] = j;
      }
      // No load may still be landing when the CTA exits (abort path included).
      volatile int no_abort = 0;
      mbar_wait(&q_full, 0, &no_abort, p.err);
      for (int s = 0; s < C::KVS; ++s) {
        if (last_k[s] >= 0) mbar_wait(&k_full[s], (last_k[s] / C::KVS) & 1, &no_abort, p.err);
        if (last_v[s] >= 0) mbar_wait(&v_full[s], (last_v[s] / C::KVS) & 1, &no_abort, p.err);
      }
    }
  } else if (warp == 1 || (NT == 2 && warp == MMA_WARP1)) {
    // ------------------------------------------------ MMA issuers, one thread per tile
    // Each tile's chain (S_t(j+1) issued, then wait P_t(j), then O_t += P_t(j) V_j)
    // runs on its own thread, so one tile's softmax never holds up the other
    // tile's next S.  K and V stages are released when both threads committed.
    if (lane == 0) {
      const int t = (warp == 1) ? 0 : 1;
      const int nt = t ? n_t1 : n_t0;
      const uint32_t idesc_s = idesc_tf32_mn(BQ, BKV, false, false);
      const uint32_t idesc_o = idesc_tf32_mn(BQ, HD, false, true);
      const uint32_t sbase = smem_u32(smem);
      const uint32_t sq = sbase + t * C::Q_BYTES;
      bool ok = mbar_wait(&q_full, 0, &abort_flag, p.err);
      if (X3 && ok) ok = mbar_wait(&qlo_full, 0, &abort_flag, p.err);
      tc_fence_after();
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj % C::KVS;       // V stage
        const int sb = jj % C::SB;       // TMEM S / P buffer
        if (!mbar_wait(&v_full[s], (jj / C::KVS) & 1, &abort_flag, p.err)) return false;
        if (X3 && !mbar_wait(&vlo_full[s], (jj / C::KVS) & 1, &abort_flag, p.err)) return false;
        tc_fence_after();
        if (jj < nt) {
          if (!mbar_wait(&p_full[t][sb], (jj / C::SB) & 1, &abort_flag, p.err)) return false;
          tc_fence_after();
          const uint32_t sv = sbase + C::OFF_V + s * C::V_BYTES;
          const uint32_t d = tmem_base + t * C::TMEM_TILE + C::SB * BKV;
          const uint32_t pa = tmem_base + t * C::TMEM_TILE + sb * BKV;  // P_t(jj) over S_t(jj)
#pragma unroll
          for (int kk = 0; kk < BKV / 8; ++kk) {
            uint64_t bd = sdesc(sv + kk * 1024, BKV * 128, 512, kLayoutSW128Base32B);
            umma_tf32_ts(d, pa + kk * 8, bd, idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          if (X3) {
            const uint32_t plo = tmem_base + C::PLO_COL + sb * BKV;
            const uint32_t svlo = sbase + C::OFF_VLO + s * C::V_BYTES;
#pragma unroll
            for (int kk = 0; kk < BKV / 8; ++kk) {
              uint64_t bd = sdesc(sv + kk * 1024, BKV * 128, 512, kLayoutSW128Base32B);
              umma_tf32_ts(d, plo + kk * 8, bd, idesc_o, 1u);
            }
#pragma unroll
            for (int kk = 0; kk < BKV / 8; ++kk) {
              uint64_t bd = sdesc(svlo + kk * 1024, BKV * 128, 512, kLayoutSW128Base32B);
              umma_tf32_ts(d, pa + kk * 8, bd, idesc_o, 1u);
            }
          }
          umma_commit(&p_empty[t][sb]);
        }
        umma_commit(&v_empty[s]);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % C::KVS;        // K stage
        const int sb = j % C::SB;        // TMEM S buffer
        // One S buffer: S(j) overwrites P(j - 1), so P(j - 1) V(j - 1) goes first.
        if (C::SB == 1 && j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
        if (!mbar_wait(&k_full[s], (j / C::KVS) & 1, &abort_flag, p.err)) { ok = false; break; }
        if (X3 && !mbar_wait(&klo_full[s], (j / C::KVS) & 1, &abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        if (j < nt) {
          // S_t(j) overwrites the columns P_t(j - SB) occupied: that P V
          // product must have finished reading them.
          if (j >= C::SB &&
              !mbar_wait(&p_empty[t][sb], ((j - C::SB) / C::SB) & 1, &abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sk = sbase + C::OFF_K + s * C::K_BYTES;
          const uint32_t d = tmem_base + t * C::TMEM_TILE + sb * BKV;
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk) {
            uint64_t ad = sdesc(sq + (kk >> 2) * (BQ * 128) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
            uint64_t bd = sdesc(sk + (kk >> 2) * (BKV * 128) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
            umma_tf32(d, ad, bd, idesc_s, kk ? 1u : 0u);
          }
          if (X3) {
            const uint32_t sklo = sbase + C::OFF_KLO + s * C::K_BYTES;
            const uint32_t qlo = tmem_base + C::QLO_COL;
#pragma unroll
            for (int kk = 0; kk < HD / 8; ++kk) {
              uint64_t ad = sdesc(sq + (kk >> 2) * (BQ * 128) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
              uint64_t bd = sdesc(sklo + (kk >> 2) * (BKV * 128) + (kk & 3) * 32, 16, 1024,
                                  kLayoutSW128);
              umma_tf32(d, ad, bd, idesc_s, 1u);
            }
#pragma unroll
            for (int kk = 0; kk < HD / 8; ++kk) {
              uint64_t bd = sdesc(sk + (kk >> 2) * (BKV * 128) + (kk & 3) * 32, 16, 1024, kLayoutSW128);
              umma_tf32_ts(d, qlo + kk * 8, bd, idesc_s, 1u);
            }
          }
          umma_commit(&s_full[t][sb]);
        }
        umma_commit(&k_empty[s]);
        if (C::SB > 1 && j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n_kv >= 1) issue_pv(n_kv - 1);
      umma_commit(&drain_bar[t]);
      volatile int no_abort = 0;
      mbar_wait(&drain_bar[t], 0, &no_abort, p.err);
    }
  } else if (X3 && warp == SPLIT_WARP) {
    // ------------------------------------------------ X3: Klo / Vlo as blocks land
    // A stage is refilled only after the S (V: P V) products that read it
    // and its low part committed, so the low part is never overwritten early.
    for (int j = 0; j < n_kv; ++j) {
      const int s = j % C::KVS;
      const uint32_t par = (j / C::KVS) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&k_full[s], par, &abort_flag, p.err))) break;
      split_low_tile(smem + C::OFF_K + s * C::K_BYTES, smem + C::OFF_KLO + s * C::K_BYTES,
                     C::K_BYTES, lane);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&klo_full[s]);
      if (!__all_sync(0xffffffffu, mbar_wait(&v_full[s], par, &abort_flag, p.err))) break;
      split_low_tile(smem + C::OFF_V + s * C::V_BYTES, smem + C::OFF_VLO + s * C::V_BYTES,
                     C::V_BYTES, lane);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&vlo_full[s]);
    }
  } else {
    // ------------------------------------------------ softmax (one row per thread)
    // Scores are carried in the log2 domain, t = (score * scale + mask) * log2(e),
    // so each probability is one ex2: p = 2^(t - m) = exp(score' - max').
    const int tile = (warp - 2) >> 2;
    const int quarter = warp & 3;                 // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;          // TMEM lane = query row in the tile
    const int qt = q0 + tile * BQ;
    const int qrow = qt + row;
    const int nt = tile ? n_t1 : n_t0;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + tile * C::TMEM_TILE;
    const uint32_t o_addr = lane_addr + C::SB * BKV;
    const float sl2 = p.scale * kLog2e;
    // Keys [0, lim) are visible to this row (causal stops at the query, Sk at
    // the end); warp_lim is the smallest lim of the warp's 32 rows.
    const int lim = p.causal ? min(p.Sk, qrow + 1) : p.Sk;
    const int warp_lim = p.causal ? min(p.Sk, qt + quarter * 32 + 1) : p.Sk;
    const float* mrow = nullptr;
    if (HAS_MASK && qrow < p.Sq) mrow = p.mask + (int64_t)qrow * p.mask_ld;
    uint8_t* pb = NT == 2 ? smem + C::OFF_O + tile * C::STAGE_O_BYTES : smem;
    float m_used = -INFINITY;   // max that P and l are relative to
    float l_run = 0.f;
    bool ok = true;
    if (X3) {
      // Qlo of this thread's query row into TMEM (the S products' third term);
      // the row sits in 128-byte chunks with the 16-byte units XOR-swizzled by
      // the row index (the TMA load's 128B swizzle).
      ok = __all_sync(0xffffffffu, mbar_wait(&q_full, 0, &abort_flag, p.err));
      if (ok) {
        const uint32_t qlo_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + C::QLO_COL;
#pragma unroll
        for (int a = 0; a < HD / 32; ++a) {
          const uint8_t* rb = smem + a * (BQ * 128) + row * 128;
          float v[32];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 f = *reinterpret_cast<const float4*>(rb + ((q ^ (row & 7)) << 4));
            v[4 * q] = tf32_low(f.x);
            v[4 * q + 1] = tf32_low(f.y);
            v[4 * q + 2] = tf32_low(f.z);
            v[4 * q + 3] = tf32_low(f.w);
          }
          tmem_st_32x32(qlo_addr + a * 32, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&qlo_full);
    }

    for (int j = 0; j < nt && ok; ++j) {
      const int s = j % C::SB;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[tile][s], (j / C::SB) & 1, &abort_flag, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float xa[32], xb[32];
      tmem_ld_32x32_nowait(lane_addr + s * BKV, xa);
      tmem_ld_32x32_nowait(lane_addr + s * BKV + 32, xb);
      tmem_ld_wait(xa);
      reg_pin(xb);
#define ATT_X(i) ((i) < 32 ? xa[(i) & 31] : xb[(i) & 31])
      const int k0 = j * BKV;
      // Every key of the block visible to every row of the warp, no mask:
      // the common case skips the per-key tests (warp-uniform branch).
      const bool full = !HAS_MASK && (k0 + BKV <= warp_lim);
      // Row max over the block: three-input max, 8 independent chains.
      float mm[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mm[c] = -INFINITY;
      if (full) {
#pragma unroll
        for (int i = 0; i < BKV; i += 2)
          mm[(i >> 1) & 7] = fmax3(mm[(i >> 1) & 7], ATT_X(i), ATT_X(i + 1));
      } else {
#pragma unroll
        for (int i = 0; i < BKV; i += 2) {
          const int key = k0 + i;
          float tv0, tv1;
          mul2(tv0, tv1, ATT_X(i), ATT_X(i + 1), sl2, sl2);
          if (HAS_MASK) {
            const float mv0 = (mrow != nullptr && key < lim) ? __ldg(mrow + key) : 0.f;
            const float mv1 = (mrow != nullptr && key + 1 < lim) ? __ldg(mrow + key + 1) : 0.f;
            tv0 = fmaf(mv0, kLog2e, tv0);
            tv1 = fmaf(mv1, kLog2e, tv1);
          }
          tv0 = key < lim ? tv0 : -INFINITY;
          tv1 = key + 1 < lim ? tv1 : -INFINITY;
          if (i < 32) { xa[i & 31] = tv0; xa[(i + 1) & 31] = tv1; }
          else { xb[i & 31] = tv0; xb[(i + 1) & 31] = tv1; }
          mm[(i >> 1) & 7] = fmax3(mm[(i >> 1) & 7], tv0, tv1);
        }
      }
      float mx = fmax3(fmax3(mm[0], mm[1], mm[2]), fmax3(mm[3], mm[4], mm[5]), fmaxf(mm[6], mm[7]));
      if (full) mx *= sl2;                        // scale > 0: max commutes with it
      // Raise the max P is taken against only when it grew past 2^8 (always
      // on the first block, which starts O); otherwise P <= 2^8 stays exact
      // in fp32 and no rescale of O is needed.
      const bool raise = (j == 0) ? true : (mx > m_used + kRescaleLog2);
      const bool warp_rescale = __any_sync(0xffffffffu, j > 0 && raise);
      float factor = 1.f;
      if (raise) {
        const float m_new = fmaxf(m_used, mx);
        factor = (m_used == m_new) ? 1.f : fast_exp2(m_used - m_new);
        l_run *= factor;
        m_used = m_new;
      }
      // A row that sees no key yet keeps p = 0 (m_used = -inf, every t = -inf).
      const float m_use = (m_used == -INFINITY) ? 0.f : m_used;
      // Probabilities two keys at a time (packed fp32 arithmetic); key i adds
      // into acc[i & 7] as a scalar loop would.
      float acc[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = 0.f;
#pragma unroll
      for (int i = 0; i < BKV; i += 2) {
        float a0, a1;
        if (full) fma2(a0, a1, ATT_X(i), ATT_X(i + 1), sl2, sl2, -m_use, -m_use);
        else sub2(a0, a1, ATT_X(i), ATT_X(i + 1), m_use, m_use);
        // Every exponential on the SFU: its ex2 pipe keeps up with the rest
        // of the loop (moving some onto an FMA-pipe polynomial measured
        // slower, the issue slots being the tighter limit).
        float p0 = fast_exp2(a0), p1 = fast_exp2(a1);
        // p in [0, 2^8] (finite, non-negative) rounded to the nearest TF32
        // value by integer ops on its bits (ties away from zero; two ALU
        // instructions, fewer issue slots than the cvt.rna form): the P V
        // product then reads it exactly, and the row sum l below adds the
        // same rounded values, so the weights applied to V sum to one.  X3
        // keeps p exact (its low part goes through the Plo term).
        if (!X3) {
          p0 = __uint_as_float((__float_as_uint(p0) + 0x1000u) & 0xFFFFE000u);
          p1 = __uint_as_float((__float_as_uint(p1) + 0x1000u) & 0xFFFFE000u);
        }
        if (i < 32) { xa[i & 31] = p0; xa[(i + 1) & 31] = p1; }
        else { xb[i & 31] = p0; xb[(i + 1) & 31] = p1; }
        add2(acc[i & 7], acc[(i + 1) & 7], acc[i & 7], acc[(i + 1) & 7], p0, p1);
      }
      {
        float s0, s1, s2, s3, u0, u1;
        add2(s0, s1, acc[0], acc[2], acc[1], acc[3]);
        add2(s2, s3, acc[4], acc[6], acc[5], acc[7]);
        add2(u0, u1, s0, s2, s1, s3);
        l_run += u0 + u1;
      }
      // P_j -> TMEM over the S_j columns just read (row = lane, one column
      // per key): the P V product takes its A operand from there.
      tmem_st_32x32(lane_addr + s * BKV, xa);
      tmem_st_32x32(lane_addr + s * BKV + 32, xb);
      if (X3) {
        // Plo (the P V products' second term) into its own TMEM buffer
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          xa[i] = tf32_low(xa[i]);
          xb[i] = tf32_low(xb[i]);
        }
        const uint32_t plo_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + C::PLO_COL + s * BKV;
        tmem_st_32x32(plo_addr, xa);
        tmem_st_32x32(plo_addr + 32, xb);
      }
#undef ATT_X
      if (warp_rescale) {
        // The previous P V product has finished: O holds every block < j.
        // (No barrier of the ring runs more than one phase ahead of these
        // waits: P(j - 1 + SB) cannot exist before this block's P.)
        if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[tile][(j - 1) % C::SB],
                                               ((j - 1) / C::SB) & 1, &abort_flag, p.err))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // O in TMEM holds blocks < j relative to the old max: scale the rows
        // that raised theirs before P_j V_j accumulates on top.
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          float v[32];
          tmem_ld_32x32(o_addr + c, v);
#pragma unroll
          for (int i = 0; i < 32; i += 2) mul2(v[i], v[i + 1], v[i], v[i + 1], factor, factor);
          tmem_st_32x32(o_addr + c, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&p_full[tile][s]);
    }
    if (ok && nt >= 1) {
      // Last P V product done -> O complete in TMEM and the P buffer free for
      // staging the output.
      ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[tile][(nt - 1) % C::SB],
                                             ((nt - 1) / C::SB) & 1, &abort_flag, p.err));
      tc_fence_after();
    }
    if (ok && nt >= 1) {
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      // Stage 32 x 32 chunks in this warp's slice of the P buffer and
      // TMA-store them into O[b, qt + 32*quarter + r, h, c..c+31].
      uint8_t* st = pb + quarter * 4096;
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        float v[32];
        tmem_ld_32x32(o_addr + c, v);
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; i += 2) mul2(v[i], v[i + 1], v[i], v[i + 1], inv, inv);
        if (!X3 && p.out_tf32) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = tf32_rna(v[i]);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(st + lane * 128 + ((q ^ (lane & 7)) << 4)) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_4d(&tm_o, smem_u32(st), c, h, qt + quarter * 32, b);
          bulk_commit();
        }
      }
      // The staging buffer only has to be read before the CTA exits; the
      // stores themselves complete before the grid does.
      if (lane == 0) bulk_wait_read<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_attn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    cudaGetLastError();
  });
  return fn;
}

// 4-D map over a (B, S, H, hd) tensor with row stride ld (elements between
// consecutive s) and batch stride bs: dims {hd, H, S, B}, box {32, 1, rows, 1}.
bool encode_bshd(CUtensorMap* map, const float* base, int B, int S, int H, int HD, int64_t ld,
                 int64_t bs, int rows, bool mn_major) {
  auto enc = get_encode_attn();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 4) % 16 || (bs * 4) % 16) return false;
  cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)HD * 4, (cuuint64_t)ld * 4, (cuuint64_t)bs * 4};
  cuuint32_t box[4] = {32, 1, (cuuint32_t)rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD, int NT, bool X3 = false>
int launch_attention_nt(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                        const CUtensorMap& mo, AttnParams p, bool has_mask) {
  using C = ACfg<HD, NT, X3>;
  constexpr int threads = att_threads(NT) + (X3 ? 32 : 0);
  static bool attr = false;
  if (!attr) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(attention_kernel<HD, false, NT, X3>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    WXX_CUDA_CHECK(cudaFuncSetAttribute(attention_kernel<HD, true, NT, X3>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr = true;
  }
  p.n_qpairs = (p.Sq + NT * BQ - 1) / (NT * BQ);
  const int64_t grid = (int64_t)p.B * p.H * p.n_qpairs;
  WXX_REQUIRE(grid < (int64_t(1) << 31), "wxx_attention: grid too large");
  if (has_mask)
    attention_kernel<HD, true, NT, X3>
        <<<(unsigned)grid, threads, C::SMEM, wxx::stream()>>>(mq, mk, mv, mo, p);
  else
    attention_kernel<HD, false, NT, X3>
        <<<(unsigned)grid, threads, C::SMEM, wxx::stream()>>>(mq, mk, mv, mo, p);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Query tiles per CTA: WXX_ATTN_TILES=1 or 2, read once.  Default 1 (two
// CTAs per SM): 191 against 169-179 TFLOP/s for two tiles per CTA at the
// GPT2-scaled shape (B 8, S 1024, 16 heads x 64, causal).
int attn_tiles_per_cta() {
  static int nt = [] {
    const char* e = std::getenv("WXX_ATTN_TILES");
    return (e != nullptr && e[0] == '2') ? 2 : 1;
  }();
  return nt;
}

template <int HD>
int launch_attention(float* O, const float* Q, const float* K, const float* V, int B, int H,
                     int Sq, int Sk, int64_t q_ld, int64_t kv_ld, int64_t o_ld, float scale,
                     const float* mask, int64_t mask_ld, int causal, int out_tf32, int mode) {
  CUtensorMap mq, mk, mv, mo;
  if (!encode_bshd(&mq, Q, B, Sq, H, HD, q_ld, q_ld * Sq, BQ, false) ||
      !encode_bshd(&mk, K, B, Sk, H, HD, kv_ld, kv_ld * Sk, BKV, false) ||
      !encode_bshd(&mv, V, B, Sk, H, HD, kv_ld, kv_ld * Sk, BKV, true) ||
      !encode_bshd(&mo, O, B, Sq, H, HD, o_ld, o_ld * Sq, 32, false)) {
    wxx::set_error("wxx_attention: operands are not 16-byte addressable for TMA");
    return WXX_E_ARG;
  }
  AttnParams p;
  memset(&p, 0, sizeof(p));
  p.B = B;
  p.H = H;
  p.Sq = Sq;
  p.Sk = Sk;
  p.scale = scale;
  p.causal = causal;
  p.out_tf32 = (out_tf32 && mode == 0) ? 1 : 0;
  p.mask = mask;
  p.mask_ld = mask_ld;
  p.err = wxx::device_error_word();
  if (mode == 1) return launch_attention_nt<HD, 1, true>(mq, mk, mv, mo, p, mask != nullptr);
  if (attn_tiles_per_cta() == 1) return launch_attention_nt<HD, 1>(mq, mk, mv, mo, p, mask != nullptr);
  return launch_attention_nt<HD, 2>(mq, mk, mv, mo, p, mask != nullptr);
}

}  // namespace

// O = softmax(scale * Q K^T (+ mask)) V per (batch, head) on the tensor cores.
// Q: (B, Sq, H, hd) with row stride q_ld elements between consecutive
// positions (H*hd for the merged projection output); K, V: (B, Sk, H, hd)
// with row stride kv_ld; O: (B, Sq, H, hd) with row stride o_ld.
// hd must be 32 or 64 and scale > 0; pointers and strides 16-byte aligned.  causal = 1 masks
// keys after the query position; mask (Sq x Sk, row stride mask_ld) is added
// to the scaled scores when given.  mode 0: TF32 products, the probabilities
// entering the P V product rounded to the nearest TF32 value; out_tf32 = 1
// also stores O rounded so (for an O read only by the TF32 output
// projection).  mode 1: 3xTF32 products (fp32-faithful; out_tf32 ignored).
WXX_EXPORT int wxx_attention(float* O, const float* Q, const float* K, const float* V, int B,
                             int H, int Sq, int Sk, int hd, int64_t q_ld, int64_t kv_ld,
                             int64_t o_ld, float scale, const float* mask, int64_t mask_ld,
                             int causal, int out_tf32, int mode) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B > 0 && H > 0 && Sq > 0 && Sk > 0, "wxx_attention: empty problem");
  WXX_REQUIRE(hd == 32 || hd == 64, "wxx_attention: head dim %d not in {32, 64}", hd);
  WXX_REQUIRE(scale > 0.f, "wxx_attention: scale must be positive");
  WXX_REQUIRE(mode == 0 || mode == 1, "wxx_attention: mode %d not in {0, 1}", mode);
  if (hd == 32)
    return launch_attention<32>(O, Q, K, V, B, H, Sq, Sk, q_ld, kv_ld, o_ld, scale, mask, mask_ld,
                                causal, out_tf32, mode);
  return launch_attention<64>(O, Q, K, V, B, H, Sq, Sk, q_ld, kv_ld, o_ld, scale, mask, mask_ld,
                              causal, out_tf32, mode);
}
