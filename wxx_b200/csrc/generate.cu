// Autoregressive generation on the device: the steps either side of the
// GPT2 forward in the reference's sampling loop (nn/gpt.py:108-170), re-done
// so that a generated token never leaves the GPU.
//
// The reference re-runs the whole prefix forward for every new token and
// copies the full (batch, seq, vocab) logits to the host to pick it.  Here:
//   * a prefill forward over the prompt fills per-layer K / V caches
//     (batch, max_len, D) and computes the LM head for the last position only;
//   * every later token is one decode step of the new position only:
//       decode_embed_kernel     tok_emb[id] + pos_emb[pos] of the last token
//       (per layer) LayerNorm, the QKV GEMM over `batch` rows,
//       decode_attention_kernel appends this position's K / V to the caches
//                               and attends over positions 0..pos
//       ... out projection, MLP, final LayerNorm, LM head (batch rows) ...
//       sample_kernel           picks the next id and advances the length
//   * the current length lives in device memory (`cur_len`), so one decode
//     step is the same launch sequence every time and is replayed from one
//     CUDA graph; the host only supplies the uniform draws (temperature > 0).
//
// Sampling follows the reference's rule exactly (nn/gpt.py:147-163):
// temperature 0 -> the first index of the maximum (numpy argmax); otherwise
// z = logits / T in float64, values below the k-th largest masked (top-k, ties
// at the cutoff kept), p = softmax(z), and the id is the first index whose
// cumulative probability exceeds the row's uniform draw (0 if none does).

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace {

// out[b, :] = tok[ids[b, p], :] + pos[p, :] with p = cur_len - 1 (the last
// token); ids outside the table give zeros and raise WXX_DEV_ERR_BAD_INDEX.
__global__ void decode_embed_kernel(float* __restrict__ out, const uint32_t* __restrict__ ids,
                                    int64_t ids_ld, const int* __restrict__ cur_len,
                                    const float* __restrict__ tok, const float* __restrict__ pos,
                                    int D, uint32_t vocab, int max_len, int* err) {
  const int b = blockIdx.x;
  const int p = *cur_len - 1;
  if (p < 0 || p >= max_len) {
    if (threadIdx.x == 0) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
    return;
  }
  const uint32_t id = ids[b * ids_ld + p];
  const bool ok = id < vocab;
  if (!ok && threadIdx.x == 0) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float t = ok ? tok[(int64_t)id * D + d] : 0.f;
    out[(int64_t)b * D + d] = t + pos[(int64_t)p * D + d];
  }
}

constexpr int kAttnThreads = 256;

// One CTA per (head, sequence).  Appends the new position's K and V (this
// head's hd columns) to the caches, then o = softmax(scale * q . K^T) V over
// positions 0..p in exact fp32.  Scores: one thread per key, its hd / 4
// float4 loads of the key row all in flight at once (a warp per key with a
// shuffle reduction per key would expose one memory latency per key).  P V:
// thread t owns column quad t % (hd / 4) and every (kAttnThreads / (hd / 4))-th
// key, and the key groups are summed in fixed order through shared memory.
// The position is causal by construction: only keys up to the query exist.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
    decode_attention_kernel(float* __restrict__ O, int64_t o_ld, const float* __restrict__ q,
                            const float* __restrict__ k_new, const float* __restrict__ v_new,
                            int64_t qkv_ld, float* __restrict__ Kc, float* __restrict__ Vc,
                            int64_t cache_bs, int D, const int* __restrict__ cur_len, int max_len,
                            float scale, int out_tf32, int* err) {
  constexpr int NQ = HD / 4;                   // float4 per head row
  constexpr int KG = kAttnThreads / NQ;        // key groups of the P V product
  constexpr int NW = kAttnThreads / 32;
  extern __shared__ float s_score[];
  __shared__ __align__(16) float s_q[HD];
  __shared__ float s_red[NW];
  __shared__ __align__(16) float s_part[KG][HD];
  const int h = blockIdx.x, b = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int p = *cur_len - 1;
  if (p < 0 || p >= max_len) {
    if (t == 0) wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
    return;
  }
  const int64_t col = (int64_t)h * HD;
  float* kb = Kc + b * cache_bs + col;
  float* vb = Vc + b * cache_bs + col;
  // The P V product's value rows (thread t: column quad t % (hd / 4), keys
  // t / (hd / 4) + KG u) are loaded first, so they arrive while the scores
  // and the softmax run; the new position's row comes from v_new.
  const int cq = t % NQ, kg = t / NQ;
  constexpr int kPre = 16;
  float4 vpre[kPre];
#pragma unroll
  for (int u = 0; u < kPre; ++u) {
    const int j = kg + u * KG;
    if (j < p) {
      vpre[u] = reinterpret_cast<const float4*>(vb + (int64_t)j * D)[cq];
    } else if (j == p) {
      const float* vn = v_new + b * qkv_ld + col + cq * 4;
      vpre[u] = make_float4(vn[0], vn[1], vn[2], vn[3]);
    } else {
      vpre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  for (int i = t; i < HD; i += kAttnThreads) {
    kb[(int64_t)p * D + i] = k_new[b * qkv_ld + col + i];
    vb[(int64_t)p * D + i] = v_new[b * qkv_ld + col + i];
    s_q[i] = q[b * qkv_ld + col + i];
  }
  __syncthreads();   // the appended K / V rows and q are visible to every thread
  // scores
  const float4* q4 = reinterpret_cast<const float4*>(s_q);
  float mx = -INFINITY;
  for (int j = t; j <= p; j += kAttnThreads) {
    const float4* kr = reinterpret_cast<const float4*>(kb + (int64_t)j * D);
    float4 kv[NQ];
#pragma unroll
    for (int e = 0; e < NQ; ++e) kv[e] = kr[e];
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < NQ; ++e) {
      const float4 qq = q4[e];
      acc = fmaf(qq.x, kv[e].x, acc);
      acc = fmaf(qq.y, kv[e].y, acc);
      acc = fmaf(qq.z, kv[e].z, acc);
      acc = fmaf(qq.w, kv[e].w, acc);
    }
    const float sc = acc * scale;
    s_score[j] = sc;
    mx = fmaxf(mx, sc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s_red[w]);
  __syncthreads();
  // probabilities and their sum
  float sum = 0.f;
  for (int j = t; j <= p; j += kAttnThreads) {
    const float e = expf(s_score[j] - mx);
    s_score[j] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) s_red[warp] = sum;
  __syncthreads();   // also publishes every s_score
  sum = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) sum += s_red[w];
  // o = sum_j p_j v_j
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto pv_add = [&](int j, const float4& v4) {
    const float pj = s_score[j];
    acc.x = fmaf(pj, v4.x, acc.x);
    acc.y = fmaf(pj, v4.y, acc.y);
    acc.z = fmaf(pj, v4.z, acc.z);
    acc.w = fmaf(pj, v4.w, acc.w);
  };
  // the prefetched rows, then four in flight per thread, then one at a time
#pragma unroll
  for (int u = 0; u < kPre; ++u) {
    const int jj = kg + u * KG;
    if (jj <= p) pv_add(jj, vpre[u]);
  }
  int j = kg + kPre * KG;
  for (; j + 3 * KG <= p; j += 4 * KG) {
    float4 v4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      v4[u] = reinterpret_cast<const float4*>(vb + (int64_t)(j + u * KG) * D)[cq];
#pragma unroll
    for (int u = 0; u < 4; ++u) pv_add(j + u * KG, v4[u]);
  }
  for (; j <= p; j += KG) pv_add(j, reinterpret_cast<const float4*>(vb + (int64_t)j * D)[cq]);
  reinterpret_cast<float4*>(&s_part[kg][0])[cq] = acc;
  __syncthreads();
  const float inv = 1.0f / sum;
  for (int i = t; i < HD; i += kAttnThreads) {
    float v = 0.f;
#pragma unroll
    for (int g = 0; g < KG; ++g) v += s_part[g][i];
    v *= inv;
    O[b * o_ld + col + i] = out_tf32 ? tf32_rna(v) : v;
  }
}

}  // namespace

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;

// Order-preserving key of an fp32 value (larger value -> larger key).
__device__ __forceinline__ uint32_t f2key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (value, index) of the block's maximum, ties to the lower index, NaN above
// every number (numpy argmax returns the first NaN).
__device__ __forceinline__ bool arg_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

// Key of the k-th largest value of row[0..V) (k >= 1, counted with
// multiplicity): four 8-bit radix passes over the candidates that share the
// digits found so far.
__device__ uint32_t kth_largest_key(const float* __restrict__ row, int V, int k,
                                    unsigned* hist /* 256 */, unsigned* s_misc /* 2 */) {
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const uint32_t key = f2key(row[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0, d = 255;
      for (; d > 0; --d) {
        if (acc + (int)hist[d] >= remaining) break;
        acc += (int)hist[d];
      }
      s_misc[0] = (unsigned)d;
      s_misc[1] = (unsigned)(remaining - acc);
    }
    __syncthreads();
    prefix |= s_misc[0] << shift;
    mask |= 255u << shift;
    remaining = (int)s_misc[1];
    __syncthreads();
  }
  return prefix;
}

// One CTA per sequence.  Writes the chosen id at ids[b, cur_len]; the last
// CTA to finish advances cur_len (done_count returns to 0 for the next step).
__global__ void __launch_bounds__(kSampleThreads)
    sample_kernel(uint32_t* __restrict__ ids, int64_t ids_ld, int* cur_len, unsigned* done_count,
                  const float* __restrict__ logits, int64_t ld, int V, float temperature,
                  int top_k, const double* __restrict__ draws, int B, int max_len, int* err) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_misc[2];
  __shared__ float s_v[kSampleWarps];
  __shared__ int s_i[kSampleWarps];
  __shared__ double s_d[kSampleWarps];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* row = logits + b * ld;
  const int len = *cur_len;
  int chosen = 0;
  // the maximum (first index): the argmax itself, or the softmax shift
  float bv = -INFINITY;
  int bi = V;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = row[i];
    if (arg_better(x, i, bv, bi)) { bv = x; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
  __syncthreads();
  bv = s_v[0];
  bi = s_i[0];
  for (int w = 1; w < kSampleWarps; ++w)
    if (arg_better(s_v[w], s_i[w], bv, bi)) { bv = s_v[w]; bi = s_i[w]; }
  __syncthreads();
  if (temperature == 0.f) {
    chosen = bi;
  } else {
    // top-k cutoff: values strictly below the k-th largest are dropped
    const bool filter = top_k > 0 && top_k < V;
    const uint32_t cut = filter ? kth_largest_key(row, V, top_k, hist, s_misc) : 0u;
    const double T = (double)temperature;
    const double m = (double)bv / T;
    // each thread owns a contiguous chunk; chunk sums of exp(z - max) in float64
    const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
    const int c0 = min(V, threadIdx.x * chunk), c1 = min(V, c0 + chunk);
    double part = 0.0;
    for (int i = c0; i < c1; ++i) {
      const float x = row[i];
      if (!filter || f2key(x) >= cut) part += exp((double)x / T - m);
    }
    // exclusive prefix of the chunk sums over the block
    double incl = part;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) s_d[warp] = incl;
    __syncthreads();
    double warp_base = 0.0, total = 0.0;
    for (int w = 0; w < kSampleWarps; ++w) {
      if (w < warp) warp_base += s_d[w];
      total += s_d[w];
    }
    const double before = warp_base + incl - part;
    // first index whose cumulative probability exceeds the draw
    const double target = draws[b] * total;
    int first = V;
    if (before + part > target && c1 > c0) {
      double run = before;
      for (int i = c0; i < c1; ++i) {
        const float x = row[i];
        if (!filter || f2key(x) >= cut) run += exp((double)x / T - m);
        if (run > target) { first = i; break; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    __syncthreads();
    if (lane == 0) s_i[warp] = first;
    __syncthreads();
    first = s_i[0];
    for (int w = 1; w < kSampleWarps; ++w) first = min(first, s_i[w]);
    chosen = first < V ? first : 0;   // no crossing: numpy's argmax of all-False is 0
  }
  if (threadIdx.x == 0) {
    if (len < 0 || len >= max_len) {
      wxx_device_fail(err, WXX_DEV_ERR_BAD_INDEX);
    } else {
      ids[b * ids_ld + len] = (uint32_t)chosen;
    }
    __threadfence();
    const unsigned prev = atomicAdd(done_count, 1u);
    if (prev == (unsigned)B - 1) {
      *done_count = 0;
      if (len >= 0 && len < max_len) *cur_len = len + 1;
      __threadfence();
    }
  }
}

}  // namespace

// Embedding of the last token of each sequence for a decode step:
// out (B, D) = tok_emb[ids[b, p]] + pos_emb[p], p = *cur_len - 1 read on the
// device.  ids (B, >= max_len) row stride ids_ld; tok_emb (vocab, D); pos_emb
// (max_len, D).  Reference: nn/gpt.py:101-103 (the token and position
// embeddings of the forward), here for one position.
WXX_EXPORT int wxx_decode_embed(float* out, const uint32_t* ids, int64_t ids_ld,
                                const int* cur_len, const float* tok_emb, const float* pos_emb,
                                int B, int D, int vocab, int max_len) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B >= 0 && D > 0 && vocab > 0 && max_len > 0, "wxx_decode_embed: bad sizes");
  if (B == 0) return WXX_OK;
  decode_embed_kernel<<<B, 256, 0, wxx::stream()>>>(out, ids, ids_ld, cur_len, tok_emb, pos_emb, D,
                                                    (uint32_t)vocab, max_len,
                                                    wxx::device_error_word());
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Attention of one new position per sequence against its K / V cache
// (nn/module.py:460-495 for a single query row, causal): the position
// p = *cur_len - 1's K and V (k_new, v_new: row b at b * qkv_ld, heads
// interleaved along D = H * hd) are appended to Kc / Vc (B, max_len, D) with
// batch stride cache_bs, then O[b] (row stride o_ld) = softmax(scale q . K^T)
// V over positions 0..p, exact fp32.  hd 32 or 64; out_tf32 = 1 stores O
// rounded to the nearest TF32 value.
WXX_EXPORT int wxx_decode_attention(float* O, int64_t o_ld, const float* q, const float* k_new,
                                    const float* v_new, int64_t qkv_ld, float* Kc, float* Vc,
                                    int64_t cache_bs, int B, int H, int hd, const int* cur_len,
                                    int max_len, float scale, int out_tf32) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B >= 0 && H > 0 && max_len > 0, "wxx_decode_attention: bad sizes");
  WXX_REQUIRE(hd == 32 || hd == 64, "wxx_decode_attention: head dim %d not in {32, 64}", hd);
  WXX_REQUIRE(!(reinterpret_cast<uintptr_t>(Kc) & 15) && !(reinterpret_cast<uintptr_t>(Vc) & 15) &&
                  cache_bs % 4 == 0,
              "wxx_decode_attention: the caches must be 16-byte aligned (float4 rows)");
  WXX_REQUIRE((int64_t)max_len * 4 <= 200 * 1024,
              "wxx_decode_attention: max_len %d exceeds the shared-memory score row", max_len);
  if (B == 0) return WXX_OK;
  const size_t smem = (size_t)max_len * sizeof(float);
  dim3 grid((unsigned)H, (unsigned)B);
  const int D = H * hd;
  // the largest score row this process asked for so far (attribute set outside
  // any graph capture in practice: the first call of a size runs eagerly)
  static size_t smem_set[2] = {0, 0};
  const int which = hd == 32 ? 0 : 1;
  if (smem > 48 * 1024 && smem > smem_set[which]) {
    if (which == 0)
      WXX_CUDA_CHECK(cudaFuncSetAttribute(decode_attention_kernel<32>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    else
      WXX_CUDA_CHECK(cudaFuncSetAttribute(decode_attention_kernel<64>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set[which] = smem;
  }
  if (hd == 32) {
    decode_attention_kernel<32><<<grid, kAttnThreads, smem, wxx::stream()>>>(
        O, o_ld, q, k_new, v_new, qkv_ld, Kc, Vc, cache_bs, D, cur_len, max_len, scale, out_tf32,
        wxx::device_error_word());
  } else {
    decode_attention_kernel<64><<<grid, kAttnThreads, smem, wxx::stream()>>>(
        O, o_ld, q, k_new, v_new, qkv_ld, Kc, Vc, cache_bs, D, cur_len, max_len, scale, out_tf32,
        wxx::device_error_word());
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Next-token choice of the reference's sampling loop (nn/gpt.py:147-163) for
// each of B rows of logits (row stride ld, V entries): temperature 0 -> first
// index of the maximum; else top_k (0 = no filter) and the inverse-CDF draw
// draws[b] in [0, 1) on the float64 softmax of logits / temperature.  The id
// goes to ids[b, *cur_len] (row stride ids_ld) and *cur_len advances by one
// once every row is written.  done_count: a device counter that starts at 0
// (it is left at 0).
WXX_EXPORT int wxx_sample_tokens(uint32_t* ids, int64_t ids_ld, int* cur_len,
                                 unsigned* done_count, const float* logits, int64_t ld, int B,
                                 int V, float temperature, int top_k, const double* draws,
                                 int max_len) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(B >= 0 && V > 0 && max_len > 0, "wxx_sample_tokens: bad sizes");
  WXX_REQUIRE(temperature >= 0.f, "wxx_sample_tokens: temperature must be non-negative");
  WXX_REQUIRE(temperature == 0.f || draws != nullptr,
              "wxx_sample_tokens: sampling needs one uniform draw per row");
  if (B == 0) return WXX_OK;
  sample_kernel<<<B, kSampleThreads, 0, wxx::stream()>>>(ids, ids_ld, cur_len, done_count, logits,
                                                         ld, V, temperature, top_k, draws, B,
                                                         max_len, wxx::device_error_word());
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
