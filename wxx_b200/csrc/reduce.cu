// Reductions, softmax and normalisation kernels (HBM-bound, single pass).
//
// Reference kernels restated (semantics kept, code our own):
//   reduce.wgsl         sum / mean / sum-of-squares over (outer, reduce, inner)
//                       (functional/reductions.py:27-197, backend/dispatch.py:173-214)
//   reduce_minmax.wgsl  values + u32 indices, with the reference's tie rule
//                       (functional/reductions.py:241-342, reduce_minmax.wgsl:18-77)
//   softmax.wgsl        (functional/activations.py:126-173)
//   meanvarnorm.wgsl    LayerNorm, eps 1e-5 (functional/normalization.py:82-145)
//   rmsnorm.wgsl        RMSNorm, eps 1e-6 (functional/normalization.py:24-79)
//   batchnorm.wgsl      eval and training (functional/normalization.py:148-206)
//
// Every reduction keeps fp32 accumulators in registers and combines them with
// warp shuffles, so one row is read from HBM exactly once (softmax and the
// norms keep the row in registers between the statistics and the output).
// Column reductions (inner > 1) split the reduce axis over a thread-block
// cluster and combine the partial sums through distributed shared memory in a
// fixed rank order, so results are deterministic without global scratch.
#include "common.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over a CTA of `nwarps` warps; every thread gets the total.
template <int NWARPS>
__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < NWARPS; ++k) t += sh[k];
  return t;
}

template <int NWARPS>
__device__ __forceinline__ float block_max(float v, float* sh) {
  v = warp_max(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = sh[0];
#pragma unroll
  for (int k = 1; k < NWARPS; ++k) t = fmaxf(t, sh[k]);
  return t;
}

__device__ __forceinline__ float reduce_elem(float x, int mode) { return mode == 2 ? x * x : x; }

// ------------------------------------------------------------ row reduce (inner == 1)

// One CTA (256 threads) per row.
__global__ void __launch_bounds__(256) row_reduce_kernel(float* __restrict__ out,
                                                         const float* __restrict__ x,
                                                         int64_t rows, int64_t n, int mode) {
  __shared__ float sh[8];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* p = x + row * n;
    float acc = 0.f;
    bool vec = ((reinterpret_cast<uintptr_t>(p) & 15) == 0);
    int64_t n4 = vec ? n / 4 : 0;
    const float4* p4 = reinterpret_cast<const float4*>(p);
    int64_t i = threadIdx.x;
    // four 16-byte loads in flight per thread, added in the same order as
    // the one-at-a-time loop
    for (; i + 768 < n4; i += 1024) {
      const float4 v0 = __ldg(p4 + i), v1 = __ldg(p4 + i + 256), v2 = __ldg(p4 + i + 512),
                   v3 = __ldg(p4 + i + 768);
      acc += reduce_elem(v0.x, mode) + reduce_elem(v0.y, mode) + reduce_elem(v0.z, mode) +
             reduce_elem(v0.w, mode);
      acc += reduce_elem(v1.x, mode) + reduce_elem(v1.y, mode) + reduce_elem(v1.z, mode) +
             reduce_elem(v1.w, mode);
      acc += reduce_elem(v2.x, mode) + reduce_elem(v2.y, mode) + reduce_elem(v2.z, mode) +
             reduce_elem(v2.w, mode);
      acc += reduce_elem(v3.x, mode) + reduce_elem(v3.y, mode) + reduce_elem(v3.z, mode) +
             reduce_elem(v3.w, mode);
    }
    for (; i < n4; i += 256) {
      float4 v = __ldg(p4 + i);
      acc += reduce_elem(v.x, mode) + reduce_elem(v.y, mode) + reduce_elem(v.z, mode) +
             reduce_elem(v.w, mode);
    }
    for (int64_t i = n4 * 4 + threadIdx.x; i < n; i += 256) acc += reduce_elem(p[i], mode);
    float t = block_sum<8>(acc, sh);
    if (threadIdx.x == 0) out[row] = mode == 1 ? t / (float)n : t;
  }
}

// One warp per row for long rows when there are many of them: each lane keeps
// eight 16-byte loads in flight (4 KB per warp), rows spread over every SM.
__global__ void __launch_bounds__(256) row_reduce_warp_vec_kernel(float* __restrict__ out,
                                                                  const float* __restrict__ x,
                                                                  int64_t rows, int64_t n,
                                                                  int mode) {
  const int l = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += warps) {
    const float* p = x + row * n;
    const float4* p4 = reinterpret_cast<const float4*>(p);
    const int64_t n4 = n / 4;   // rows are 16-byte aligned (checked by the host)
    float acc = 0.f;
    int64_t i = l;
    for (; i + 224 < n4; i += 256) {
      float4 v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = __ldg(p4 + i + 32 * q);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        acc += reduce_elem(v[q].x, mode) + reduce_elem(v[q].y, mode) + reduce_elem(v[q].z, mode) +
               reduce_elem(v[q].w, mode);
    }
    for (; i < n4; i += 32) {
      const float4 v = __ldg(p4 + i);
      acc += reduce_elem(v.x, mode) + reduce_elem(v.y, mode) + reduce_elem(v.z, mode) +
             reduce_elem(v.w, mode);
    }
    for (int64_t j = n4 * 4 + l; j < n; j += 32) acc += reduce_elem(p[j], mode);
    acc = warp_sum(acc);
    if (l == 0) out[row] = mode == 1 ? acc / (float)n : acc;
  }
}

// One warp per row (short rows).
__global__ void __launch_bounds__(256) row_reduce_warp_kernel(float* __restrict__ out,
                                                              const float* __restrict__ x,
                                                              int64_t rows, int n, int mode) {
  int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  int l = threadIdx.x & 31;
  if (row >= rows) return;
  const float* p = x + row * n;
  float acc = 0.f;
  for (int i = l; i < n; i += 32) acc += reduce_elem(p[i], mode);
  acc = warp_sum(acc);
  if (l == 0) out[row] = mode == 1 ? acc / (float)n : acc;
}

// ------------------------------------------------------------ column reduce (inner > 1)

constexpr int kColCluster = 8;

// grid.x = col_blocks * kColCluster (cluster along x), grid.y = outer slice.
// CTA = 16 (column quads: 64 columns) x 16 (row lanes).
__global__ void __launch_bounds__(256) col_reduce_cluster_kernel(float* __restrict__ out,
                                                                 const float* __restrict__ x,
                                                                 int64_t outer, int64_t reduce,
                                                                 int64_t inner, int mode) {
  __shared__ float part[16][65];
  __shared__ float red[64];
  cg::cluster_group cluster = cg::this_cluster();
  int split = (int)cluster.block_rank();
  int64_t cb = blockIdx.x / kColCluster;
  int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  int64_t c0 = cb * 64 + tx * 4;
  int64_t chunk = (reduce + kColCluster - 1) / kColCluster;
  int64_t r_begin = split * chunk;
  int64_t r_end = r_begin + chunk < reduce ? r_begin + chunk : reduce;
  for (int64_t o = blockIdx.y; o < outer; o += gridDim.y) {
    const float* base = x + o * reduce * inner;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int64_t r = r_begin + ty;
    if (c0 + 3 < inner && ((reinterpret_cast<uintptr_t>(base + c0) | (inner * 4)) & 15) == 0) {
      // 16-byte loads, eight rows in flight, same per-thread addition order
      for (; r + 112 < r_end; r += 128) {
        float4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          v[q] = __ldg(reinterpret_cast<const float4*>(base + (r + 16 * q) * inner + c0));
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          a0 += reduce_elem(v[q].x, mode);
          a1 += reduce_elem(v[q].y, mode);
          a2 += reduce_elem(v[q].z, mode);
          a3 += reduce_elem(v[q].w, mode);
        }
      }
    }
    for (; r < r_end; r += 16) {
      const float* p = base + r * inner + c0;
      if (c0 + 3 < inner) {
        a0 += reduce_elem(p[0], mode);
        a1 += reduce_elem(p[1], mode);
        a2 += reduce_elem(p[2], mode);
        a3 += reduce_elem(p[3], mode);
      } else {
        if (c0 + 0 < inner) a0 += reduce_elem(p[0], mode);
        if (c0 + 1 < inner) a1 += reduce_elem(p[1], mode);
        if (c0 + 2 < inner) a2 += reduce_elem(p[2], mode);
      }
    }
    part[ty][tx * 4 + 0] = a0;
    part[ty][tx * 4 + 1] = a1;
    part[ty][tx * 4 + 2] = a2;
    part[ty][tx * 4 + 3] = a3;
    __syncthreads();
    if (threadIdx.x < 64) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) t += part[k][threadIdx.x];
      red[threadIdx.x] = t;
    }
    cluster.sync();
    if (split == 0 && threadIdx.x < 64) {
      float t = 0.f;
      for (int k = 0; k < kColCluster; ++k) t += cluster.map_shared_rank(red, k)[threadIdx.x];
      int64_t c = cb * 64 + threadIdx.x;
      if (c < inner) out[o * inner + c] = mode == 1 ? t / (float)reduce : t;
    }
    cluster.sync();
  }
}

// ------------------------------------------------------------ argmax / argmin

// The same rule with one warp per output row (inner == 1): lane l holds the
// slots l + 32 j (j = 0..7), each scanning its stride-256 sequence in order;
// the tree's strides 128, 64 and 32 pair slots of one lane (j with j + 4,
// j + 2, j + 1) and strides 16..1 pair lanes by shuffles -- the same
// comparisons in the same order as the CTA form below, without shared memory
// or barriers.  The row is read in 128-byte warp segments.
__global__ void __launch_bounds__(256) argminmax_warp_kernel(float* __restrict__ vals,
                                                             uint32_t* __restrict__ idx,
                                                             const float* __restrict__ x,
                                                             int64_t rows, int64_t reduce,
                                                             int op) {
  const int l = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += warps) {
    const float* base = x + row * reduce;
    float bv[8];
    uint32_t bi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      bv[j] = op == 0 ? -1e38f : 1e38f;
      bi[j] = 0;
    }
    for (int64_t r0 = 0; r0 < reduce; r0 += 256) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t r = r0 + l + 32 * j;
        v[j] = r < reduce ? __ldg(base + r) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t r = r0 + l + 32 * j;
        const bool better = op == 0 ? (v[j] > bv[j]) : (v[j] < bv[j]);
        if (r < reduce && better) {
          bv[j] = v[j];
          bi[j] = (uint32_t)r;
        }
      }
    }
#pragma unroll
    for (int s = 4; s >= 1; s >>= 1) {   // slot strides 128, 64, 32
#pragma unroll
      for (int j = 0; j < s; ++j) {
        const bool better = op == 0 ? (bv[j + s] > bv[j]) : (bv[j + s] < bv[j]);
        if (better) {
          bv[j] = bv[j + s];
          bi[j] = bi[j + s];
        }
      }
    }
    float b = bv[0];
    uint32_t a = bi[0];
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, b, s);
      const uint32_t oi = __shfl_down_sync(0xffffffffu, a, s);
      const bool better = op == 0 ? (ov > b) : (ov < b);
      if (l < s && better) {
        b = ov;
        a = oi;
      }
    }
    if (l == 0) {
      vals[row] = b;
      idx[row] = a;
    }
  }
}

// One CTA of exactly 256 threads per output, reproducing reduce_minmax.wgsl:
// thread t scans r = t, t+256, ... keeping the first strictly better value
// (initial value -1e38 for max / 1e38 for min, index 0); then a tree over the
// 256 slots with strides 128..1 where slot i takes slot i+s only if strictly
// better, so ties keep the lower slot.
__global__ void __launch_bounds__(256) argminmax_kernel(float* __restrict__ vals,
                                                        uint32_t* __restrict__ idx,
                                                        const float* __restrict__ x,
                                                        int64_t outer, int64_t reduce,
                                                        int64_t inner, int op) {
  __shared__ float sv[256];
  __shared__ uint32_t si[256];
  int t = threadIdx.x;
  int64_t total = outer * inner;
  for (int64_t out_i = blockIdx.x; out_i < total; out_i += gridDim.x) {
    int64_t o = out_i / inner, i = out_i - o * inner;
    const float* base = x + o * reduce * inner + i;
    float best = op == 0 ? -1e38f : 1e38f;
    uint32_t arg = 0;
    for (int64_t r = t; r < reduce; r += 256) {
      float v = base[r * inner];
      bool better = op == 0 ? (v > best) : (v < best);
      if (better) {
        best = v;
        arg = (uint32_t)r;
      }
    }
    // Strides 128, 64, 32 through shared memory.
    sv[t] = best;
    si[t] = arg;
    __syncthreads();
#pragma unroll
    for (int s = 128; s >= 32; s >>= 1) {
      if (t < s) {
        float ov = sv[t + s];
        bool better = op == 0 ? (ov > sv[t]) : (ov < sv[t]);
        if (better) {
          sv[t] = ov;
          si[t] = si[t + s];
        }
      }
      __syncthreads();
    }
    // Strides 16..1 inside warp 0 with shuffles (same pairing: lane i <- i+s).
    if (t < 32) {
      float bv = sv[t];
      uint32_t bi = si[t];
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) {
        float ov = __shfl_down_sync(0xffffffffu, bv, s);
        uint32_t oi = __shfl_down_sync(0xffffffffu, bi, s);
        bool better = op == 0 ? (ov > bv) : (ov < bv);
        if (t < s && better) {
          bv = ov;
          bi = oi;
        }
      }
      if (t == 0) {
        vals[out_i] = bv;
        idx[out_i] = bi;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ softmax

// Row softmax, one warp per row, row held in registers (n <= 32 * PER).
// With a mask, row r computes softmax(x[r] + mask[r % mask_rows]) (the
// attention mask broadcast over batch and heads), the sum rounded to fp32
// exactly as a separate add would be.
template <int PER>
__global__ void __launch_bounds__(256) softmax_warp_kernel(float* __restrict__ y,
                                                           const float* __restrict__ x,
                                                           int64_t rows, int n,
                                                           const float* __restrict__ mask,
                                                           int64_t mask_ld, int64_t mask_rows) {
  int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  int l = threadIdx.x & 31;
  if (row >= rows) return;
  const float* p = x + row * n;
  float* q = y + row * n;
  const float* mrow = mask ? mask + (row % mask_rows) * mask_ld : nullptr;
  float v[PER];
  bool vec = (n % 4 == 0) && !((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(q) |
                                reinterpret_cast<uintptr_t>(mrow)) & 15);
  float m = -1e38f;
  if (vec) {
#pragma unroll
    for (int k = 0; k < PER / 4; ++k) {
      int c = (k * 32 + l) * 4;
      if (c < n) {
        float4 t = reinterpret_cast<const float4*>(p)[k * 32 + l];
        if (mrow) {
          float4 mm = reinterpret_cast<const float4*>(mrow)[k * 32 + l];
          t.x += mm.x; t.y += mm.y; t.z += mm.z; t.w += mm.w;
        }
        v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
      } else {
        v[4 * k] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = -INFINITY;
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int c = k * 32 + l;
      v[k] = c < n ? (mrow ? p[c] + mrow[c] : p[c]) : -INFINITY;
    }
  }
#pragma unroll
  for (int k = 0; k < PER; ++k) m = fmaxf(m, v[k]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    v[k] = expf(v[k] - m);
    s += v[k];
  }
  s = warp_sum(s);
  float inv = 1.0f / s;
  if (vec) {
#pragma unroll
    for (int k = 0; k < PER / 4; ++k) {
      int c = (k * 32 + l) * 4;
      if (c < n)
        reinterpret_cast<float4*>(q)[k * 32 + l] =
            make_float4(v[4 * k] * inv, v[4 * k + 1] * inv, v[4 * k + 2] * inv, v[4 * k + 3] * inv);
    }
  } else {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int c = k * 32 + l;
      if (c < n) q[c] = v[k] * inv;
    }
  }
}

// Long rows: one CTA per row, two reads (the second mostly from L2).
__global__ void __launch_bounds__(256) softmax_block_kernel(float* __restrict__ y,
                                                            const float* __restrict__ x,
                                                            int64_t rows, int64_t n) {
  __shared__ float sh[8];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* p = x + row * n;
    float* q = y + row * n;
    float m = -1e38f, s = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += 256) {
      float v = p[i];
      float nm = fmaxf(m, v);
      s = s * expf(m - nm) + expf(v - nm);
      m = nm;
    }
    float gm = block_max<8>(m, sh);
    s = s * expf(m - gm);
    float gs = block_sum<8>(s, sh);
    float inv = 1.0f / gs;
    for (int64_t i = threadIdx.x; i < n; i += 256) q[i] = expf(p[i] - gm) * inv;
  }
}

// Softmax over a non-last axis: threads run along `inner` (coalesced).
__global__ void softmax_strided_kernel(float* __restrict__ y, const float* __restrict__ x,
                                       int64_t outer, int64_t n, int64_t inner) {
  int64_t total = outer * inner;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t o = t / inner, i = t - o * inner;
    const float* p = x + o * n * inner + i;
    float* q = y + o * n * inner + i;
    float m = -1e38f;
    for (int64_t c = 0; c < n; ++c) m = fmaxf(m, p[c * inner]);
    float s = 0.f;
    for (int64_t c = 0; c < n; ++c) s += expf(p[c * inner] - m);
    float inv = 1.0f / s;
    for (int64_t c = 0; c < n; ++c) q[c * inner] = expf(p[c * inner] - m) * inv;
  }
}

// ------------------------------------------------------------ layer / rms norm

// Row norms, one warp per row, row in registers (n <= 32 * PER).
// kind 0: LayerNorm  y = (x - mean) * inv * g[c] + b[c], inv = var>0 ? rsqrt(var+eps) : 0
// kind 1: RMSNorm    y = x * inv * g[c],                 inv = ms>0 ? rsqrt(ms+eps) : 0
template <int PER>
__global__ void __launch_bounds__(256) norm_warp_kernel(float* __restrict__ y,
                                                        float* __restrict__ stat0,
                                                        float* __restrict__ stat1,
                                                        const float* __restrict__ x,
                                                        const float* __restrict__ g,
                                                        const float* __restrict__ b,
                                                        int64_t rows, int n, float eps, int kind) {
  // kind bit 0: RMSNorm (else LayerNorm); bit 1: y rounded to the nearest TF32 value
  const bool rnd = (kind & 2) != 0;
  kind &= 1;
  int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  int l = threadIdx.x & 31;
  if (row >= rows) return;
  const float* p = x + row * n;
  float* q = y + row * n;
  float v[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    int c = k * 32 + l;
    v[k] = c < n ? p[c] : 0.f;
  }
  float inv, mean = 0.f;
  if (kind == 0) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) s += v[k];
    mean = warp_sum(s) / (float)n;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int c = k * 32 + l;
      float d = c < n ? v[k] - mean : 0.f;
      ss += d * d;
    }
    float var = fmaxf(0.f, warp_sum(ss) / (float)n);
    inv = var > 0.f ? rsqrtf(var + eps) : 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int c = k * 32 + l;
      if (c < n) {
        const float o = (v[k] - mean) * inv * g[c] + b[c];
        q[c] = rnd ? tf32_rna(o) : o;
      }
    }
    if (l == 0) {
      if (stat0) stat0[row] = mean;
      if (stat1) stat1[row] = inv;
    }
  } else {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) ss += v[k] * v[k];
    float ms = warp_sum(ss) / (float)n;
    inv = ms > 0.f ? rsqrtf(ms + eps) : 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int c = k * 32 + l;
      if (c < n) {
        const float o = v[k] * inv * g[c];
        q[c] = rnd ? tf32_rna(o) : o;
      }
    }
    if (l == 0 && stat0) stat0[row] = inv;
  }
}

// norm_warp_kernel with 16-byte accesses: lane l holds the float4 quads
// l, l + 32, ... of its row (Q of them, n <= 128 Q, n a multiple of 4 and
// every pointer 16-byte aligned).  A quarter of the load / store instructions
// of the scalar form, the same two-pass mean / variance.
template <int Q>
__global__ void __launch_bounds__(256) norm_warp4_kernel(float* __restrict__ y,
                                                         float* __restrict__ stat0,
                                                         float* __restrict__ stat1,
                                                         const float* __restrict__ x,
                                                         const float* __restrict__ g,
                                                         const float* __restrict__ b,
                                                         int64_t rows, int n, float eps, int kind) {
  const bool rnd = (kind & 2) != 0;
  kind &= 1;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* p = reinterpret_cast<const float4*>(x + row * n);
  float4* q = reinterpret_cast<float4*>(y + row * n);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  const int n4 = n >> 2;
  float4 v[Q];
#pragma unroll
  for (int k = 0; k < Q; ++k) {
    const int c = k * 32 + l;
    v[k] = c < n4 ? p[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mean = 0.f, inv;
  if (kind == 0) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < Q; ++k) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    mean = warp_sum(s) / (float)n;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < Q; ++k) {
      if (k * 32 + l < n4) {
        const float d0 = v[k].x - mean, d1 = v[k].y - mean, d2 = v[k].z - mean, d3 = v[k].w - mean;
        ss += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
      }
    }
    const float var = fmaxf(0.f, warp_sum(ss) / (float)n);
    inv = var > 0.f ? rsqrtf(var + eps) : 0.f;
  } else {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < Q; ++k)
      ss += (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w);
    const float ms = warp_sum(ss) / (float)n;
    inv = ms > 0.f ? rsqrtf(ms + eps) : 0.f;
  }
#pragma unroll
  for (int k = 0; k < Q; ++k) {
    const int c = k * 32 + l;
    if (c < n4) {
      const float4 gg = __ldg(g4 + c);
      float4 o;
      if (kind == 0) {
        const float4 bb = __ldg(b4 + c);
        o = make_float4((v[k].x - mean) * inv * gg.x + bb.x, (v[k].y - mean) * inv * gg.y + bb.y,
                        (v[k].z - mean) * inv * gg.z + bb.z, (v[k].w - mean) * inv * gg.w + bb.w);
      } else {
        o = make_float4(v[k].x * inv * gg.x, v[k].y * inv * gg.y, v[k].z * inv * gg.z,
                        v[k].w * inv * gg.w);
      }
      if (rnd) o = make_float4(tf32_rna(o.x), tf32_rna(o.y), tf32_rna(o.z), tf32_rna(o.w));
      q[c] = o;
    }
  }
  if (l == 0) {
    if (kind == 0) {
      if (stat0) stat0[row] = mean;
      if (stat1) stat1[row] = inv;
    } else if (stat0) {
      stat0[row] = inv;
    }
  }
}

// Generic (outer, reduce, inner) norm: one CTA per (o, i) column, two reads.
__global__ void __launch_bounds__(256) norm_generic_kernel(float* __restrict__ y,
                                                           float* __restrict__ stat0,
                                                           float* __restrict__ stat1,
                                                           const float* __restrict__ x,
                                                           const float* __restrict__ g,
                                                           const float* __restrict__ b,
                                                           int64_t outer, int64_t n,
                                                           int64_t inner, float eps, int kind) {
  const bool rnd = (kind & 2) != 0;   // bit 1: y rounded to the nearest TF32 value
  kind &= 1;
  __shared__ float sh[8];
  int64_t total = outer * inner;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    int64_t o = t / inner, i = t - o * inner;
    const float* p = x + o * n * inner + i;
    float* q = y + o * n * inner + i;
    if (kind == 0) {
      float s = 0.f;
      for (int64_t r = threadIdx.x; r < n; r += 256) s += p[r * inner];
      float mean = block_sum<8>(s, sh) / (float)n;
      float ss = 0.f;
      for (int64_t r = threadIdx.x; r < n; r += 256) {
        float d = p[r * inner] - mean;
        ss += d * d;
      }
      float var = fmaxf(0.f, block_sum<8>(ss, sh) / (float)n);
      float inv = var > 0.f ? rsqrtf(var + eps) : 0.f;
      for (int64_t r = threadIdx.x; r < n; r += 256) {
        const float o = (p[r * inner] - mean) * inv * g[r] + b[r];
        q[r * inner] = rnd ? tf32_rna(o) : o;
      }
      if (threadIdx.x == 0) {
        if (stat0) stat0[t] = mean;
        if (stat1) stat1[t] = inv;
      }
    } else {
      float ss = 0.f;
      for (int64_t r = threadIdx.x; r < n; r += 256) {
        float v = p[r * inner];
        ss += v * v;
      }
      float ms = block_sum<8>(ss, sh) / (float)n;
      float inv = ms > 0.f ? rsqrtf(ms + eps) : 0.f;
      for (int64_t r = threadIdx.x; r < n; r += 256) {
        const float o = p[r * inner] * inv * g[r];
        q[r * inner] = rnd ? tf32_rna(o) : o;
      }
      if (threadIdx.x == 0 && stat0) stat0[t] = inv;
    }
  }
}

// ------------------------------------------------------------ batch norm

// Eval: y = (x - rm[c]) * rsqrt(rv[c] + eps) * g[c] + b[c] over NCHW.
__global__ void batchnorm_eval_kernel(float* __restrict__ y, const float* __restrict__ x,
                                      const float* __restrict__ g, const float* __restrict__ b,
                                      const float* __restrict__ rm, const float* __restrict__ rv,
                                      int64_t total, int C, int64_t hw, float eps) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int c = (int)((i / hw) % C);
    float inv = rsqrtf(rv[c] + eps);
    y[i] = (x[i] - rm[c]) * inv * g[c] + b[c];
  }
}

// Training statistics: one CTA per channel; writes saved mean / inv_std and
// updates the running statistics with momentum (unbiased variance).
__global__ void __launch_bounds__(256) batchnorm_stats_kernel(float* __restrict__ saved_mean,
                                                              float* __restrict__ saved_inv,
                                                              float* __restrict__ rm,
                                                              float* __restrict__ rv,
                                                              const float* __restrict__ x, int B,
                                                              int C, int64_t hw, float eps,
                                                              float momentum) {
  __shared__ float sh[8];
  int c = blockIdx.x;
  int64_t m = (int64_t)B * hw;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < m; i += 256) {
    int64_t bb = i / hw, sp = i - bb * hw;
    s += x[(bb * C + c) * hw + sp];
  }
  float mean = block_sum<8>(s, sh) / (float)m;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < m; i += 256) {
    int64_t bb = i / hw, sp = i - bb * hw;
    float d = x[(bb * C + c) * hw + sp] - mean;
    ss += d * d;
  }
  float var = fmaxf(0.f, block_sum<8>(ss, sh) / (float)m);
  if (threadIdx.x == 0) {
    float inv = rsqrtf(var + eps);
    saved_mean[c] = mean;
    saved_inv[c] = inv;
    float unbiased = m > 1 ? var * ((float)m / (float)(m - 1)) : var;
    rm[c] = (1.f - momentum) * rm[c] + momentum * mean;
    rv[c] = (1.f - momentum) * rv[c] + momentum * unbiased;
  }
}

__global__ void batchnorm_apply_kernel(float* __restrict__ y, const float* __restrict__ x,
                                       const float* __restrict__ g, const float* __restrict__ b,
                                       const float* __restrict__ mean,
                                       const float* __restrict__ inv, int64_t total, int C,
                                       int64_t hw) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int c = (int)((i / hw) % C);
    y[i] = (x[i] - mean[c]) * inv[c] * g[c] + b[c];
  }
}

template <typename K, typename... Args>
int launch_cluster(K kernel, dim3 grid, dim3 block, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = wxx::stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WXX_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, args...));
  return wxx::after_launch(__FILE__, __LINE__);
}

}  // namespace

// ============================================================ exports

// out[o, i] = reduce_r x[o, r, i]; mode 0 sum, 1 mean, 2 sum of squares.
WXX_EXPORT int wxx_reduce(float* out, const float* x, int64_t outer, int64_t reduce, int64_t inner,
                          int mode) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(mode >= 0 && mode <= 2, "wxx_reduce: mode %d not in 0..2", mode);
  WXX_REQUIRE(outer >= 0 && reduce >= 0 && inner >= 0, "wxx_reduce: negative size");
  if (outer * inner == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  if (reduce == 0) {
    WXX_CUDA_CHECK(cudaMemsetAsync(out, 0, outer * inner * sizeof(float), s));
    return WXX_OK;
  }
  if (inner == 1) {
    if (reduce <= 1024) {
      unsigned grid = (unsigned)((outer + 7) / 8);
      row_reduce_warp_kernel<<<grid, 256, 0, s>>>(out, x, outer, (int)reduce, mode);
    } else if (outer >= 2 * (int64_t)wxx::num_sms() * 8 && reduce % 4 == 0 &&
               (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
      row_reduce_warp_vec_kernel<<<wxx::grid_for(outer * 32, 256), 256, 0, s>>>(out, x, outer,
                                                                               reduce, mode);
    } else {
      row_reduce_kernel<<<wxx::grid_for(outer * 256, 256, 16), 256, 0, s>>>(out, x, outer, reduce,
                                                                            mode);
    }
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  int64_t col_blocks = (inner + 63) / 64;
  WXX_REQUIRE(col_blocks * kColCluster < (int64_t(1) << 31), "wxx_reduce: inner too large");
  unsigned gy = (unsigned)(outer < 65535 ? outer : 65535);
  dim3 grid((unsigned)(col_blocks * kColCluster), gy, 1);
  return launch_cluster(col_reduce_cluster_kernel, grid, dim3(256), kColCluster, out, x, outer,
                        reduce, inner, mode);
}

// vals/idx[o, i] = max (op 0) or min (op 1) over r of x[o, r, i], reference tie rule.
WXX_EXPORT int wxx_argminmax(float* vals, uint32_t* idx, const float* x, int64_t outer,
                             int64_t reduce, int64_t inner, int op) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(op == 0 || op == 1, "wxx_argminmax: op must be 0 (max) or 1 (min)");
  int64_t total = outer * inner;
  if (total == 0) return WXX_OK;
  if (inner == 1) {
    argminmax_warp_kernel<<<wxx::grid_for(outer * 32, 256), 256, 0, wxx::stream()>>>(
        vals, idx, x, outer, reduce, op);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  unsigned grid = (unsigned)(total < (int64_t)wxx::num_sms() * 64 ? total : (int64_t)wxx::num_sms() * 64);
  argminmax_kernel<<<grid, 256, 0, wxx::stream()>>>(vals, idx, x, outer, reduce, inner, op);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Softmax of a dense tensor along an axis of length n: x viewed as (outer, n, inner).
WXX_EXPORT int wxx_softmax(float* y, const float* x, int64_t outer, int64_t n, int64_t inner) {
  WXX_REQUIRE_INIT();
  if (outer * n * inner == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  if (inner == 1) {
    unsigned grid = (unsigned)((outer + 7) / 8);
    const float* nm = nullptr;
    if (n <= 128) softmax_warp_kernel<4><<<grid, 256, 0, s>>>(y, x, outer, (int)n, nm, 0, 1);
    else if (n <= 256) softmax_warp_kernel<8><<<grid, 256, 0, s>>>(y, x, outer, (int)n, nm, 0, 1);
    else if (n <= 512) softmax_warp_kernel<16><<<grid, 256, 0, s>>>(y, x, outer, (int)n, nm, 0, 1);
    else if (n <= 1024) softmax_warp_kernel<32><<<grid, 256, 0, s>>>(y, x, outer, (int)n, nm, 0, 1);
    else softmax_block_kernel<<<wxx::grid_for(outer * 256, 256, 16), 256, 0, s>>>(y, x, outer, n);
  } else {
    softmax_strided_kernel<<<wxx::grid_for(outer * inner, 256), 256, 0, s>>>(y, x, outer, n, inner);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// y[r, :] = softmax(x[r, :] + mask[r % mask_rows, :]) over rows of length n
// (n <= 1024); the mask rows have stride mask_ld.  Fuses the attention mask
// add (nn/module.py:487-488) into the softmax pass.
WXX_EXPORT int wxx_softmax_masked(float* y, const float* x, int64_t rows, int64_t n,
                                  const float* mask, int64_t mask_ld, int64_t mask_rows) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(n > 0 && n <= 1024, "wxx_softmax_masked: row length %lld outside [1, 1024]",
              (long long)n);
  WXX_REQUIRE(mask != nullptr && mask_rows > 0, "wxx_softmax_masked: mask required");
  if (rows == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  unsigned grid = (unsigned)((rows + 7) / 8);
  if (n <= 128) softmax_warp_kernel<4><<<grid, 256, 0, s>>>(y, x, rows, (int)n, mask, mask_ld, mask_rows);
  else if (n <= 256) softmax_warp_kernel<8><<<grid, 256, 0, s>>>(y, x, rows, (int)n, mask, mask_ld, mask_rows);
  else if (n <= 512) softmax_warp_kernel<16><<<grid, 256, 0, s>>>(y, x, rows, (int)n, mask, mask_ld, mask_rows);
  else softmax_warp_kernel<32><<<grid, 256, 0, s>>>(y, x, rows, (int)n, mask, mask_ld, mask_rows);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

namespace {
int launch_norm(float* y, float* s0, float* s1, const float* x, const float* g, const float* b,
                int64_t outer, int64_t n, int64_t inner, float eps, int kind) {
  if (outer * n * inner == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  const bool vec = n % 4 == 0 && n >= 128 &&
                   !((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(x) |
                      reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(b)) & 15);
  if (inner == 1 && n <= 1024 && vec) {
    unsigned grid = (unsigned)((outer + 7) / 8);
    if (n <= 256) norm_warp4_kernel<2><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
    else if (n <= 512) norm_warp4_kernel<4><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
    else norm_warp4_kernel<8><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
  } else if (inner == 1 && n <= 1024) {
    unsigned grid = (unsigned)((outer + 7) / 8);
    if (n <= 128) norm_warp_kernel<4><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
    else if (n <= 256) norm_warp_kernel<8><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
    else if (n <= 512) norm_warp_kernel<16><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
    else norm_warp_kernel<32><<<grid, 256, 0, s>>>(y, s0, s1, x, g, b, outer, (int)n, eps, kind);
  } else {
    norm_generic_kernel<<<wxx::grid_for(outer * inner * 256, 256, 16), 256, 0, s>>>(
        y, s0, s1, x, g, b, outer, n, inner, eps, kind);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
}  // namespace

// LayerNorm over the reduce axis of x (outer, n, inner); gamma/beta have n
// entries; mean/inv_std (outer*inner) may be NULL.  out_tf32 = 1 stores y
// rounded to the nearest TF32 value (y read only by TF32 products).
WXX_EXPORT int wxx_layernorm(float* y, float* mean, float* inv_std, const float* x,
                             const float* gamma, const float* beta, int64_t outer, int64_t n,
                             int64_t inner, float eps, int out_tf32) {
  WXX_REQUIRE_INIT();
  return launch_norm(y, mean, inv_std, x, gamma, beta, outer, n, inner, eps,
                     out_tf32 ? 2 : 0);
}

// RMSNorm over the reduce axis; inv_rms (outer*inner) may be NULL; out_tf32
// as for wxx_layernorm.
WXX_EXPORT int wxx_rmsnorm(float* y, float* inv_rms, const float* x, const float* gamma,
                           int64_t outer, int64_t n, int64_t inner, float eps, int out_tf32) {
  WXX_REQUIRE_INIT();
  return launch_norm(y, inv_rms, nullptr, x, gamma, gamma, outer, n, inner, eps,
                     out_tf32 ? 3 : 1);
}

// BatchNorm over NCHW x (B, C, hw).  training=0: running statistics are used
// (the reference stores a variance in `running_std`); training=1: batch
// statistics are computed, saved_mean/saved_inv written and the running
// statistics updated with `momentum`.
WXX_EXPORT int wxx_batchnorm(float* y, float* saved_mean, float* saved_inv, const float* x,
                             const float* gamma, const float* beta, float* running_mean,
                             float* running_var, int B, int C, int64_t hw, float eps,
                             float momentum, int training) {
  WXX_REQUIRE_INIT();
  int64_t total = (int64_t)B * C * hw;
  if (total == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  if (!training) {
    batchnorm_eval_kernel<<<wxx::grid_for(total, 256), 256, 0, s>>>(y, x, gamma, beta, running_mean,
                                                                   running_var, total, C, hw, eps);
  } else {
    WXX_REQUIRE(saved_mean && saved_inv, "wxx_batchnorm: training needs saved_mean/saved_inv");
    batchnorm_stats_kernel<<<C, 256, 0, s>>>(saved_mean, saved_inv, running_mean, running_var, x, B,
                                             C, hw, eps, momentum);
    WXX_LAUNCH_CHECK();
    batchnorm_apply_kernel<<<wxx::grid_for(total, 256), 256, 0, s>>>(y, x, gamma, beta, saved_mean,
                                                                    saved_inv, total, C, hw);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
