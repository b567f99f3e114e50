// Real FFTs and the fused FFT causal convolution.
//
// Reference semantics (functional/fft.py:484-645, fft_*.wgsl, nn/hyena.py:208-216):
//   rfft(x, n)  = numpy.fft.rfft(x, n): zero-pad / truncate the last axis to
//                 the power of two n, unnormalised forward transform, n/2+1 bins
//   irfft(X, n) = numpy.fft.irfft(X, n): bins beyond the input are zero, the
//                 imaginary parts of bins 0 and n/2 are ignored, 1/n scaling
//   fft_conv1d  = irfft(rfft(x, n) * rfft(h, n), n)[..., :L]
// The reference runs log2(n) radix-2 passes through global memory per
// transform.  Here one CTA owns one row: the real signal of length n is packed
// as a complex signal of length N = n/2 (z[m] = x[2m] + i x[2m+1]) held in
// shared memory, transformed with in-place Stockham passes (radix-16
// butterflies in registers, twiddles from a two-level table of N-th roots in
// shared memory), and unpacked into the n/2+1 real-FFT bins.  The fused
// convolution multiplies by the filter spectrum, re-packs for the inverse and
// runs the inverse passes without the spectrum ever leaving the SM: HBM sees
// one read of x, one read of H (L2-resident, shared by the batch) and one
// write of y.
//
// Rows longer than n = 32768 (N > 16384 complex values, beyond one CTA's
// shared memory) use the same algorithm with radix-2 Stockham passes through
// global scratch.
#include "common.cuh"
#include "tc_gemm.cuh"  // mbarrier helpers (bounded waits)

#include <cstring>

extern "C" int wxx_malloc(void** out, uint64_t nbytes);
extern "C" int wxx_free(void* p);

namespace {

// ------------------------------------------------------------ complex helpers

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

// Shared-memory index with one pad slot per 32 elements (breaks the
// power-of-two strides of the first Stockham pass into distinct banks).
// Shared-memory padding: one spare slot after every 16 values.  Every access
// pattern of a pass (16 consecutive indices per half-warp on load; 17j + r
// or consecutive indices on store) then takes the minimum two wavefronts per
// warp, and because the pass strides are multiples of 16, pad(i + c*16m) =
// pad(i) + c*17m: each thread computes one base and uses constant offsets.
__device__ __forceinline__ int swz(int i) { return i + (i >> 4); }

__host__ __device__ constexpr int bitrev_c(int i, int bits) {
  int r = 0;
  for (int b = 0; b < bits; ++b) r |= ((i >> b) & 1) << (bits - 1 - b);
  return r;
}

__host__ __device__ constexpr int log2_c(int r) { return r <= 1 ? 0 : 1 + log2_c(r >> 1); }

// e^{-2 pi i q / 16} for q = 0..7 (the roots a radix-16 butterfly needs).
__host__ __device__ constexpr float cos16(int q) {
  return q == 0 ? 1.0f
       : q == 1 ? 0.92387953251128674f
       : q == 2 ? 0.70710678118654752f
       : q == 3 ? 0.38268343236508978f
       : q == 4 ? 0.0f
       : q == 5 ? -0.38268343236508978f
       : q == 6 ? -0.70710678118654752f
                : -0.92387953251128674f;
}
__host__ __device__ constexpr float sin16(int q) {
  return q == 0 ? 0.0f
       : q == 1 ? 0.38268343236508978f
       : q == 2 ? 0.70710678118654752f
       : q == 3 ? 0.92387953251128674f
       : q == 4 ? 1.0f
       : q == 5 ? 0.92387953251128674f
       : q == 6 ? 0.70710678118654752f
                : 0.38268343236508978f;
}

// Multiplies b by e^{-+2 pi i q/16} (forward: minus), special-casing 1 and -+i.
template <bool INV>
__device__ __forceinline__ float2 rot16(float2 b, int q) {
  if (q == 0) return b;
  if (q == 4) return INV ? make_float2(-b.y, b.x) : make_float2(b.y, -b.x);
  float c = cos16(q), s = INV ? sin16(q) : -sin16(q);
  return make_float2(b.x * c - b.y * s, b.x * s + b.y * c);
}

// e^{-2 pi i q / 32} = cos32(q) - i sin32(q), q = 0..15 (written out like
// cos16 / sin16 so that every use folds to constants).
__host__ __device__ constexpr float cos32(int q) {
  return q == 0 ? 1.0f
       : q == 1 ? 0.98078528040323043f
       : q == 2 ? 0.92387953251128674f
       : q == 3 ? 0.83146961230254524f
       : q == 4 ? 0.70710678118654757f
       : q == 5 ? 0.55557023301960229f
       : q == 6 ? 0.38268343236508984f
       : q == 7 ? 0.19509032201612833f
       : q == 8 ? 6.123233995736766e-17f
       : q == 9 ? -0.19509032201612819f
       : q == 10 ? -0.38268343236508973f
       : q == 11 ? -0.55557023301960196f
       : q == 12 ? -0.70710678118654746f
       : q == 13 ? -0.83146961230254535f
       : q == 14 ? -0.92387953251128674f
                 : -0.98078528040323043f;
}
__host__ __device__ constexpr float sin32(int q) {
  return q == 0 ? 0.0f
       : q == 1 ? 0.19509032201612825f
       : q == 2 ? 0.38268343236508978f
       : q == 3 ? 0.55557023301960218f
       : q == 4 ? 0.70710678118654746f
       : q == 5 ? 0.83146961230254524f
       : q == 6 ? 0.92387953251128674f
       : q == 7 ? 0.98078528040323043f
       : q == 8 ? 1.0f
       : q == 9 ? 0.98078528040323043f
       : q == 10 ? 0.92387953251128674f
       : q == 11 ? 0.83146961230254546f
       : q == 12 ? 0.70710678118654757f
       : q == 13 ? 0.55557023301960218f
       : q == 14 ? 0.38268343236508989f
                 : 0.19509032201612861f;
}

// Multiplies b by e^{-+2 pi i q/32}, q < 16, special-casing 1 and -+i.
template <bool INV>
__device__ __forceinline__ float2 rot32(float2 b, int q) {
  if (q == 0) return b;
  if (q == 8) return INV ? make_float2(-b.y, b.x) : make_float2(b.y, -b.x);
  float c = cos32(q), s = INV ? sin32(q) : -sin32(q);
  return make_float2(b.x * c - b.y * s, b.x * s + b.y * c);
}

template <int R, bool INV>
__device__ __forceinline__ void reg_fft(float2 (&v)[R]);

// 32-point DFT as two 16-point DFTs (even / odd samples) and one combine
// stage: X[k] = E[k] + w^k O[k], X[k + 16] = E[k] - w^k O[k], w = e^{-2 pi i/32}.
template <bool INV>
__device__ __forceinline__ void reg_fft32(float2 (&v)[32]) {
  float2 e[16], o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    e[i] = v[2 * i];
    o[i] = v[2 * i + 1];
  }
  reg_fft<16, INV>(e);
  reg_fft<16, INV>(o);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float2 b = rot32<INV>(o[k], k);
    v[k] = cadd(e[k], b);
    v[k + 16] = csub(e[k], b);
  }
}

// In-register radix-R DFT (R <= 32), natural order in and out.
template <int R, bool INV>
__device__ __forceinline__ void reg_fft(float2 (&v)[R]) {
  if constexpr (R == 32) {
    reg_fft32<INV>(v);
    return;
  }
  constexpr int BITS = log2_c(R);
  float2 t[R];
#pragma unroll
  for (int i = 0; i < R; ++i) t[bitrev_c(i, BITS)] = v[i];
#pragma unroll
  for (int m = 2; m <= R; m <<= 1) {
#pragma unroll
    for (int k = 0; k < R; k += m) {
#pragma unroll
      for (int j = 0; j < m / 2; ++j) {
        float2 a = t[k + j];
        float2 b = R <= 16 ? rot16<INV>(t[k + j + m / 2], j * (16 / m))
                           : rot32<INV>(t[k + j + m / 2], j * (32 / m));
        t[k + j] = cadd(a, b);
        t[k + j + m / 2] = csub(a, b);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) v[i] = t[i];
}

// ------------------------------------------------------------ twiddle tables
//
// One table per transform size N = 2^L complex values (L <= kMaxSmemLogN),
// filled once per device (wxx::fft_init_tables, at wxx_init) in double
// precision:
//   for each pass in order (radix R, sub-transform size NS before it):
//     (R - 1) * NS entries  w[(r - 1) * NS + k] = exp(-2 pi i r k / (R NS))
//   then N/2 + 1 entries    u[k] = exp(-i pi k / N)   (real-FFT unpack / pack)
// Stored [r - 1][k], so a warp's twiddle loads (consecutive k) are contiguous.

constexpr int kMaxSmemLogN = 14;  // N = 16384 complex values per CTA

// Radix of the pass that follows sub-transforms of size ns in an n-point
// transform (n = 2^L): radix-16 passes, then either one radix-32 pass
// (L = 1 mod 4), two (L = 2 mod 4, L >= 10) or a final radix 2/4/8 -- the
// larger radices come last, where every store stride is a multiple of 16.
__host__ __device__ constexpr int pass_radix(int n, int ns) {
  const int L = log2_c(n), done = log2_c(ns);
  const int tail32 = (L >= 10 && L % 4 == 2) ? 2 : ((L >= 5 && L % 4 == 1) ? 1 : 0);
  const int head = L - 5 * tail32;
  if (done < head) return head - done >= 4 ? 16 : (1 << (head - done));
  return 32;
}

__host__ __device__ constexpr int tw_passes_size(int n) {
  int total = 0;
  for (int ns = 1; ns < n; ns *= pass_radix(n, ns)) total += (pass_radix(n, ns) - 1) * ns;
  return total;
}

__host__ __device__ constexpr int tw_size(int l) { return tw_passes_size(1 << l) + (1 << l) / 2 + 1; }

__host__ __device__ constexpr int tw_offset(int l) {
  int o = 0;
  for (int i = 0; i < l; ++i) o += tw_size(i);
  return o;
}

constexpr int kTwTotal = tw_offset(kMaxSmemLogN + 1);
static __device__ float2 g_fft_tw[kTwTotal];

__global__ void fft_twiddle_init_kernel() {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < kTwTotal; e += gridDim.x * blockDim.x) {
    int l = 0;
    while (l < kMaxSmemLogN && e >= tw_offset(l + 1)) ++l;
    int local = e - tw_offset(l);
    const int n = 1 << l;
    double angle = 0.0;   // in units of pi
    bool done = false;
    for (int ns = 1; ns < n && !done; ns *= pass_radix(n, ns)) {
      const int r = pass_radix(n, ns);
      const int seg = (r - 1) * ns;
      if (local < seg) {
        const int rr = local / ns + 1, k = local % ns;
        angle = -2.0 * (double)rr * (double)k / ((double)r * (double)ns);
        done = true;
      } else {
        local -= seg;
      }
    }
    if (!done) angle = -(double)local / (double)n;
    double sn, cs;
    sincospi(angle, &sn, &cs);
    g_fft_tw[e] = make_float2((float)cs, (float)sn);
  }
}

// One in-place Stockham pass of radix R over N values whose sub-transforms
// so far have size NS (compile-time, so every stride is a constant).
// Butterfly j loads buf[j + r*N/R], multiplies by w[(r-1)*NS + j mod NS],
// runs the radix-R DFT in registers and stores to
// (j - j mod NS) * R + j mod NS + r*NS.  All loads finish (barrier) before any
// store, so a single buffer suffices.
template <int N, int R, int NS, int T, bool INV>
__device__ __forceinline__ void fft_pass(float2* buf, const float2* __restrict__ tw) {
  constexpr int NB = N / R;
  constexpr int PER = (NB + T - 1) / T;
  // Constant-offset forms (see swz): loads stride NB, stores stride NS.
  constexpr bool LOAD_LIN = NB % 16 == 0;
  // NS == 1 with R = 16 or 32: d = R j is a multiple of 16, so
  // pad(d + r) = pad(d) + r + r / 16.
  constexpr bool STORE_LIN = NS % 16 == 0 || (NS == 1 && (R == 16 || R == 32));
  float2 v[PER][R];
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int j = threadIdx.x + p * T;
    if (NB % T == 0 || j < NB) {
      if constexpr (LOAD_LIN) {
        const float2* lb = buf + swz(j);
#pragma unroll
        for (int r = 0; r < R; ++r) v[p][r] = lb[r * (NB / 16 * 17)];
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) v[p][r] = buf[swz(j + r * NB)];
      }
      if (NS > 1) {
        const int k = j & (NS - 1);
        const float2* tb = tw + k;
#pragma unroll
        for (int r = 1; r < R; ++r) {
          float2 w = __ldg(tb + (r - 1) * NS);
          if (INV) w.y = -w.y;
          v[p][r] = cmul(v[p][r], w);
        }
      }
      reg_fft<R, INV>(v[p]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int j = threadIdx.x + p * T;
    if (NB % T == 0 || j < NB) {
      const int k = j & (NS - 1);
      const int d = (j - k) * R + k;
      if constexpr (STORE_LIN) {
        float2* sb = buf + swz(d);
#pragma unroll
        for (int r = 0; r < R; ++r) sb[NS == 1 ? r + (r >> 4) : r * (NS / 16 * 17)] = v[p][r];
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) buf[swz(d + r * NS)] = v[p][r];
      }
    }
  }
  __syncthreads();
}

// All passes of an N-point transform: radix 16 while it fits, then one pass
// of the remaining radix; the table pointer advances pass by pass.
template <int N, int T, bool INV, int NS = 1>
__device__ __forceinline__ void fft_passes(float2* buf, const float2* __restrict__ tw) {
  if constexpr (NS < N) {
    constexpr int R = pass_radix(N, NS);
    fft_pass<N, R, NS, T, INV>(buf, tw);
    fft_passes<N, T, INV, NS * R>(buf, tw + (R - 1) * NS);
  }
}

// ------------------------------------------------------------ row kernels

struct RowArgs {
  // real input rows (modes 0, 2): element t of row (b, d) at
  //   in[in_off + b*in_sb + d*in_sd + t*in_st], t < in_len (zero beyond)
  const float* in;
  int64_t in_off, in_sb, in_sd, in_st;
  int in_len;
  // spectrum input (mode 1): row r at spec_in[r*spec_ld], spec_len bins
  const float2* spec_in;
  int64_t spec_ld;
  int spec_len;
  // filter spectrum (mode 2): channel d at H[d*h_ld], N+1 bins
  const float2* H;
  int64_t h_ld;
  // outputs: mode 0 -> spec_out[row*out_ld + k], k <= N
  //          modes 1, 2 -> out[row*out_ld + t], t < out_len
  float2* spec_out;
  float* out;
  int64_t out_ld;
  int out_len;
  int rows_b, rows_d;  // row (b, d) -> output row b*rows_d + d
  // optional gate (conv mode): y[b, d, t] *= gate[g_off + b*g_sb + d*g_sd + t*g_st]
  const float* gate;
  int64_t g_off, g_sb, g_sd, g_st;
};

constexpr int kModeRfft = 0;
constexpr int kModeIrfft = 1;
constexpr int kModeConv = 2;

template <int LOGN>
struct RowCfg {
  static constexpr int N = 1 << LOGN;
  // One radix-16 butterfly per thread (radix-32 passes leave half of them
  // idle): holding two across a pass's barrier sends one to local memory.
  static constexpr int TB = N / 16;
  static constexpr int T = TB < 64 ? 64 : (TB > 512 ? 512 : TB);
  static constexpr int SMEM = (N + N / 16 + 1) * 8;
  static constexpr int MINB = T >= 512 ? 1 : 2;
};

// Unpacks Z (FFT of the packed real signal) into the real-FFT bins X[k] and
// X[N-k] for k in [0, N/2] (thread-owned pairs).
// exp(-i pi k / N) computed directly (global-memory path, N beyond the tables).
__device__ __forceinline__ float2 unpack_twiddle(int k, int N) {
  float s, c;
  sincospif(-(float)k / (float)N, &s, &c);
  return make_float2(c, s);
}

// u = exp(-i pi k / N) from the table.
__device__ __forceinline__ void rfft_unpack_pair(float2 zk, float2 znk, float2 u, float2& xk,
                                                 float2& xnk) {
  float2 bc = cconj(znk);
  float2 fe = cscale(cadd(zk, bc), 0.5f);
  float2 d = csub(zk, bc);
  float2 fo = make_float2(0.5f * d.y, -0.5f * d.x);  // (zk - bc) / (2i)
  float2 wf = cmul(u, fo);
  xk = cadd(fe, wf);
  xnk = cconj(csub(fe, wf));
}

// Packs the Hermitian spectrum pair (Y[k], Y[N-k]) into Z'[k], Z'[N-k] of the
// length-N complex signal whose inverse FFT interleaves the real output.
// u = exp(-i pi k / N) from the table (conj(u) is applied).
__device__ __forceinline__ void irfft_pack_pair(float2 yk, float2 ynk, float2 u, float2& zk,
                                                float2& znk) {
  float2 bc = cconj(ynk);
  float2 fe = cscale(cadd(yk, bc), 0.5f);
  float2 d = cscale(csub(yk, bc), 0.5f);
  float2 fo = cmul(cconj(u), d);
  zk = make_float2(fe.x - fo.y, fe.y + fo.x);     // fe + i fo
  znk = make_float2(fe.x + fo.y, -fe.y + fo.x);   // conj(fe) + i conj(fo)
}

// One CTA per row.  The inverse transform is evaluated as
// IFFT(z) = conj(FFT(conj(z))) / N: the packed spectrum is stored conjugated
// and the output conjugated back, so a single (forward) instance of the
// passes serves both directions (one copy of the unrolled code, which keeps
// the conv kernel free of register spills).
template <int LOGN, int MODE>
__global__ void __launch_bounds__(RowCfg<LOGN>::T, RowCfg<LOGN>::MINB)
    fft_row_kernel(RowArgs a) {
  using C = RowCfg<LOGN>;
  constexpr int N = C::N;
  constexpr int T = C::T;
  extern __shared__ float2 buf[];
  const float2* tw = g_fft_tw + tw_offset(LOGN);
  const float2* utw = tw + tw_passes_size(N);   // exp(-i pi k / N), k <= N/2
  const int tid = threadIdx.x;

  int d = blockIdx.x / a.rows_b;
  int b = blockIdx.x - d * a.rows_b;
  int64_t row = (int64_t)b * a.rows_d + d;

  if (MODE != kModeIrfft) {
    // z[m] = x[2m] + i x[2m+1], zero-padded / truncated to N
    const float* x = a.in + a.in_off + (int64_t)b * a.in_sb + (int64_t)d * a.in_sd;
    const int len = a.in_len;
    const bool vec = a.in_st == 1 && ((reinterpret_cast<uintptr_t>(x) & 7) == 0);
    for (int m = tid; m < N; m += T) {
      int t0 = 2 * m;
      float2 z = make_float2(0.f, 0.f);
      if (t0 + 1 < len) {
        if (vec) z = *reinterpret_cast<const float2*>(x + t0);
        else z = make_float2(x[(int64_t)t0 * a.in_st], x[(int64_t)(t0 + 1) * a.in_st]);
      } else if (t0 < len) {
        z.x = x[(int64_t)t0 * a.in_st];
      }
      buf[swz(m)] = z;
    }
  } else {
    // conj of the packed spectrum Z'[k] (bins beyond the input are zero)
    const float2* Y = a.spec_in + row * a.spec_ld;
    const int len = a.spec_len;
    for (int k = tid; k <= N / 2; k += T) {
      float2 yk = k < len ? Y[k] : make_float2(0.f, 0.f);
      float2 ynk = (N - k) < len ? Y[N - k] : make_float2(0.f, 0.f);
      if (k == 0) {
        float y0 = yk.x, yn = ynk.x;  // imaginary parts of bins 0 and N are ignored
        buf[swz(0)] = make_float2(0.5f * (y0 + yn), -0.5f * (y0 - yn));
      } else {
        float2 pk, pnk;
        irfft_pack_pair(yk, ynk, __ldg(utw + k), pk, pnk);
        buf[swz(k)] = cconj(pk);
        if (k != N - k) buf[swz(N - k)] = cconj(pnk);
      }
    }
  }
  __syncthreads();

#pragma unroll 1
  for (int phase = (MODE == kModeIrfft) ? 1 : 0; phase < 2; ++phase) {
    fft_passes<N, T, false>(buf, tw);
    if (phase == 1) break;
    if (MODE == kModeRfft) {
      float2* X = a.spec_out + row * a.out_ld;
      for (int k = tid; k <= N / 2; k += T) {
        float2 zk = buf[swz(k)];
        if (k == 0) {
          X[0] = make_float2(zk.x + zk.y, 0.f);
          X[N] = make_float2(zk.x - zk.y, 0.f);
        } else {
          float2 xk, xnk;
          rfft_unpack_pair(zk, buf[swz(N - k)], __ldg(utw + k), xk, xnk);
          X[k] = xk;
          if (k != N - k) X[N - k] = xnk;
        }
      }
      return;
    }
    // Fused convolution: Y = X * H, packed (conjugated) for the inverse.
    const float2* H = a.H + (int64_t)d * a.h_ld;
    for (int k = tid; k <= N / 2; k += T) {
      float2 zk = buf[swz(k)];
      if (k == 0) {
        float y0 = (zk.x + zk.y) * H[0].x;   // bins 0 and N are real
        float yn = (zk.x - zk.y) * H[N].x;
        buf[swz(0)] = make_float2(0.5f * (y0 + yn), -0.5f * (y0 - yn));
      } else {
        const float2 u = __ldg(utw + k);
        float2 xk, xnk;
        rfft_unpack_pair(zk, buf[swz(N - k)], u, xk, xnk);
        float2 pk, pnk;
        irfft_pack_pair(cmul(xk, H[k]), cmul(xnk, H[N - k]), u, pk, pnk);
        buf[swz(k)] = cconj(pk);
        if (k != N - k) buf[swz(N - k)] = cconj(pnk);
      }
    }
    __syncthreads();
  }

  // y[2m] + i y[2m+1] = conj(FFT(conj Z'))[m] / N
  float* y = a.out + row * a.out_ld;
  const float scale = 1.0f / (float)N;
  const int olen = a.out_len;
  const bool vec = ((reinterpret_cast<uintptr_t>(y) & 7) == 0);
  const float* g = a.gate == nullptr
                       ? nullptr
                       : a.gate + a.g_off + (int64_t)b * a.g_sb + (int64_t)d * a.g_sd;
  for (int m = tid; m < N; m += T) {
    int t0 = 2 * m;
    if (t0 >= olen) break;
    const float2 w = buf[swz(m)];
    float2 z = make_float2(w.x * scale, -w.y * scale);
    if (g != nullptr) {
      z.x *= g[(int64_t)t0 * a.g_st];
      if (t0 + 1 < olen) z.y *= g[(int64_t)(t0 + 1) * a.g_st];
    }
    if (t0 + 1 < olen) {
      if (vec) *reinterpret_cast<float2*>(y + t0) = z;
      else { y[t0] = z.x; y[t0 + 1] = z.y; }
    } else {
      y[t0] = z.x;
    }
  }
}

// n == 1: rfft(x)[0] = x[0]; irfft(X)[0] = Re X[0]; conv = x[0] * Re H[0].
__global__ void fft_n1_kernel(RowArgs a, int mode, int64_t rows) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows;
       i += (int64_t)gridDim.x * blockDim.x) {
    int d = (int)(i / a.rows_b), b = (int)(i - (int64_t)d * a.rows_b);
    int64_t row = (int64_t)b * a.rows_d + d;
    if (mode == kModeIrfft) {
      float v = a.spec_len > 0 ? a.spec_in[row * a.spec_ld].x : 0.f;
      if (a.out_len > 0) a.out[row * a.out_ld] = v;
      continue;
    }
    float x0 = a.in_len > 0 ? a.in[a.in_off + (int64_t)b * a.in_sb + (int64_t)d * a.in_sd] : 0.f;
    if (mode == kModeRfft) a.spec_out[row * a.out_ld] = make_float2(x0, 0.f);
    else if (a.out_len > 0)
      a.out[row * a.out_ld] =
          x0 * a.H[(int64_t)d * a.h_ld].x *
          (a.gate != nullptr ? a.gate[a.g_off + (int64_t)b * a.g_sb + (int64_t)d * a.g_sd] : 1.f);
  }
}

// ------------------------------------------------------------ global fallback (N > 16384)

// z[row][m] = (x[2m], x[2m+1]) with zero padding.
__global__ void pack_real_kernel(float2* __restrict__ z, RowArgs a, int N, int64_t rows) {
  int64_t total = rows * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / N;
    int m = (int)(i - r * N);
    int d = (int)(r / a.rows_b), b = (int)(r - (int64_t)d * a.rows_b);
    const float* x = a.in + a.in_off + (int64_t)b * a.in_sb + (int64_t)d * a.in_sd;
    int t0 = 2 * m;
    float2 v = make_float2(0.f, 0.f);
    if (t0 < a.in_len) v.x = x[(int64_t)t0 * a.in_st];
    if (t0 + 1 < a.in_len) v.y = x[(int64_t)(t0 + 1) * a.in_st];
    z[(int64_t)(b * a.rows_d + d) * N + m] = v;
  }
}

// One radix-2 Stockham pass over every row: dst[(j-k)*2 + k + r*Ns] from src[j + r*N/2].
__global__ void stockham2_global_kernel(float2* __restrict__ dst, const float2* __restrict__ src,
                                        int N, int Ns, int64_t rows, int inv) {
  int half = N / 2;
  int64_t total = rows * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / half;
    int j = (int)(i - r * half);
    const float2* s = src + r * N;
    float2* o = dst + r * N;
    float2 v0 = s[j], v1 = s[j + half];
    int k = j & (Ns - 1);
    if (Ns > 1) {
      float sn, cs;
      sincospif((inv ? 1.0f : -1.0f) * (float)k / (float)Ns, &sn, &cs);
      v1 = cmul(v1, make_float2(cs, sn));
    }
    int dd = (j - k) * 2 + k;
    o[dd] = cadd(v0, v1);
    o[dd + Ns] = csub(v0, v1);
  }
}

// Real-FFT unpack (mode 0) or unpack * H * repack (mode 2), one thread per pair.
__global__ void unpack_global_kernel(float2* __restrict__ z, RowArgs a, int N, int64_t rows,
                                     int mode) {
  int pairs = N / 2 + 1;
  int64_t total = rows * pairs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / pairs;
    int k = (int)(i - r * pairs);
    int d = (int)(r / a.rows_b), b = (int)(r - (int64_t)d * a.rows_b);
    int64_t row = (int64_t)b * a.rows_d + d;
    float2* zr = z + row * N;
    float2 zk = zr[k];
    if (mode == kModeRfft) {
      float2* X = a.spec_out + row * a.out_ld;
      if (k == 0) {
        X[0] = make_float2(zk.x + zk.y, 0.f);
        X[N] = make_float2(zk.x - zk.y, 0.f);
      } else {
        float2 xk, xnk;
        rfft_unpack_pair(zk, zr[N - k], unpack_twiddle(k, N), xk, xnk);
        X[k] = xk;
        if (k != N - k) X[N - k] = xnk;
      }
    } else {
      const float2* H = a.H + (int64_t)d * a.h_ld;
      if (k == 0) {
        float y0 = (zk.x + zk.y) * H[0].x, yn = (zk.x - zk.y) * H[N].x;
        zr[0] = make_float2(0.5f * (y0 + yn), 0.5f * (y0 - yn));
      } else {
        float2 xk, xnk, pk, pnk;
        rfft_unpack_pair(zk, zr[N - k], unpack_twiddle(k, N), xk, xnk);
        irfft_pack_pair(cmul(xk, H[k]), cmul(xnk, H[N - k]), unpack_twiddle(k, N), pk, pnk);
        zr[k] = pk;
        if (k != N - k) zr[N - k] = pnk;
      }
    }
  }
}

__global__ void pack_spectrum_global_kernel(float2* __restrict__ z, RowArgs a, int N,
                                            int64_t rows) {
  int pairs = N / 2 + 1;
  int64_t total = rows * pairs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = i / pairs;
    int k = (int)(i - row * pairs);
    const float2* Y = a.spec_in + row * a.spec_ld;
    float2 yk = k < a.spec_len ? Y[k] : make_float2(0.f, 0.f);
    float2 ynk = (N - k) < a.spec_len ? Y[N - k] : make_float2(0.f, 0.f);
    float2* zr = z + row * N;
    if (k == 0) {
      zr[0] = make_float2(0.5f * (yk.x + ynk.x), 0.5f * (yk.x - ynk.x));
    } else {
      float2 pk, pnk;
      irfft_pack_pair(yk, ynk, unpack_twiddle(k, N), pk, pnk);
      zr[k] = pk;
      if (k != N - k) zr[N - k] = pnk;
    }
  }
}

__global__ void unpack_real_global_kernel(const float2* __restrict__ z, RowArgs a, int N,
                                          int64_t rows) {
  int64_t total = rows * N;
  float scale = 1.0f / (float)N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = i / N;
    int m = (int)(i - row * N);
    int t0 = 2 * m;
    if (t0 >= a.out_len) continue;
    float2 v = cscale(z[row * N + m], scale);
    if (a.gate != nullptr) {
      const int b = (int)(row / a.rows_d), d = (int)(row - (int64_t)b * a.rows_d);
      const float* g = a.gate + a.g_off + (int64_t)b * a.g_sb + (int64_t)d * a.g_sd;
      v.x *= g[(int64_t)t0 * a.g_st];
      if (t0 + 1 < a.out_len) v.y *= g[(int64_t)(t0 + 1) * a.g_st];
    }
    float* y = a.out + row * a.out_ld;
    y[t0] = v.x;
    if (t0 + 1 < a.out_len) y[t0 + 1] = v.y;
  }
}

// ------------------------------------------------------------ planar pair kernels (N >= 256)
//
// The production path for N = 256 .. 16384 complex values per row.  Every
// thread carries two butterflies, one per lane of Blackwell's paired FP32
// instructions (add/sub/mul/fma .f32x2): a CP holds the real parts of two
// complex values in one 64-bit register pair and their imaginary parts in
// another, so one paired instruction does the arithmetic of both butterflies.
// The row sits in shared memory as two planar float arrays (re, im), padded
// (pad3), so the two lanes of a pair are adjacent and 8-byte aligned and
// every pass moves them with 64-bit accesses.
//
// Per fused convolution the shared-memory traffic is cut three ways:
//  * the first forward pass reads x straight from global memory;
//  * the last forward pass, the spectrum product and the first inverse pass
//    run in registers: that pass pairs butterfly j with its mirror N/R - j,
//    whose outputs are exactly the bins N - k the real-FFT unpack needs, and
//    the first inverse pass (stride N/R, like the last forward pass) reads
//    the same elements the thread already holds;
//  * the last inverse pass writes y straight to global memory.
// A micro-benchmark of one 8192-point radix-16 pass: 2.65 us per SM with the
// float2 butterflies (~900 issued instructions per butterfly, mostly integer
// moves), 0.65 us with the paired form (~125), which is ~80 % of the
// shared-memory bandwidth.

typedef unsigned long long u64;

__device__ __forceinline__ u64 p_add(u64 a, u64 b) {
  u64 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 p_sub(u64 a, u64 b) {
  u64 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 p_mul(u64 a, u64 b) {
  u64 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 p_fma(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ u64 p_make(float lo, float hi) {
  return ((u64)__float_as_uint(hi) << 32) | (u64)__float_as_uint(lo);
}
__device__ __forceinline__ float p_lo(u64 a) { return __uint_as_float((unsigned)a); }
__device__ __forceinline__ float p_hi(u64 a) { return __uint_as_float((unsigned)(a >> 32)); }

struct CP {
  u64 re, im;
};

__device__ __forceinline__ float2 cp_get(const CP& v, int lane) {
  return lane == 0 ? make_float2(p_lo(v.re), p_lo(v.im)) : make_float2(p_hi(v.re), p_hi(v.im));
}
__device__ __forceinline__ void cp_set(CP& v, int lane, float2 z) {
  if (lane == 0) {
    v.re = p_make(z.x, p_hi(v.re));
    v.im = p_make(z.y, p_hi(v.im));
  } else {
    v.re = p_make(p_lo(v.re), z.x);
    v.im = p_make(p_lo(v.im), z.y);
  }
}

// v <- v * exp(-i theta) for lane-wise (cos theta, sin theta) = (c, s).
__device__ __forceinline__ void p_twiddle(CP& v, u64 c, u64 s) {
  const u64 re = p_fma(v.re, c, p_mul(v.im, s));
  v.im = p_sub(p_mul(v.im, c), p_mul(v.re, s));
  v.re = re;
}

// a, b <- a + w b, a - w b with w = exp(-2 pi i Q / R), R <= 32.
template <int R, int Q>
__device__ __forceinline__ void p_bfly(CP& a, CP& b) {
  constexpr int q32 = Q * (32 / R);
  CP s, d;
  if constexpr (q32 == 0) {
    s = CP{p_add(a.re, b.re), p_add(a.im, b.im)};
    d = CP{p_sub(a.re, b.re), p_sub(a.im, b.im)};
  } else if constexpr (q32 == 8) {  // w = -i: w b = (b.im, -b.re)
    s = CP{p_add(a.re, b.im), p_sub(a.im, b.re)};
    d = CP{p_sub(a.re, b.im), p_add(a.im, b.re)};
  } else {
    // w b = (re c + im s) + i (im c - re s), (c, s) = (cos, sin)(2 pi Q / R)
    constexpr float c = cos32(q32), sn = sin32(q32);
    const u64 C = p_make(c, c), S = p_make(sn, sn), NS = p_make(-sn, -sn);
    const u64 wr = p_fma(b.re, C, p_mul(b.im, S));
    const u64 wi = p_fma(b.im, C, p_mul(b.re, NS));
    s = CP{p_add(a.re, wr), p_add(a.im, wi)};
    d = CP{p_sub(a.re, wr), p_sub(a.im, wi)};
  }
  a = s;
  b = d;
}

template <int R, int M, int K, int J>
__device__ __forceinline__ void p_stage(CP (&t)[R]) {
  if constexpr (K < R) {
    if constexpr (J < M / 2) {
      p_bfly<R, J * (R / M)>(t[K + J], t[K + J + M / 2]);
      p_stage<R, M, K, J + 1>(t);
    } else {
      p_stage<R, M, K + M, 0>(t);
    }
  }
}

template <int R, int M = 2>
__device__ __forceinline__ void p_stages(CP (&t)[R]) {
  if constexpr (M <= R) {
    p_stage<R, M, 0, 0>(t);
    p_stages<R, M * 2>(t);
  }
}

// Radix-R forward DFT of both lanes, natural order in and out.
template <int R>
__device__ __forceinline__ void p_dft(CP (&v)[R]) {
  CP t[R];
#pragma unroll
  for (int i = 0; i < R; ++i) t[bitrev_c(i, log2_c(R))] = v[i];
  p_stages<R>(t);
#pragma unroll
  for (int i = 0; i < R; ++i) v[i] = t[i];
}

// Shared-memory index of element i of a planar row: two spare floats every 32
// and sixteen more every 512.  The two lanes of a pair stay adjacent and
// 8-byte aligned, and the 64-bit store patterns of a half-warp in every pass
// of the plans below (groups of 8 pairs, 256 or 512 elements apart in the
// radix-16 and radix-32 passes) fall on 32 distinct banks.
__device__ __forceinline__ int pad3(int i) { return i + ((i >> 5) << 1) + ((i >> 9) << 4); }
// pad3 for compile-time arguments.  Address identities used by the passes
// (all sizes powers of two):
//   pad3(j + r*NB) = pad3(j) + pad3c(r*NB)   for j < NB, NB >= 32;
//   pad3(X + Y)    = pad3(X) + pad3(Y)       for X a multiple of 512;
//   pad3(k + r*NS) = k + pad3c(r*NS)         for k < NS <= 16;
//   pad3(b + r)    = pad3(b) + r             for b a multiple of 2R', r < R' <= 32, r + b % 32 < 32;
// so a thread computes one base per pass and every access adds a constant.
__host__ __device__ constexpr int pad3c(int i) { return i + ((i >> 5) << 1) + ((i >> 9) << 4); }
__host__ __device__ constexpr int padded3(int n) { return n + n / 16 + n / 32 + 32; }
__device__ __forceinline__ u64 lds2(const float* p) { return *reinterpret_cast<const u64*>(p); }
__device__ __forceinline__ void sts2(float* p, u64 v) { *reinterpret_cast<u64*>(p) = v; }
__device__ __forceinline__ u64 ldg2(const float* p) { return __ldg(reinterpret_cast<const u64*>(p)); }

__device__ __forceinline__ CP cp_mul(const CP& a, const CP& b) {
  return CP{p_sub(p_mul(a.re, b.re), p_mul(a.im, b.im)), p_fma(a.re, b.im, p_mul(a.im, b.re))};
}
__device__ __forceinline__ CP cp_sqr(const CP& a) {
  return CP{p_sub(p_mul(a.re, a.re), p_mul(a.im, a.im)), p_mul(p_add(a.re, a.re), a.im)};
}
// a * exp(-i pi Q / R) for a compile-time angle (R <= 16: a multiple of pi/16).
template <int R, int Q>
__device__ __forceinline__ CP cp_rot_half(const CP& a) {
  if constexpr (Q == 0) {
    return a;
  } else {
    constexpr int q32 = Q * (16 / R);   // exp(-i pi Q / R) = exp(-2 pi i q32 / 32)
    constexpr float c = cos32(q32), sn = sin32(q32);
    const u64 C = p_make(c, c), S = p_make(sn, sn);
    // (re + i im)(c - i sn)
    return CP{p_fma(a.re, C, p_mul(a.im, S)), p_sub(p_mul(a.im, C), p_mul(a.re, S))};
  }
}
__device__ __forceinline__ float f_sel(bool c, float a, float b) { return c ? a : b; }

struct PBuf {
  float* re;
  float* im;
};

// Pass plans for N = 2^L (L = 8..14), variant V = 0 (fft_pair_kernel) or
// V = 1 (the staged convolution at L = 13): forward radices first to last;
// the inverse runs them in reverse order.  L = 13, V = 0 has a radix-32
// middle pass, three passes each way at 256 threads (measured: 19.4k cycles
// per row against 21.5k with the radix-32 pass first); the staged kernel
// transforms in place, where a radix-32 pass would hold 128 registers across
// its barrier, so its radix-32 pass comes first (reading the staged input)
// and last (writing global memory).  L = 14 has 512 threads (128 registers
// each) and four passes; smaller rows a small first radix, then radix 16.
__host__ __device__ constexpr int pp_count(int L, int V = 0) {
  return L == 8 ? 2 : (L == 14 ? 4 : 3);
}
__host__ __device__ constexpr int pp_radix(int L, int V, int p) {
  return L == 13   ? (p == (V ? 0 : 1) ? 32 : 16)
         : L == 14 ? (p == 2 ? 4 : 16)
         : (p == 0 && (L - 8) % 4 != 0) ? (1 << ((L - 8) % 4))
                                         : 16;
}
// Sub-transform size before forward pass p / inverse pass q.
__host__ __device__ constexpr int pp_ns_fwd(int L, int V, int p) {
  int ns = 1;
  for (int i = 0; i < p; ++i) ns *= pp_radix(L, V, i);
  return ns;
}
__host__ __device__ constexpr int pp_radix_inv(int L, int V, int q) {
  return pp_radix(L, V, pp_count(L, V) - 1 - q);
}
__host__ __device__ constexpr int pp_ns_inv(int L, int V, int q) {
  int ns = 1;
  for (int i = 0; i < q; ++i) ns *= pp_radix_inv(L, V, i);
  return ns;
}

// Twiddle tables (floats), one block per plan (L = 8..14 with V = 0, then
// L = 13 with V = 1): the forward passes p = 1..P-1 then the inverse passes
// q = 1..P-1, each a segment of (R-1)*NS cosines followed by (R-1)*NS sines of
// 2 pi r k / (R NS), entry (r-1)*NS + k.
constexpr int kPairMinL = 8;
constexpr int kPlans = 8;
__host__ __device__ constexpr int plan_L(int i) { return i == 7 ? 13 : kPairMinL + i; }
__host__ __device__ constexpr int plan_V(int i) { return i == 7 ? 1 : 0; }
__host__ __device__ constexpr int plan_index(int L, int V) { return V ? 7 : L - kPairMinL; }
__host__ __device__ constexpr int pt_seg(int R, int NS) { return 2 * (R - 1) * NS; }
__host__ __device__ constexpr int pt_size(int L, int V) {
  int s = 0;
  for (int p = 1; p < pp_count(L, V); ++p) s += pt_seg(pp_radix(L, V, p), pp_ns_fwd(L, V, p));
  for (int q = 1; q < pp_count(L, V); ++q) s += pt_seg(pp_radix_inv(L, V, q), pp_ns_inv(L, V, q));
  return s;
}
__host__ __device__ constexpr int pt_base_i(int i) {
  int o = 0;
  for (int k = 0; k < i; ++k) o += pt_size(plan_L(k), plan_V(k));
  return o;
}
__host__ __device__ constexpr int pt_base(int L, int V) { return pt_base_i(plan_index(L, V)); }
__host__ __device__ constexpr int pt_fwd_off(int L, int V, int p) {
  int o = pt_base(L, V);
  for (int i = 1; i < p; ++i) o += pt_seg(pp_radix(L, V, i), pp_ns_fwd(L, V, i));
  return o;
}
__host__ __device__ constexpr int pt_inv_off(int L, int V, int q) {
  int o = pt_fwd_off(L, V, pp_count(L, V));
  for (int i = 1; i < q; ++i) o += pt_seg(pp_radix_inv(L, V, i), pp_ns_inv(L, V, i));
  return o;
}
constexpr int kPtTotal = pt_base_i(kPlans);
static __device__ __align__(16) float g_fft_ptw[kPtTotal];

__global__ void fft_pair_twiddle_init_kernel() {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < kPtTotal; e += gridDim.x * blockDim.x) {
    int i = 0;
    while (i + 1 < kPlans && e >= pt_base_i(i + 1)) ++i;
    const int L = plan_L(i), V = plan_V(i);
    int local = e - pt_base_i(i);
    const int P = pp_count(L, V);
    for (int s = 0; s < 2 * (P - 1); ++s) {
      const bool inv = s >= P - 1;
      const int idx = inv ? s - (P - 1) + 1 : s + 1;
      const int R = inv ? pp_radix_inv(L, V, idx) : pp_radix(L, V, idx);
      const int NS = inv ? pp_ns_inv(L, V, idx) : pp_ns_fwd(L, V, idx);
      const int seg = pt_seg(R, NS);
      if (local < seg) {
        const int half = (R - 1) * NS;
        const bool is_sin = local >= half;
        const int j = is_sin ? local - half : local;
        const int rr = j / NS + 1, k = j % NS;
        double sn, cs;
        sincospi(2.0 * (double)rr * (double)k / ((double)R * (double)NS), &sn, &cs);
        g_fft_ptw[e] = (float)(is_sin ? sn : cs);
        break;
      }
      local -= seg;
    }
  }
}

template <int L>
struct PCfg {
  static constexpr int N = 1 << L;
  static constexpr int P = pp_count(L, 0);
  static constexpr int T = N / 32 < 32 ? 32 : N / 32;
  static constexpr int BUF = 2 * padded3(N);  // floats of one planar row (re, then im)
  // Two row buffers where they fit: passes then run out of place, with one
  // barrier each and every thread storing as soon as its butterflies are done.
  static constexpr bool DB = 2 * BUF * 4 <= 200 * 1024;
  static constexpr int SMEM = (DB ? 2 : 1) * BUF * 4;
};

// Forward pass 0 (NS = 1) from the real input row: z[m] = x[2m] + i x[2m+1].
// Output r of butterfly j goes to j R + r; the two lanes' outputs r, r+1 are
// regrouped into one 64-bit store per lane.
template <int N, int R, int T, bool SMEMX = false>
__device__ __forceinline__ void pp_first(PBuf dst, const float* x, int64_t st, int len, bool vec) {
  constexpr int NB = N / R, PAIRS = NB / 2, PER = (PAIRS + T - 1) / T;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int q = threadIdx.x + p * T;
    if (PAIRS % T == 0 || q < PAIRS) {
      const int j = 2 * q;
      CP v[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int t0 = 2 * (j + r * NB);
        float4 xv;
        if (SMEMX) {
          // staged row: len floats, len % 4 == 0
          xv = t0 < len ? *reinterpret_cast<const float4*>(x + t0) : make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (vec && t0 + 3 < len) {
          xv = *reinterpret_cast<const float4*>(x + t0);
        } else {
          xv.x = t0 < len ? x[(int64_t)t0 * st] : 0.f;
          xv.y = t0 + 1 < len ? x[(int64_t)(t0 + 1) * st] : 0.f;
          xv.z = t0 + 2 < len ? x[(int64_t)(t0 + 2) * st] : 0.f;
          xv.w = t0 + 3 < len ? x[(int64_t)(t0 + 3) * st] : 0.f;
        }
        v[r].re = p_make(xv.x, xv.z);
        v[r].im = p_make(xv.y, xv.w);
      }
      p_dft<R>(v);
      // j even: j R and (j + 1) R are multiples of R with room for r < R
      // inside their 32-slot group, so pad3(base + r) = pad3(base) + r.
      const int b0 = pad3(j * R), b1 = pad3((j + 1) * R);
#pragma unroll
      for (int r = 0; r < R; r += 2) {
        sts2(dst.re + b0 + r, p_make(p_lo(v[r].re), p_lo(v[r + 1].re)));
        sts2(dst.im + b0 + r, p_make(p_lo(v[r].im), p_lo(v[r + 1].im)));
        sts2(dst.re + b1 + r, p_make(p_hi(v[r].re), p_hi(v[r + 1].re)));
        sts2(dst.im + b1 + r, p_make(p_hi(v[r].im), p_hi(v[r + 1].im)));
      }
    }
  }
  __syncthreads();
}

// Loads butterflies j, j+1 (j even) of a Stockham pass, applies the twiddles
// of k = j mod NS, k+1, and transforms them.
template <int N, int R, int NS>
__device__ __forceinline__ void pp_load_dft(CP (&v)[R], PBuf src, int j,
                                            const float* __restrict__ tw) {
  constexpr int NB = N / R;
  if constexpr (NB >= 32) {
    const int jb = pad3(j);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      v[r].re = lds2(src.re + jb + pad3c(r * NB));
      v[r].im = lds2(src.im + jb + pad3c(r * NB));
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      v[r].re = lds2(src.re + pad3(j + r * NB));
      v[r].im = lds2(src.im + pad3(j + r * NB));
    }
  }
  const int k = j & (NS - 1);
#pragma unroll
  for (int r = 1; r < R; ++r)
    p_twiddle(v[r], ldg2(tw + (r - 1) * NS + k), ldg2(tw + (R - 1 + r - 1) * NS + k));
  p_dft<R>(v);
}

template <int N, int R, int NS>
__device__ __forceinline__ void pp_store(const CP (&v)[R], PBuf dst, int j) {
  const int k = j & (NS - 1);
  const int d = (j - k) * R + k;
  if constexpr (NS * R >= 512 && (NS >= 32 || NS <= 16)) {
    // d = X + k with X a multiple of NS R (>= 512) and k < NS
    const int base = pad3(d - k) + (NS >= 32 ? pad3(k) : k);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      sts2(dst.re + base + pad3c(r * NS), v[r].re);
      sts2(dst.im + base + pad3c(r * NS), v[r].im);
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      sts2(dst.re + pad3(d + r * NS), v[r].re);
      sts2(dst.im + pad3(d + r * NS), v[r].im);
    }
  }
}

// One Stockham pass (NS >= 2), lanes = butterflies j, j+1.  In place (src ==
// dst) every load precedes a barrier and every store; out of place each
// thread stores its butterflies right after transforming them.
template <int N, int R, int NS, int T, bool INPLACE>
__device__ __forceinline__ void pp_pass(PBuf src, PBuf dst, const float* __restrict__ tw) {
  constexpr int NB = N / R, PAIRS = NB / 2, PER = (PAIRS + T - 1) / T;
  if constexpr (INPLACE) {
    CP v[PER][R];
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int q = threadIdx.x + p * T;
      if (PAIRS % T == 0 || q < PAIRS) pp_load_dft<N, R, NS>(v[p], src, 2 * q, tw);
    }
    __syncthreads();
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int q = threadIdx.x + p * T;
      if (PAIRS % T == 0 || q < PAIRS) pp_store<N, R, NS>(v[p], dst, 2 * q);
    }
  } else {
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int q = threadIdx.x + p * T;
      if (PAIRS % T == 0 || q < PAIRS) {
        CP v[R];
        pp_load_dft<N, R, NS>(v, src, 2 * q, tw);
        pp_store<N, R, NS>(v, dst, 2 * q);
      }
    }
  }
  __syncthreads();
}

// The mirror step on two bin pairs at once, one per lane: zk = (Z[k0], Z[k1])
// and znk = (Z[N-k0], Z[N-k1]) of the packed forward transform, u =
// exp(-i pi k / N) per lane.  Out: the conj of the packed inverse input at
// the same places (conv: after the product with the filter spectrum H; irfft:
// made from the input spectrum, z unused), or the spectrum bins written to
// global memory (rfft).  The algebra of rfft_unpack_pair / irfft_pack_pair,
// written out on paired registers.
template <typename Ld>
__device__ __forceinline__ float2 ld_h(const float2* p) {
  return Ld::kShared ? *p : __ldg(p);
}
struct HFromGlobal { static constexpr bool kShared = false; };
struct HFromShared { static constexpr bool kShared = true; };

template <int MODE, typename HL>
__device__ __forceinline__ void pp_bin_pairs2(int k0, int k1, int N, CP& zk, CP& znk, const CP& u,
                                              const RowArgs& a, int64_t row, const float2* H) {
  const u64 ur = u.re, ui = u.im;
  const u64 half = p_make(0.5f, 0.5f);
  CP yk, ynk;
  if (MODE != kModeIrfft) {
    // X[k] = fe + u fo, X[N-k] = conj(fe - u fo), fe = (Z[k] + conj Z[N-k]) / 2,
    // fo = (Z[k] - conj Z[N-k]) / 2i = (dim, -dre)
    const u64 fe_re = p_mul(p_add(zk.re, znk.re), half);
    const u64 fe_im = p_mul(p_sub(zk.im, znk.im), half);
    const u64 dre = p_mul(p_sub(zk.re, znk.re), half);
    const u64 dim = p_mul(p_add(zk.im, znk.im), half);
    const u64 wr = p_fma(ur, dim, p_mul(ui, dre));
    const u64 wi = p_sub(p_mul(ui, dim), p_mul(ur, dre));
    const CP xk{p_add(fe_re, wr), p_add(fe_im, wi)};
    const CP xnk{p_sub(fe_re, wr), p_sub(wi, fe_im)};
    if (MODE == kModeRfft) {
      float2* X = a.spec_out + row * a.out_ld;
      X[k0] = make_float2(p_lo(xk.re), p_lo(xk.im));
      X[k1] = make_float2(p_hi(xk.re), p_hi(xk.im));
      X[N - k0] = make_float2(p_lo(xnk.re), p_lo(xnk.im));
      X[N - k1] = make_float2(p_hi(xnk.re), p_hi(xnk.im));
      return;
    }
    const float2 h0 = ld_h<HL>(H + k0), h1 = ld_h<HL>(H + k1);
    const float2 g0 = ld_h<HL>(H + N - k0), g1 = ld_h<HL>(H + N - k1);
    const u64 hr = p_make(h0.x, h1.x), hi = p_make(h0.y, h1.y);
    const u64 gr = p_make(g0.x, g1.x), gi = p_make(g0.y, g1.y);
    yk = CP{p_sub(p_mul(xk.re, hr), p_mul(xk.im, hi)), p_fma(xk.re, hi, p_mul(xk.im, hr))};
    ynk = CP{p_sub(p_mul(xnk.re, gr), p_mul(xnk.im, gi)), p_fma(xnk.re, gi, p_mul(xnk.im, gr))};
  } else {
    const float2* Y = a.spec_in + row * a.spec_ld;
    const int len = a.spec_len;
    const float2 z = make_float2(0.f, 0.f);
    const float2 y0 = k0 < len ? Y[k0] : z, y1 = k1 < len ? Y[k1] : z;
    const float2 n0 = N - k0 < len ? Y[N - k0] : z, n1 = N - k1 < len ? Y[N - k1] : z;
    yk = CP{p_make(y0.x, y1.x), p_make(y0.y, y1.y)};
    ynk = CP{p_make(n0.x, n1.x), p_make(n0.y, n1.y)};
  }
  // Z'[k] = fe + i fo, Z'[N-k] = conj(fe) + i conj(fo), fe = (Y[k] + conj Y[N-k]) / 2,
  // fo = conj(u) (Y[k] - conj Y[N-k]) / 2; stored conjugated
  const u64 fe_re = p_mul(p_add(yk.re, ynk.re), half);
  const u64 fe_im = p_mul(p_sub(yk.im, ynk.im), half);
  const u64 dr = p_mul(p_sub(yk.re, ynk.re), half);
  const u64 di = p_mul(p_add(yk.im, ynk.im), half);
  const u64 fo_re = p_fma(ur, dr, p_mul(ui, di));
  const u64 fo_im = p_sub(p_mul(ur, di), p_mul(ui, dr));
  zk = CP{p_sub(fe_re, fo_im), p_sub(p_sub(p_make(0.f, 0.f), fe_im), fo_re)};
  znk = CP{p_add(fe_re, fo_im), p_sub(fe_im, fo_re)};
}

// Bins 0 and N (both real) -> conj of the packed inverse input Z'[0].
template <int MODE, typename HL>
__device__ __forceinline__ float2 pp_bin_dc(int N, float2 z0, const RowArgs& a, int64_t row,
                                            const float2* H) {
  if (MODE == kModeRfft) {
    float2* X = a.spec_out + row * a.out_ld;
    X[0] = make_float2(z0.x + z0.y, 0.f);
    X[N] = make_float2(z0.x - z0.y, 0.f);
    return z0;
  }
  float y0, yn;
  if (MODE == kModeConv) {
    y0 = (z0.x + z0.y) * ld_h<HL>(H).x;
    yn = (z0.x - z0.y) * ld_h<HL>(H + N).x;
  } else {
    const float2* Y = a.spec_in + row * a.spec_ld;
    y0 = 0 < a.spec_len ? Y[0].x : 0.f;
    yn = N < a.spec_len ? Y[N].x : 0.f;
  }
  return make_float2(0.5f * (y0 + yn), -0.5f * (y0 - yn));
}

template <int N, int R>
__device__ __forceinline__ void pp_store_transposed(const CP (&v)[R], PBuf dst, int j0, int j1) {
  // j R is a multiple of R <= 16 and r < R stays inside its 32-slot group
  const int b0 = pad3(j0 * R), b1 = pad3(j1 * R);
#pragma unroll
  for (int r = 0; r < R; r += 2) {
    sts2(dst.re + b0 + r, p_make(p_lo(v[r].re), p_lo(v[r + 1].re)));
    sts2(dst.im + b0 + r, p_make(p_lo(v[r].im), p_lo(v[r + 1].im)));
    sts2(dst.re + b1 + r, p_make(p_hi(v[r].re), p_hi(v[r + 1].re)));
    sts2(dst.im + b1 + r, p_make(p_hi(v[r].im), p_hi(v[r + 1].im)));
  }
}

// The bin-pair step of pp_mirror for outputs r and its mirrors, r < R/2.
// Lanes of an ordinary thread: butterflies j0 and j1 = N/R - j0, so v[r]
// holds two bins k < N/2 and the lane-swapped v[R-1-r] their mirrors.  Thread
// 0 (s0) has butterflies 0 and N/(2R), each its own mirror: its lane 1 pairs
// v[r] with v[R-1-r] as above, its lane 0 pairs v[r] with v[R-r] (r >= 1) and,
// at r = 0, takes the self-mirrored bin N/2 (output R/2); bin 0 is done apart.
// Selects keep every thread on one instruction stream.
template <int N, int R, int MODE, typename HL, int r>
__device__ __forceinline__ void pp_pairs(CP (&w)[R], const CP& u, bool s0, int j0, int j1,
                                         const RowArgs& a, int64_t row, const float2* H) {
  if constexpr (r < R / 2) {
    constexpr int NB = N / R;
    CP ur = cp_rot_half<R, r>(u);  // u[j + r N/R] = u[j] exp(-i pi r / R)
    CP zk, znk;
    int k0 = j0 + r * NB;
    const int k1 = j1 + r * NB;
    if constexpr (r == 0) {
      ur.re = p_make(f_sel(s0, 0.f, p_lo(ur.re)), p_hi(ur.re));
      ur.im = p_make(f_sel(s0, -1.f, p_lo(ur.im)), p_hi(ur.im));
      k0 = s0 ? N / 2 : k0;
      zk.re = p_make(f_sel(s0, p_lo(w[R / 2].re), p_lo(w[0].re)), p_hi(w[0].re));
      zk.im = p_make(f_sel(s0, p_lo(w[R / 2].im), p_lo(w[0].im)), p_hi(w[0].im));
      znk.re = p_make(f_sel(s0, p_lo(w[R / 2].re), p_hi(w[R - 1].re)),
                      f_sel(s0, p_hi(w[R - 1].re), p_lo(w[R - 1].re)));
      znk.im = p_make(f_sel(s0, p_lo(w[R / 2].im), p_hi(w[R - 1].im)),
                      f_sel(s0, p_hi(w[R - 1].im), p_lo(w[R - 1].im)));
    } else {
      zk = w[r];
      znk.re = p_make(f_sel(s0, p_lo(w[R - r].re), p_hi(w[R - 1 - r].re)),
                      f_sel(s0, p_hi(w[R - 1 - r].re), p_lo(w[R - 1 - r].re)));
      znk.im = p_make(f_sel(s0, p_lo(w[R - r].im), p_hi(w[R - 1 - r].im)),
                      f_sel(s0, p_hi(w[R - 1 - r].im), p_lo(w[R - 1 - r].im)));
    }
    pp_bin_pairs2<MODE, HL>(k0, k1, N, zk, znk, ur, a, row, H);
    if (MODE != kModeRfft) {
      if constexpr (r == 0) {
        w[0].re = p_make(f_sel(s0, p_lo(w[0].re), p_lo(zk.re)), p_hi(zk.re));
        w[0].im = p_make(f_sel(s0, p_lo(w[0].im), p_lo(zk.im)), p_hi(zk.im));
        w[R / 2].re = p_make(f_sel(s0, p_lo(zk.re), p_lo(w[R / 2].re)), p_hi(w[R / 2].re));
        w[R / 2].im = p_make(f_sel(s0, p_lo(zk.im), p_lo(w[R / 2].im)), p_hi(w[R / 2].im));
      } else {
        w[r] = zk;
        w[R - r].re = p_make(f_sel(s0, p_lo(znk.re), p_lo(w[R - r].re)), p_hi(w[R - r].re));
        w[R - r].im = p_make(f_sel(s0, p_lo(znk.im), p_lo(w[R - r].im)), p_hi(w[R - r].im));
      }
      w[R - 1 - r].re = p_make(f_sel(s0, p_lo(w[R - 1 - r].re), p_hi(znk.re)),
                               f_sel(s0, p_hi(znk.re), p_lo(znk.re)));
      w[R - 1 - r].im = p_make(f_sel(s0, p_lo(w[R - 1 - r].im), p_hi(znk.im)),
                               f_sel(s0, p_hi(znk.im), p_lo(znk.im)));
    }
    pp_pairs<N, R, MODE, HL, r + 1>(w, u, s0, j0, j1, a, row, H);
  }
}

// Last forward pass (radix R, NS = N/R) + the bin-pair step + first inverse
// pass (radix R, NS = 1), in registers.  Lanes: butterflies j and N/R - j
// (thread 0: 0 and N/(2R)).  Output r of butterfly j holds Z[j + r N/R],
// whose mirror N - k is output R-1-r of butterfly N/R - j; the first inverse
// pass reads input r of butterfly j from j + r N/R, exactly the element in
// hand, and writes j R + r.  The pass twiddles exp(-2 pi i r j / N) are
// products of two table roots (u[2j], u[8j] with u[k] = exp(-i pi k / N)), at
// most three roundings from exact.
template <int N, int R, int T, int MODE, bool INPLACE, typename HL = HFromGlobal>
__device__ __forceinline__ void pp_mirror(PBuf src, PBuf dst, const float2* __restrict__ utw,
                                          const RowArgs& a, int64_t row, const float2* H) {
  static_assert(R == 16, "the mirror pass is radix 16");
  constexpr int NB = N / R, PAIRS = NB / 2, PER = (PAIRS + T - 1) / T;
  constexpr int KEEP = INPLACE ? PER : 1;
  CP v[KEEP][R];
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    CP(&w)[R] = v[INPLACE ? p : 0];
    const int q = threadIdx.x + p * T;
    const bool s0 = q == 0;
    const int j0 = q, j1 = s0 ? NB / 2 : NB - q;
    if (PAIRS % T == 0 || q < PAIRS) {
      const float2 ua = __ldg(utw + j0), ub = __ldg(utw + j1);
      const CP u{p_make(ua.x, ub.x), p_make(ua.y, ub.y)};
      if (MODE != kModeIrfft) {
        if constexpr (NB >= 32) {
          const int b0 = pad3(j0), b1 = pad3(j1);   // j0, j1 < NB: base + constant
#pragma unroll
          for (int r = 0; r < R; ++r) {
            w[r].re = p_make(src.re[b0 + pad3c(r * NB)], src.re[b1 + pad3c(r * NB)]);
            w[r].im = p_make(src.im[b0 + pad3c(r * NB)], src.im[b1 + pad3c(r * NB)]);
          }
        } else {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            w[r].re = p_make(src.re[pad3(j0 + r * NB)], src.re[pad3(j1 + r * NB)]);
            w[r].im = p_make(src.im[pad3(j0 + r * NB)], src.im[pad3(j1 + r * NB)]);
          }
        }
        const float2 a1 = __ldg(utw + 2 * j0), b1 = __ldg(utw + 2 * j1);
        const float2 a4 = __ldg(utw + 8 * j0), b4 = __ldg(utw + 8 * j1);
        CP z[R];
        z[1] = CP{p_make(a1.x, b1.x), p_make(a1.y, b1.y)};
        z[4] = CP{p_make(a4.x, b4.x), p_make(a4.y, b4.y)};
        z[2] = cp_sqr(z[1]);
        z[3] = cp_mul(z[2], z[1]);
        z[8] = cp_sqr(z[4]);
        z[12] = cp_mul(z[8], z[4]);
#pragma unroll
        for (int r = 1; r < 4; ++r) {
          z[4 + r] = cp_mul(z[4], z[r]);
          z[8 + r] = cp_mul(z[8], z[r]);
          z[12 + r] = cp_mul(z[12], z[r]);
        }
#pragma unroll
        for (int r = 1; r < R; ++r) w[r] = cp_mul(w[r], z[r]);
        p_dft<R>(w);
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) w[r] = CP{0ull, 0ull};
      }
      if (s0) {
        const float2 o = pp_bin_dc<MODE, HL>(N, cp_get(w[0], 0), a, row, H);
        if (MODE != kModeRfft) cp_set(w[0], 0, o);
      }
      pp_pairs<N, R, MODE, HL, 0>(w, u, s0, j0, j1, a, row, H);
      if (MODE != kModeRfft) {
        p_dft<R>(w);
        if (!INPLACE) pp_store_transposed<N, R>(w, dst, j0, j1);
      }
    }
  }
  if (MODE == kModeRfft) return;
  if (INPLACE) {
    __syncthreads();
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int q = threadIdx.x + p * T;
      if (PAIRS % T == 0 || q < PAIRS)
        pp_store_transposed<N, R>(v[p], dst, q, q == 0 ? NB / 2 : NB - q);
    }
  }
  __syncthreads();
}

// Last inverse pass (radix R, NS = N/R) to the real output row:
// y[2m] + i y[2m+1] = conj(W[m]) / N.
constexpr int kGateNone = 0, kGateGlobal = 1, kGateShared = 2;

template <int N, int R, int T, int GATE = kGateNone>
__device__ __forceinline__ void pp_last(PBuf src, const float* __restrict__ tw, float* y,
                                        int olen, bool vec, const float* g = nullptr,
                                        int64_t g_st = 1, bool gvec = false) {
  constexpr int NB = N / R, NS = NB, PAIRS = NB / 2, PER = (PAIRS + T - 1) / T;
  const float scale = 1.0f / (float)N;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    const int q = threadIdx.x + p * T;
    if (PAIRS % T == 0 || q < PAIRS) {
      const int j = 2 * q;
      CP v[R];
      pp_load_dft<N, R, NS>(v, src, j, tw);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int t0 = 2 * (j + r * NS);
        if (t0 >= olen) break;
        float4 o = make_float4(p_lo(v[r].re) * scale, -p_lo(v[r].im) * scale,
                               p_hi(v[r].re) * scale, -p_hi(v[r].im) * scale);
        if (GATE != kGateNone) {
          if (gvec && t0 + 3 < olen) {
            const float4 gv = GATE == kGateShared ? *reinterpret_cast<const float4*>(g + t0)
                                                  : __ldg(reinterpret_cast<const float4*>(g + t0));
            o = make_float4(o.x * gv.x, o.y * gv.y, o.z * gv.z, o.w * gv.w);
          } else {
            o.x *= g[(int64_t)t0 * g_st];
            if (t0 + 1 < olen) o.y *= g[(int64_t)(t0 + 1) * g_st];
            if (t0 + 2 < olen) o.z *= g[(int64_t)(t0 + 2) * g_st];
            if (t0 + 3 < olen) o.w *= g[(int64_t)(t0 + 3) * g_st];
          }
        }
        if (vec && t0 + 3 < olen) {
          *reinterpret_cast<float4*>(y + t0) = o;
        } else {
          y[t0] = o.x;
          if (t0 + 1 < olen) y[t0 + 1] = o.y;
          if (t0 + 2 < olen) y[t0 + 2] = o.z;
          if (t0 + 3 < olen) y[t0 + 3] = o.w;
        }
      }
    }
  }
}

// Middle passes; with two buffers each pass reads buffer CUR and writes the other.
template <int L, int V, int T, bool DB, int p, int CUR>
__device__ __forceinline__ void pp_fwd_middle(const PBuf (&bufs)[2]) {
  if constexpr (p <= pp_count(L, V) - 2) {
    constexpr int NXT = DB ? 1 - CUR : CUR;
    pp_pass<(1 << L), pp_radix(L, V, p), pp_ns_fwd(L, V, p), T, !DB>(
        bufs[CUR], bufs[NXT], g_fft_ptw + pt_fwd_off(L, V, p));
    pp_fwd_middle<L, V, T, DB, p + 1, NXT>(bufs);
  }
}

template <int L, int V, int T, bool DB, int q, int CUR>
__device__ __forceinline__ void pp_inv_middle(const PBuf (&bufs)[2]) {
  if constexpr (q <= pp_count(L, V) - 2) {
    constexpr int NXT = DB ? 1 - CUR : CUR;
    pp_pass<(1 << L), pp_radix_inv(L, V, q), pp_ns_inv(L, V, q), T, !DB>(
        bufs[CUR], bufs[NXT], g_fft_ptw + pt_inv_off(L, V, q));
    pp_inv_middle<L, V, T, DB, q + 1, NXT>(bufs);
  }
}

// Gate row of (b, d) and whether it takes 16-byte vector loads.
__device__ __forceinline__ const float* gate_row(const RowArgs& a, int b, int d, bool& gvec) {
  if (a.gate == nullptr) {
    gvec = false;
    return nullptr;
  }
  const float* g = a.gate + a.g_off + (int64_t)b * a.g_sb + (int64_t)d * a.g_sd;
  gvec = a.g_st == 1 && (reinterpret_cast<uintptr_t>(g) & 15) == 0;
  return g;
}

// One CTA per row, N = 2^L complex values (n = 2N real samples).
template <int L, int MODE>
__global__ void __launch_bounds__(PCfg<L>::T, 1) fft_pair_kernel(RowArgs a) {
  using C = PCfg<L>;
  constexpr int N = C::N, T = C::T, P = C::P;
  constexpr bool DB = C::DB;
  extern __shared__ __align__(16) float psm[];
  const PBuf bufs[2] = {PBuf{psm, psm + padded3(N)},
                        DB ? PBuf{psm + C::BUF, psm + C::BUF + padded3(N)}
                           : PBuf{psm, psm + padded3(N)}};
  // buffer holding the row before the mirror pass / before the last pass
  constexpr int CUR_MIRROR = DB ? (P - 2) % 2 : 0;
  constexpr int CUR_INV = DB ? 1 - CUR_MIRROR : 0;
  constexpr int CUR_LAST = DB ? (CUR_INV + P - 2) % 2 : 0;
  const float2* utw = g_fft_tw + tw_offset(L) + tw_passes_size(N);  // exp(-i pi k / N)

  const int d = blockIdx.x / a.rows_b;
  const int b = blockIdx.x - d * a.rows_b;
  const int64_t row = (int64_t)b * a.rows_d + d;

  if (MODE != kModeIrfft) {
    const float* x = a.in + a.in_off + (int64_t)b * a.in_sb + (int64_t)d * a.in_sd;
    const bool vec = a.in_st == 1 && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    pp_first<N, pp_radix(L, 0, 0), T>(bufs[0], x, a.in_st, a.in_len, vec);
    pp_fwd_middle<L, 0, T, DB, 1, 0>(bufs);
  }
  pp_mirror<N, pp_radix(L, 0, P - 1), T, MODE, !DB>(bufs[CUR_MIRROR], bufs[CUR_INV], utw, a, row,
                                                 MODE == kModeConv ? a.H + (int64_t)d * a.h_ld
                                                                   : nullptr);
  if (MODE == kModeRfft) return;
  pp_inv_middle<L, 0, T, DB, 1, CUR_INV>(bufs);
  float* y = a.out + row * a.out_ld;
  const bool vec = (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  bool gvec;
  const float* g = MODE == kModeConv ? gate_row(a, b, d, gvec) : nullptr;
  if (g != nullptr)
    pp_last<N, pp_radix_inv(L, 0, P - 1), T, kGateGlobal>(
        bufs[CUR_LAST], g_fft_ptw + pt_inv_off(L, 0, P - 1), y, a.out_len, vec, g, a.g_st, gvec);
  else
    pp_last<N, pp_radix_inv(L, 0, P - 1), T>(bufs[CUR_LAST], g_fft_ptw + pt_inv_off(L, 0, P - 1),
                                             y, a.out_len, vec);
}

// Persistent fused convolution for L <= 13 with the next row's inputs staged
// in shared memory while the current row is transformed: one async bulk copy
// (cp.async.bulk, no multicast) brings the next row's x (issued once the
// first pass has consumed the current one), one its filter-spectrum row
// (issued once the mirror pass has used the current one) and, for the gated
// form, one its gate row (issued at the end of the row), each completing on
// its own mbarrier.  The first pass and the spectrum product then read
// shared memory instead of waiting on HBM and L2.  The row is transformed in
// place (one planar buffer).  Requirements (checked by the host): x rows
// contiguous, 16-byte aligned, staged length a multiple of 4 floats; H rows
// 16-byte aligned with N + 2 complex values readable.
template <int L>
struct SCfg {
  static constexpr int N = 1 << L;
  static constexpr int T = PCfg<L>::T;
  static constexpr int H_FLOATS = 2 * (N + 2);      // staged H row (N + 2 complex)
  static constexpr int BUF_FLOATS = 2 * padded3(N);
  // shared memory: staged x (xlen floats), staged gate (glen), H row, row buffer
  static constexpr int smem(int xlen, int glen) { return (xlen + glen + H_FLOATS + BUF_FLOATS) * 4; }
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          wxx_tc::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(wxx_tc::smem_u32(bar))
      : "memory");
}

template <int L>
__global__ void __launch_bounds__(SCfg<L>::T, 1)
    fft_conv_staged_kernel(RowArgs a, int64_t rows, int xlen, int glen, int* err) {
  using C = SCfg<L>;
  constexpr int N = C::N, T = C::T, V = L == 13 ? 1 : 0, P = pp_count(L, V);
  extern __shared__ __align__(128) float ssm[];
  __shared__ __align__(8) uint64_t bars[3];  // x, H, gate staged
  __shared__ int abort_flag;
  float* sx = ssm;
  float* sg = ssm + xlen;
  float2* sh = reinterpret_cast<float2*>(ssm + xlen + glen);
  float* bb = ssm + xlen + glen + C::H_FLOATS;
  const PBuf bufs[2] = {PBuf{bb, bb + padded3(N)}, PBuf{bb, bb + padded3(N)}};
  const float2* utw = g_fft_tw + tw_offset(L) + tw_passes_size(N);
  const uint32_t xbytes = (uint32_t)xlen * 4u, hbytes = (uint32_t)(N + 2) * 8u;
  const uint32_t gbytes = (uint32_t)glen * 4u;
  auto g_row = [&](int64_t r) {
    const int d = (int)(r / a.rows_b), b = (int)(r - (int64_t)d * a.rows_b);
    return a.gate + a.g_off + (int64_t)b * a.g_sb + (int64_t)d * a.g_sd;
  };

  auto x_row = [&](int64_t r) {
    const int d = (int)(r / a.rows_b), b = (int)(r - (int64_t)d * a.rows_b);
    return a.in + a.in_off + (int64_t)b * a.in_sb + (int64_t)d * a.in_sd;
  };
  auto h_row = [&](int64_t r) { return a.H + (r / a.rows_b) * a.h_ld; };

  if (threadIdx.x == 0) {
    wxx_tc::mbar_init(&bars[0], 1);
    wxx_tc::mbar_init(&bars[1], 1);
    wxx_tc::mbar_init(&bars[2], 1);
    wxx_tc::fence_barrier_init();
    abort_flag = 0;
  }
  __syncthreads();
  int64_t r = blockIdx.x;
  if (threadIdx.x == 0 && r < rows) {
    wxx_tc::mbar_arrive_expect_tx(&bars[0], xbytes);
    bulk_g2s(sx, x_row(r), xbytes, &bars[0]);
    wxx_tc::mbar_arrive_expect_tx(&bars[1], hbytes);
    bulk_g2s(sh, h_row(r), hbytes, &bars[1]);
    if (glen > 0) {
      wxx_tc::mbar_arrive_expect_tx(&bars[2], gbytes);
      bulk_g2s(sg, g_row(r), gbytes, &bars[2]);
    }
  }
  uint32_t phase = 0;
  for (; r < rows; r += gridDim.x, phase ^= 1u) {
    const int64_t nxt = r + gridDim.x;
    const int d = (int)(r / a.rows_b), b = (int)(r - (int64_t)d * a.rows_b);
    const int64_t row = (int64_t)b * a.rows_d + d;

    bool ok = wxx_tc::mbar_wait(&bars[0], phase, &abort_flag, err);
    if (__syncthreads_or(!ok)) return;
    pp_first<N, pp_radix(L, V, 0), T, true>(bufs[0], sx, 1, xlen, true);
    if (threadIdx.x == 0 && nxt < rows) {
      wxx_tc::mbar_arrive_expect_tx(&bars[0], xbytes);
      bulk_g2s(sx, x_row(nxt), xbytes, &bars[0]);
    }
    pp_fwd_middle<L, V, T, false, 1, 0>(bufs);

    ok = wxx_tc::mbar_wait(&bars[1], phase, &abort_flag, err);
    if (__syncthreads_or(!ok)) return;
    pp_mirror<N, pp_radix(L, V, P - 1), T, kModeConv, true, HFromShared>(bufs[0], bufs[0], utw, a,
                                                                       row, sh);
    if (threadIdx.x == 0 && nxt < rows) {
      wxx_tc::mbar_arrive_expect_tx(&bars[1], hbytes);
      bulk_g2s(sh, h_row(nxt), hbytes, &bars[1]);
    }
    pp_inv_middle<L, V, T, false, 1, 0>(bufs);
    float* y = a.out + row * a.out_ld;
    const bool vec = (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    const float* tl = g_fft_ptw + pt_inv_off(L, V, P - 1);
    if (glen > 0) {
      ok = wxx_tc::mbar_wait(&bars[2], phase, &abort_flag, err);
      if (__syncthreads_or(!ok)) return;
      pp_last<N, pp_radix_inv(L, V, P - 1), T, kGateShared>(bufs[0], tl, y, a.out_len, vec, sg, 1,
                                                            true);
    } else if (a.gate != nullptr) {
      bool gvec;
      const float* g = gate_row(a, b, d, gvec);
      pp_last<N, pp_radix_inv(L, V, P - 1), T, kGateGlobal>(bufs[0], tl, y, a.out_len, vec, g,
                                                            a.g_st, gvec);
    } else {
      pp_last<N, pp_radix_inv(L, V, P - 1), T>(bufs[0], tl, y, a.out_len, vec);
    }
    __syncthreads();  // the next row's first pass overwrites the buffer
    if (glen > 0 && threadIdx.x == 0 && nxt < rows) {
      wxx_tc::mbar_arrive_expect_tx(&bars[2], gbytes);
      bulk_g2s(sg, g_row(nxt), gbytes, &bars[2]);
    }
  }
}

// ------------------------------------------------------------ two-CTA convolution (n = 16384)
//
// The fused convolution at N = 8192 complex values per row, sized so that two
// CTAs share an SM (256 threads, <= 128 registers each, one 72 KB planar row
// buffer): while one CTA waits at a pass barrier or on memory the other
// issues.  Plan (radices of fft_pair_kernel<13>): forward 16 | 32 | 16 with the
// last forward pass, the spectrum product and the first inverse pass fused in
// registers (pp_mirror), then inverse 32 | 16 to global memory.  Every pass
// transforms in place: loads, barrier, stores.  x, the filter spectrum and the
// gate are read straight from global memory (the spectrum and gate stay in
// L2 across the batch); the radix-32 passes are split over two threads so
// that no thread holds more than 16 paired values.

__device__ __forceinline__ u64 p_sel(bool c, u64 a, u64 b) { return c ? a : b; }

// One in-place Stockham pass of radix 32 (sub-transform size NS before it)
// over butterfly pairs (j, j+1), each pair shared by two threads: the thread of
// parity h loads the inputs r = 2m + h (m = 0..15), twiddles them and runs a
// 16-point DFT, giving E_h[s] = sum_m x[2m+h] w16^(ms).  The 32 outputs are
// X[s] = E_0[s] + w32^s E_1[s] and X[s+16] = E_0[s] - w32^s E_1[s]; thread
// h = 0 makes those of s = 0..7 and thread h = 1 those of s = 8..15, after
// trading E_0[8..15] for E_1[0..7] with its partner (lane xor 1).
// w32^(8+i) = -i w32^i, so both threads use the constants w32^i.
template <int N, int NS, int T>
__device__ __forceinline__ void pp_split32(PBuf buf, const float* __restrict__ tw) {
  constexpr int R = 32, NB = N / R;
  static_assert(NB == T, "one thread per half butterfly pair");
  const int h = threadIdx.x & 1;
  const bool odd = h != 0;
  const int j = (threadIdx.x >> 1) * 2;
  const int k = j & (NS - 1);
  CP v[16];
  // j + h NB < 512 and 2 m NB is a multiple of 512: base + constant
  const int lb = pad3(j + h * NB);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    v[m].re = lds2(buf.re + lb + pad3c(2 * m * NB));
    v[m].im = lds2(buf.im + lb + pad3c(2 * m * NB));
  }
  {
    // m = 0: input r = h; r = 0 has no twiddle
    const u64 c = ldg2(tw + k), sn = ldg2(tw + (R - 1) * NS + k);
    const CP t = v[0];
    CP w = t;
    p_twiddle(w, c, sn);
    v[0].re = p_sel(odd, w.re, t.re);
    v[0].im = p_sel(odd, w.im, t.im);
  }
#pragma unroll
  for (int m = 1; m < 16; ++m) {
    const int r = 2 * m + h;
    p_twiddle(v[m], ldg2(tw + (r - 1) * NS + k), ldg2(tw + (R - 1 + r - 1) * NS + k));
  }
  p_dft<16>(v);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // send E_h[8+i] (h = 0) or E_h[i] (h = 1); receive the partner's
    const u64 sre = p_sel(odd, v[i].re, v[8 + i].re);
    const u64 sim = p_sel(odd, v[i].im, v[8 + i].im);
    const u64 rre = __shfl_xor_sync(0xffffffffu, sre, 1);
    const u64 rim = __shfl_xor_sync(0xffffffffu, sim, 1);
    // a = E_0[s], b = E_1[s], s = 8h + i
    const CP a{p_sel(odd, rre, v[i].re), p_sel(odd, rim, v[i].im)};
    const CP b{p_sel(odd, v[8 + i].re, rre), p_sel(odd, v[8 + i].im, rim)};
    const float c = cos32(i), sn = sin32(i);   // constants once unrolled
    const u64 C = p_make(c, c), S = p_make(sn, sn), NS_ = p_make(-sn, -sn);
    // t = w32^i b = (re c + im sn) + i (im c - re sn)
    u64 tr = p_fma(b.re, C, p_mul(b.im, S));
    u64 ti = p_fma(b.im, C, p_mul(b.re, NS_));
    // h = 1: t *= -i  ->  (ti, -tr)
    const u64 ntr = p_sub(0ull, tr);
    const u64 tr2 = p_sel(odd, ti, tr);
    const u64 ti2 = p_sel(odd, ntr, ti);
    v[i] = CP{p_add(a.re, tr2), p_add(a.im, ti2)};        // output 8h + i
    v[8 + i] = CP{p_sub(a.re, tr2), p_sub(a.im, ti2)};    // output 16 + 8h + i
  }
  __syncthreads();   // every input is read before any output is stored
  static_assert(NS == 16, "store offsets written for NS = 16");
  // outputs r0 = 8h + i and r1 = 16 + 8h + i at (j - k) R + k + r NS: the
  // (j - k) R part is a multiple of 512, and pad3(16 r) = 136 h + pad3c(16 i)
  // (+ 256 for r1), so base + constant
  const int sb = pad3((j - k) * R) + k + 136 * h;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sts2(buf.re + sb + pad3c(16 * i), v[i].re);
    sts2(buf.im + sb + pad3c(16 * i), v[i].im);
    sts2(buf.re + sb + pad3c(256 + 16 * i), v[8 + i].re);
    sts2(buf.im + sb + pad3c(256 + 16 * i), v[8 + i].im);
  }
  __syncthreads();
}

template <int L>
struct C2Cfg {
  static constexpr int N = 1 << L;
  static constexpr int T = 256;
  static constexpr int SMEM = 2 * padded3(N) * 4;   // one planar row buffer
};

template <int L, bool GATED>
__global__ void __launch_bounds__(C2Cfg<L>::T, 2) fft_conv2_kernel(RowArgs a) {
  static_assert(L == 13, "plan written for N = 8192");
  constexpr int N = C2Cfg<L>::N, T = C2Cfg<L>::T;
  extern __shared__ __align__(16) float psm[];
  const PBuf buf{psm, psm + padded3(N)};
  const float2* utw = g_fft_tw + tw_offset(L) + tw_passes_size(N);  // exp(-i pi k / N)
  const int d = blockIdx.x / a.rows_b;
  const int b = blockIdx.x - d * a.rows_b;
  const int64_t row = (int64_t)b * a.rows_d + d;
  const float* x = a.in + a.in_off + (int64_t)b * a.in_sb + (int64_t)d * a.in_sd;
  const bool xvec = a.in_st == 1 && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  pp_first<N, 16, T>(buf, x, a.in_st, a.in_len, xvec);
  pp_split32<N, 16, T>(buf, g_fft_ptw + pt_fwd_off(L, 0, 1));
  pp_mirror<N, 16, T, kModeConv, true>(buf, buf, utw, a, row, a.H + (int64_t)d * a.h_ld);
  pp_split32<N, 16, T>(buf, g_fft_ptw + pt_inv_off(L, 0, 1));
  float* y = a.out + row * a.out_ld;
  const bool vec = (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  const float* tl = g_fft_ptw + pt_inv_off(L, 0, 2);
  if constexpr (GATED) {
    bool gvec;
    const float* g = gate_row(a, b, d, gvec);
    pp_last<N, 16, T, kGateGlobal>(buf, tl, y, a.out_len, vec, g, a.g_st, gvec);
  } else {
    pp_last<N, 16, T>(buf, tl, y, a.out_len, vec);
  }
}

// ------------------------------------------------------------ dispatch

template <int LOGN, int MODE>
int launch_row(const RowArgs& a, int64_t rows) {
  static bool attr = false;
  if constexpr (LOGN >= kPairMinL) {
    using C = PCfg<LOGN>;
    if (!attr) {
      WXX_CUDA_CHECK(cudaFuncSetAttribute(fft_pair_kernel<LOGN, MODE>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      attr = true;
    }
    fft_pair_kernel<LOGN, MODE><<<(unsigned)rows, C::T, C::SMEM, wxx::stream()>>>(a);
  } else {
    using C = RowCfg<LOGN>;
    if (!attr) {
      WXX_CUDA_CHECK(cudaFuncSetAttribute(fft_row_kernel<LOGN, MODE>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      attr = true;
    }
    fft_row_kernel<LOGN, MODE><<<(unsigned)rows, C::T, C::SMEM, wxx::stream()>>>(a);
  }
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

template <int MODE>
int launch_row_any(int logn, const RowArgs& a, int64_t rows) {
  switch (logn) {
    case 0: return launch_row<0, MODE>(a, rows);
    case 1: return launch_row<1, MODE>(a, rows);
    case 2: return launch_row<2, MODE>(a, rows);
    case 3: return launch_row<3, MODE>(a, rows);
    case 4: return launch_row<4, MODE>(a, rows);
    case 5: return launch_row<5, MODE>(a, rows);
    case 6: return launch_row<6, MODE>(a, rows);
    case 7: return launch_row<7, MODE>(a, rows);
    case 8: return launch_row<8, MODE>(a, rows);
    case 9: return launch_row<9, MODE>(a, rows);
    case 10: return launch_row<10, MODE>(a, rows);
    case 11: return launch_row<11, MODE>(a, rows);
    case 12: return launch_row<12, MODE>(a, rows);
    case 13: return launch_row<13, MODE>(a, rows);
    case 14: return launch_row<14, MODE>(a, rows);
    default: wxx::set_error("fft: unsupported size"); return WXX_E_ARG;
  }
}

int ilog2_exact(int64_t n) {
  if (n < 1 || (n & (n - 1))) return -1;
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return l;
}

// The two-CTA convolution at N = 8192 (fft_conv2_kernel).
template <bool GATED>
int launch_conv2(const RowArgs& a, int64_t rows) {
  static bool attr = false;
  if (!attr) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(fft_conv2_kernel<13, GATED>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C2Cfg<13>::SMEM));
    attr = true;
  }
  fft_conv2_kernel<13, GATED><<<(unsigned)rows, C2Cfg<13>::T, C2Cfg<13>::SMEM, wxx::stream()>>>(a);
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

bool conv2_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("WXX_FFT_CONV2");
    on = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// The staged persistent convolution, when the rows allow bulk copies.
// Dynamic shared memory the staged kernels may request: the opt-in limit per
// block less their static shared variables (mbarriers, abort flag) and slack.
constexpr int kMaxDynSmem = 227 * 1024 - 256;

template <int L>
int launch_conv_staged(const RowArgs& a, int64_t rows, int xlen, int glen) {
  using C = SCfg<L>;
  static int sms = 0;
  if (sms == 0) {
    WXX_CUDA_CHECK(cudaFuncSetAttribute(fft_conv_staged_kernel<L>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem));
    int dev = 0;
    WXX_CUDA_CHECK(cudaGetDevice(&dev));
    WXX_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int smem = C::smem(xlen, glen);
  int per_sm = 0;
  WXX_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fft_conv_staged_kernel<L>,
                                                               C::T, smem));
  const int64_t cap = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  fft_conv_staged_kernel<L><<<grid, C::T, smem, wxx::stream()>>>(a, rows, xlen, glen,
                                                                 wxx::device_error_word());
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}

// Rows that bulk copies can move (16-byte aligned starts and sizes): x and H
// always, the gate when it has them too (else the last pass loads it from
// global memory).  Returns false when the staged kernel does not apply.
bool conv_stageable(const RowArgs& a, int L, int* xlen, int* glen) {
  const int N = 1 << L;
  const int64_t xl = a.in_len < 2 * (int64_t)N ? a.in_len : 2 * (int64_t)N;
  *xlen = (int)xl;
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(a.in + a.in_off);
  if (!(a.in_st == 1 && xl > 0 && xl % 4 == 0 && (x0 & 15) == 0 && a.in_sb % 4 == 0 &&
        a.in_sd % 4 == 0 && (reinterpret_cast<uintptr_t>(a.H) & 15) == 0 && a.h_ld % 2 == 0 &&
        a.h_ld >= N + 2))
    return false;
  const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.gate + a.g_off);
  *glen = (a.gate != nullptr && a.g_st == 1 && a.out_len > 0 && a.out_len % 4 == 0 &&
           (g0 & 15) == 0 && a.g_sb % 4 == 0 && a.g_sd % 4 == 0)
              ? a.out_len
              : 0;
  const int fixed = 2 * (N + 2) + 2 * padded3(N);
  if ((*xlen + *glen + fixed) * 4 > kMaxDynSmem) *glen = 0;
  return (*xlen + *glen + fixed) * 4 <= kMaxDynSmem;
}

// Runs `mode` over all rows, choosing the shared-memory or global path.
int run_rows(int mode, int64_t n, RowArgs a, int64_t rows, const float2* Hspec) {
  if (rows == 0) return WXX_OK;
  cudaStream_t s = wxx::stream();
  if (n == 1) {
    fft_n1_kernel<<<wxx::grid_for(rows, 256), 256, 0, s>>>(a, mode, rows);
    WXX_LAUNCH_CHECK();
    return WXX_OK;
  }
  int logN = ilog2_exact(n) - 1;
  int N = (int)(n / 2);
  WXX_REQUIRE(rows < (int64_t(1) << 31), "fft: too many rows");
  if (logN <= kMaxSmemLogN) {
    int xlen = 0, glen = 0;
    if (mode == kModeConv && logN == 13 && conv2_enabled())
      return a.gate != nullptr ? launch_conv2<true>(a, rows) : launch_conv2<false>(a, rows);
    if (mode == kModeConv && logN >= kPairMinL && logN <= 13 &&
        conv_stageable(a, logN, &xlen, &glen)) {
      switch (logN) {
        case 8: return launch_conv_staged<8>(a, rows, xlen, glen);
        case 9: return launch_conv_staged<9>(a, rows, xlen, glen);
        case 10: return launch_conv_staged<10>(a, rows, xlen, glen);
        case 11: return launch_conv_staged<11>(a, rows, xlen, glen);
        case 12: return launch_conv_staged<12>(a, rows, xlen, glen);
        default: return launch_conv_staged<13>(a, rows, xlen, glen);
      }
    }
    if (mode == kModeRfft) return launch_row_any<kModeRfft>(logN, a, rows);
    if (mode == kModeIrfft) return launch_row_any<kModeIrfft>(logN, a, rows);
    return launch_row_any<kModeConv>(logN, a, rows);
  }
  // Global path: ping-pong scratch of rows * N complex values each.
  (void)Hspec;
  void* s0 = nullptr;
  void* s1 = nullptr;
  uint64_t bytes = (uint64_t)rows * N * sizeof(float2);
  int st = wxx_malloc(&s0, bytes);
  if (st) return st;
  st = wxx_malloc(&s1, bytes);
  if (st) { wxx_free(s0); return st; }
  float2* cur = (float2*)s0;
  float2* oth = (float2*)s1;
  unsigned g = wxx::grid_for(rows * N, 256);
  int rc = WXX_OK;
  auto passes = [&](int inv) {
    for (int Ns = 1; Ns < N; Ns *= 2) {
      stockham2_global_kernel<<<g, 256, 0, s>>>(oth, cur, N, Ns, rows, inv);
      float2* t = cur; cur = oth; oth = t;
    }
  };
  if (mode != kModeIrfft) {
    pack_real_kernel<<<g, 256, 0, s>>>(cur, a, N, rows);
    passes(0);
    unpack_global_kernel<<<g, 256, 0, s>>>(cur, a, N, rows, mode == kModeRfft ? kModeRfft : kModeConv);
  } else {
    pack_spectrum_global_kernel<<<g, 256, 0, s>>>(cur, a, N, rows);
  }
  if (mode != kModeRfft) {
    passes(1);
    unpack_real_global_kernel<<<g, 256, 0, s>>>(cur, a, N, rows);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    wxx::set_error("fft global path launch failed: %s", cudaGetErrorString(e));
    rc = WXX_E_CUDA;
  }
  wxx_free(s0);
  wxx_free(s1);
  return rc;
}

}  // namespace

namespace wxx {
// Fills the FFT twiddle tables of every shared-memory size (called by wxx_init).
int fft_init_tables() {
  fft_twiddle_init_kernel<<<64, 256, 0, wxx::stream()>>>();
  WXX_LAUNCH_CHECK();
  fft_pair_twiddle_init_kernel<<<64, 256, 0, wxx::stream()>>>();
  WXX_LAUNCH_CHECK();
  return WXX_OK;
}
}  // namespace wxx

// X[r, k] (c64, row stride out_ld complex) = rfft(x[r, :in_len], n), k <= n/2.
// x rows are dense with row stride in_ld floats.
WXX_EXPORT int wxx_rfft(void* X, int64_t out_ld, const float* x, int64_t in_ld, int64_t rows,
                        int64_t in_len, int64_t n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(ilog2_exact(n) >= 0, "wxx_rfft: n=%lld is not a positive power of two", (long long)n);
  WXX_REQUIRE(n <= (int64_t(1) << 30), "wxx_rfft: n too large");
  RowArgs a;
  memset(&a, 0, sizeof(a));
  a.in = x;
  a.in_sb = in_ld;
  a.in_st = 1;
  a.in_len = (int)in_len;
  a.spec_out = (float2*)X;
  a.out_ld = out_ld;
  a.rows_b = (int)rows;
  a.rows_d = 1;
  // row (b, d=0) -> output row b
  return run_rows(kModeRfft, n, a, rows, nullptr);
}

// y[r, t] (row stride out_ld floats, t < n) = irfft(X[r, :in_len], n).
WXX_EXPORT int wxx_irfft(float* y, int64_t out_ld, const void* X, int64_t in_ld, int64_t rows,
                         int64_t in_len, int64_t n) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(ilog2_exact(n) >= 0, "wxx_irfft: n=%lld is not a positive power of two", (long long)n);
  WXX_REQUIRE(n <= (int64_t(1) << 30), "wxx_irfft: n too large");
  RowArgs a;
  memset(&a, 0, sizeof(a));
  a.spec_in = (const float2*)X;
  a.spec_ld = in_ld;
  a.spec_len = (int)in_len;
  a.out = y;
  a.out_ld = out_ld;
  a.out_len = (int)n;
  a.rows_b = (int)rows;
  a.rows_d = 1;
  return run_rows(kModeIrfft, n, a, rows, nullptr);
}

// Causal FFT convolution with a precomputed filter spectrum:
//   y[b, d, t] = irfft(rfft(x[b, d, :], n) * H[d, :], n)[t],  t < out_len
// x is a strided (B, D, L) view (element strides sb, sd, sl from x_off);
// H is (D, n/2+1) c64 with row stride h_ld; y is dense (B, D, out_len).
static int fftconv_spectrum_impl(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                                 int64_t sl, const void* H, int64_t h_ld, int B, int D, int L,
                                 int64_t n, int out_len, const float* gate, int64_t g_off,
                                 int64_t g_sb, int64_t g_sd, int64_t g_sl);

WXX_EXPORT int wxx_fftconv_spectrum(float* y, const float* x, int64_t x_off, int64_t sb,
                                    int64_t sd, int64_t sl, const void* H, int64_t h_ld, int B,
                                    int D, int L, int64_t n, int out_len) {
  return fftconv_spectrum_impl(y, x, x_off, sb, sd, sl, H, h_ld, B, D, L, n, out_len, nullptr, 0,
                               0, 0, 0);
}

static int fftconv_spectrum_impl(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                                 int64_t sl, const void* H, int64_t h_ld, int B, int D, int L,
                                 int64_t n, int out_len, const float* gate, int64_t g_off,
                                 int64_t g_sb, int64_t g_sd, int64_t g_sl) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(ilog2_exact(n) >= 0, "wxx_fftconv: n=%lld is not a positive power of two", (long long)n);
  WXX_REQUIRE(out_len >= 0 && out_len <= n, "wxx_fftconv: out_len must be in [0, n]");
  RowArgs a;
  memset(&a, 0, sizeof(a));
  a.in = x;
  a.in_off = x_off;
  a.in_sb = sb;
  a.in_sd = sd;
  a.in_st = sl;
  a.in_len = L;
  a.H = (const float2*)H;
  a.h_ld = h_ld;
  a.out = y;
  a.out_ld = out_len;
  a.out_len = out_len;
  a.rows_b = B;
  a.rows_d = D;
  a.gate = gate;
  a.g_off = g_off;
  a.g_sb = g_sb;
  a.g_sd = g_sd;
  a.g_st = g_sl;
  return run_rows(kModeConv, n, a, (int64_t)B * D, (const float2*)H);
}

// Causal FFT convolution with a time-domain filter h (D, Lh) (dense, row
// stride h_ld floats): computes H = rfft(h, n) into a temporary and runs
// wxx_fftconv_spectrum.  This is Hyena's fft_conv1d (nn/hyena.py:208-216):
//   y = irfft(rfft(x, n) * rfft(h, n), n)[..., :out_len]
static int fftconv_impl(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                        int64_t sl, const float* h, int64_t h_ld, int Lh, int B, int D, int L,
                        int64_t n, int out_len, const float* gate, int64_t g_off, int64_t g_sb,
                        int64_t g_sd, int64_t g_sl);

WXX_EXPORT int wxx_fftconv(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                           int64_t sl, const float* h, int64_t h_ld, int Lh, int B, int D, int L,
                           int64_t n, int out_len) {
  return fftconv_impl(y, x, x_off, sb, sd, sl, h, h_ld, Lh, B, D, L, n, out_len, nullptr, 0, 0, 0,
                      0);
}

// Gated form: y[b, d, t] = gate[b, d, t] * fftconv(x, h)[b, d, t] for a
// strided (B, D, out_len) gate view (element strides g_sb, g_sd, g_sl from
// g_off).  Hyena's z = gates[i] * fft_conv1d(z, h) (nn/hyena.py:240) in one
// pass: the product is applied as the output is stored.
// wxx_fftconv_spectrum whose output is multiplied by a strided gate view as it
// is stored (Hyena's gates[i] * fft_conv1d(z, h) with the filter spectrum made
// once and kept).
WXX_EXPORT int wxx_fftconv_spectrum_gated(float* y, const float* x, int64_t x_off, int64_t sb,
                                          int64_t sd, int64_t sl, const void* H, int64_t h_ld,
                                          int B, int D, int L, int64_t n, int out_len,
                                          const float* gate, int64_t g_off, int64_t g_sb,
                                          int64_t g_sd, int64_t g_sl) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(gate != nullptr, "wxx_fftconv_spectrum_gated: gate is null");
  return fftconv_spectrum_impl(y, x, x_off, sb, sd, sl, H, h_ld, B, D, L, n, out_len, gate, g_off,
                               g_sb, g_sd, g_sl);
}

WXX_EXPORT int wxx_fftconv_gated(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                                 int64_t sl, const float* h, int64_t h_ld, int Lh, int B, int D,
                                 int L, int64_t n, int out_len, const float* gate, int64_t g_off,
                                 int64_t g_sb, int64_t g_sd, int64_t g_sl) {
  WXX_REQUIRE(gate != nullptr, "wxx_fftconv_gated: gate is null");
  return fftconv_impl(y, x, x_off, sb, sd, sl, h, h_ld, Lh, B, D, L, n, out_len, gate, g_off,
                      g_sb, g_sd, g_sl);
}

static int fftconv_impl(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                        int64_t sl, const float* h, int64_t h_ld, int Lh, int B, int D, int L,
                        int64_t n, int out_len, const float* gate, int64_t g_off, int64_t g_sb,
                        int64_t g_sd, int64_t g_sl) {
  WXX_REQUIRE_INIT();
  WXX_REQUIRE(ilog2_exact(n) >= 0, "wxx_fftconv: n=%lld is not a positive power of two", (long long)n);
  // spectrum rows of n/2 + 2 complex values: 16-byte aligned, so the fused
  // kernel can bulk-copy them
  int64_t ld = n / 2 + 2;
  void* Hs = nullptr;
  int st = wxx_malloc(&Hs, (uint64_t)D * ld * sizeof(float2));
  if (st) return st;
  st = wxx_rfft(Hs, ld, h, h_ld, D, Lh, n);
  if (st == WXX_OK)
    st = fftconv_spectrum_impl(y, x, x_off, sb, sd, sl, Hs, ld, B, D, L, n, out_len, gate, g_off,
                               g_sb, g_sd, g_sl);
  int st2 = wxx_free(Hs);
  return st ? st : st2;
}
