/*
 * wxx_cuda.h -- C ABI of libwxx_cuda.so, the sm_100a (B200) kernel library
 * behind the wxx.functional operator layer.
 *
 * Conventions
 *   - Every function returns 0 on success or a negative status:
 *       -1 WXX_E_ARG  -2 WXX_E_CUDA  -3 WXX_E_TIMEOUT  -4 WXX_E_UNSUPPORTED  -5 WXX_E_STATE
 *     and wxx_last_error() returns the message of the last failure (per host thread).
 *   - All pointers are device pointers unless stated; sizes and strides are in
 *     elements (4-byte f32/u32 or 8-byte interleaved c64) unless stated.
 *   - Work is enqueued on the library's per-process stream in call order; the
 *     only host synchronisation points are wxx_sync, wxx_memcpy_d2h and
 *     wxx_device_status.  One process drives one GPU (wxx_init(device)).
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the reference project Mo-Ehab/wxx, src/wxx/...).
 */
#ifndef WXX_CUDA_H
#define WXX_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- runtime
 * Replaces backend/device.py:9-28 (WebGPUContext), :31-141 (GPUBufferPool),
 * :144-255 (GPUCommandBuffer: batching, keep_alive, flush).                 */

const char* wxx_last_error(void);
const char* wxx_version(void);
/* No reference counterpart: kernels launched by this library so far (per process). */
int wxx_launch_count(int64_t* out);
int wxx_device_count(int* count);
/* backend/device.py:258 (module-level WebGPUContext()) */
int wxx_init(int device);
int wxx_current_device(int* device);
int wxx_num_sms(int* sms);
/* backend/device.py:40-47 create_buffer / :91-105 release */
int wxx_malloc(void** out, uint64_t nbytes);
int wxx_free(void* ptr);
/* backend/device.py:115-133 get_memory_snapshot: out[0] active bytes, out[1] live
 * blocks, out[2] pool reserved bytes, out[3] peak active, out[4] allocs, out[5] frees */
int wxx_mem_stats(int64_t* out6);
/* backend/device.py:135-141 clear_cache */
int wxx_mem_trim(void);
/* No reference counterpart: restarts the peak of wxx_mem_stats at the active bytes. */
int wxx_mem_reset_peak(void);
int wxx_host_alloc(void** out, uint64_t nbytes);          /* pinned host memory */
int wxx_host_free(void* ptr);
/* Tensor.py:66-90 (buffer upload), Tensor.py:552-569 read_buffer */
int wxx_memcpy_h2d(void* dst, const void* src, uint64_t nbytes);
int wxx_memcpy_d2h(void* dst, const void* src, uint64_t nbytes);
int wxx_memcpy_d2h_async(void* dst, const void* src, uint64_t nbytes);
int wxx_memcpy_d2d(void* dst, const void* src, uint64_t nbytes);
int wxx_memset(void* dst, int value, uint64_t nbytes);
/* backend/device.py:208-247 flush(wait=True) */
int wxx_sync(void);
void* wxx_get_stream(void);
int wxx_set_stream(void* stream);
/* No reference counterpart (kernels have no error channel there): reads and
 * clears the device error word (1 = bounded wait expired, 2 = index out of range). */
int wxx_device_status(int* code);
/* No reference counterpart: self-test of the device failure path.  One CTA runs the
 * tensor-core kernels' bounded mbarrier wait with a limit of limit_ns (0 < limit <= 10 s) on a
 * barrier that receives its arrival only when `arrive` is 1.  *result_dev (a device int) = 1
 * when the wait completed, 0 when it gave up; giving up sets the device error word to 1
 * (bounded wait expired), read and cleared by wxx_device_status. */
int wxx_wait_probe(int arrive, int64_t limit_ns, int* result_dev);
/* No reference counterpart (the reference has no sanitizer mode): check mode on / off.  After
 * every kernel launch the library then waits for the kernel and reads the device error word,
 * so the launching call returns WXX_E_TIMEOUT (expired bounded wait) or WXX_E_ARG (index
 * outside its table) naming its source line.  Also enabled by WXX_CHECK=1 at wxx_init. */
int wxx_set_check_mode(int on);
int wxx_get_check_mode(int* on);
/* No reference counterpart (the reference has no tracing): NVTX range push / pop around a
 * functional call (the Python side does it for every op when WXX_NVTX=1). */
int wxx_nvtx_push(const char* name);
int wxx_nvtx_pop(void);
int wxx_event_create(void** ev);
int wxx_event_destroy(void* ev);
int wxx_event_record(void* ev);
int wxx_event_elapsed_ms(void* start, void* stop, float* ms);
/* CUDA graphs.  The closest reference counterpart is backend/device.py:144-255
 * (GPUCommandBuffer records dispatches and submits them as one batch); here a
 * whole step is recorded once and replayed.  wxx_graph_begin opens a capture of
 * the library stream with an arena of arena_bytes that serves every wxx_malloc
 * until wxx_graph_end (fixed addresses for every replay; arena blocks freed
 * after the capture stay reserved until wxx_graph_destroy).  Host
 * synchronisation inside a capture fails it.  wxx_graph_stats: out[0] arena
 * bytes, out[1] peak bytes used in the capture, out[2] kernels per replay. */
int wxx_graph_begin(uint64_t arena_bytes, void** handle);
int wxx_graph_end(void* handle);
int wxx_graph_launch(void* handle);
int wxx_graph_stats(void* handle, int64_t* out3);
int wxx_graph_destroy(void* handle);

/* ---------------------------------------------------------------- elementwise */

/* functional/pointwise.py:29-98 pointwise (pointwise.wgsl) and :232-291
 * _pointwise (in place when out == a).  op: 0 add, 1 sub, 2 mul, 3 div. */
int wxx_binary(float* out, const float* a, int64_t a_off, const int64_t* stride_a,
               const float* b, int64_t b_off, const int64_t* stride_b, int rank,
               const int64_t* shape, int op);
/* functional/pointwise.py:101-146 scalarpointwise.  op: 0 add, 1 sub, 2 mul, 3 pow, 4 div;
 * op 5 is functional/utils.py:585-616 masked_fill (maskedfill.wgsl): x != 0 ? x : c. */
int wxx_scalar(float* out, const float* x, int64_t n, int op, float c, int reverse);
/* functional/pointwise.py:149-178 clamp (clamp.wgsl) */
int wxx_clamp(float* out, const float* x, int64_t n, float lo, float hi);
/* functional/activations.py:22-120 and functional/pointwise.py:294-355 via
 * backend/dispatch.py:59-89 _unary_op.  op: 0 relu, 1 gelu (tanh form, +-10 clamps),
 * 2 sigmoid (input clamped to +-88), 3 sin, 4 cos, 5 exp, 6 log, 7 sqrt, 8 rsqrt,
 * 9 abs, 10 sign, 11 negate, 12 square, 13 silu, 14 selu. */
int wxx_unary(float* out, const float* x, int64_t n, int op);
/* functional/utils.py:316-369 contiguous (contiguous.wgsl), :29-101 assign
 * (assign.wgsl), functional/fft.py:295-342 complex_contiguous.  elem_bytes 4 or 8. */
int wxx_strided_copy(void* dst, int64_t dst_off, const int64_t* dst_stride, const void* src,
                     int64_t src_off, const int64_t* src_stride, int rank, const int64_t* shape,
                     int elem_bytes);
/* functional/utils.py:36-55 assign with a scalar value */
int wxx_strided_fill(void* dst, int64_t dst_off, const int64_t* dst_stride, int rank,
                     const int64_t* shape, uint32_t value_bits);
/* functional/layers.py:161-206 embed (embed.wgsl) */
int wxx_embed(float* out, const uint32_t* ids, const float* weight, int64_t n_tokens, int dim,
              uint32_t vocab);
/* functional/convolution.py:1188-1257 causal_conv1d (causal_conv1d.wgsl) */
int wxx_causal_conv1d(float* out, const float* x, int64_t x_off, int64_t sb, int64_t sc,
                      int64_t sl, const float* w, const float* bias, int B, int D, int L, int K);
/* functional/pointwise.py:357-404 decay_window (decay_window.wgsl) */
int wxx_decay_window(float* out, const float* decay, int rows, int channels, int length,
                     int stage);
/* nn/module.py MultiHeadAttention q/k/v weights (module.py:447-495, each (K, N)) transposed and
 * stacked in one launch into the (n*N, K) K-major operand of the fused QKV projection:
 * dst[b*cols + c, r] = srcs[b][r, c]; srcs is a host array of n <= 8 device pointers to dense
 * (rows, cols) arrays.  round_tf32 = 1 stores the values rounded to the nearest TF32 value. */
int wxx_transpose_stack(float* dst, const float* const* srcs, int n, int rows, int cols,
                        int round_tf32);
/* No reference counterpart: dst[0..n) = src[0..n) rounded to the nearest TF32 value (a weight
 * copy read only by TF32 products, e.g. the tied LM head of nn/gpt.py). */
int wxx_round_tf32(float* dst, const float* src, int64_t n);
/* nn/hyena.py:127-130 ImplicitFilter.forward (Linear -> Sine(omega) -> Linear over the positional
 * encoding, transposed) and :236-239 (h * decay_window) for all `n` filters of an operator in one
 * launch, exact fp32: out (n, D, L) dense, filter i = (sin(omega * (pe @ w1[i] + b1[i])) @ w2[i]
 * + b2[i])^T * exp(-|decay[i, d]| * t).  pe (L, F); w1[i] (F, H), b1[i] (H), w2[i] (H, D),
 * b2[i] (D) device arrays passed as host arrays of n device pointers; decay (n, D).  n <= 8,
 * F <= 32, H <= 64 and a multiple of 4, else WXX_E_UNSUPPORTED with nothing enqueued. */
int wxx_hyena_filters(float* out, const float* pe, int L, int F, int H, int D, int n,
                      const float* const* w1, const float* const* b1, const float* const* w2,
                      const float* const* b2, float omega, const float* decay);
/* functional/fft.py:168-213 complex_mul (complex_mul.wgsl) */
int wxx_complex_mul(void* out, const void* a, int64_t a_off, const int64_t* stride_a,
                    const void* b, int64_t b_off, const int64_t* stride_b, int rank,
                    const int64_t* shape, int conj_a, int conj_b);
/* functional/fft.py:344-383 complex_conj / complex_add_inplace */
int wxx_complex_conj(void* out, const void* x, int64_t n);
int wxx_complex_add_inplace(void* acc, const void* x, int64_t n);
/* functional/utils.py:509-582 equal / equal_number (equal.wgsl) */
int wxx_equal(float* out, const void* a, const void* b, int64_t n, int mode, uint32_t number);

/* ---------------------------------------------------------------- reductions / norms */

/* functional/reductions.py:27-197 sum / mean / sumsq (reduce.wgsl) with the
 * (outer, reduce, inner) mapping of backend/dispatch.py:173-214.  mode 0 sum, 1 mean, 2 sumsq. */
int wxx_reduce(float* out, const float* x, int64_t outer, int64_t reduce, int64_t inner, int mode);
/* functional/reductions.py:241-342 max / min (reduce_minmax.wgsl), op 0 max, 1 min;
 * indices follow the reference's tie rule bit for bit. */
int wxx_argminmax(float* vals, uint32_t* idx, const float* x, int64_t outer, int64_t reduce,
                  int64_t inner, int op);
/* functional/activations.py:126-173 softmax (softmax.wgsl) */
int wxx_softmax(float* y, const float* x, int64_t outer, int64_t n, int64_t inner);
/* nn/module.py:484-488 (score + mask, then softmax) fused: row r uses mask row r % mask_rows. */
int wxx_softmax_masked(float* y, const float* x, int64_t rows, int64_t n, const float* mask,
                       int64_t mask_ld, int64_t mask_rows);
/* functional/normalization.py:82-145 meanvarnorm (meanvarnorm.wgsl), eps 1e-5.
 * out_tf32 = 1 stores y rounded to the nearest TF32 value (for a y that only feeds TF32
 * products, e.g. the LayerNorm before a projection); 0 stores the fp32 result. */
int wxx_layernorm(float* y, float* mean, float* inv_std, const float* x, const float* gamma,
                  const float* beta, int64_t outer, int64_t n, int64_t inner, float eps,
                  int out_tf32);
/* functional/normalization.py:24-79 rmsnorm (rmsnorm.wgsl), eps 1e-6; out_tf32 as above */
int wxx_rmsnorm(float* y, float* inv_rms, const float* x, const float* gamma, int64_t outer,
                int64_t n, int64_t inner, float eps, int out_tf32);
/* functional/normalization.py:148-206 batchnorm (batchnorm.wgsl) */
int wxx_batchnorm(float* y, float* saved_mean, float* saved_inv, const float* x,
                  const float* gamma, const float* beta, float* running_mean, float* running_var,
                  int B, int C, int64_t hw, float eps, float momentum, int training);

/* ---------------------------------------------------------------- contractions */

/* functional/utils.py:378-499 matmul_add (matmul.wgsl).  C dense [batch, M, N].
 * trans_a: element (m, k) at A[b*a_bs + k*lda + m]; else A[b*a_bs + m*lda + k].
 * trans_b: element (k, n) at B[b*b_bs + n*ldb + k]; else B[b*b_bs + k*ldb + n].
 * a_bs/b_bs = 0 broadcasts over the batch.  bias_mode 0 none, 1 (N,), 2 (M,N), 3 (batch,M,N).
 * mode 0 TF32 tcgen05, 1 3xTF32 tcgen05, 2 fp32 SIMT, 3 TF32 tcgen05 with C rounded to the
 * nearest TF32 value.  C = alpha * op(A) op(B) + bias. */
int wxx_matmul(float* C, const float* A, const float* B, const float* bias, int64_t batch,
               int64_t M, int64_t N, int64_t K, int64_t a_bs, int64_t b_bs, int64_t lda,
               int64_t ldb, int trans_a, int trans_b, int bias_mode, float alpha, int mode);
/* nn/module.py Linear.forward followed by GELU (shaders/activations/gelu.wgsl)
 * or by the block's residual add (functional/pointwise.py:29 add), fused into
 * the GEMM epilogue: C = act(alpha * A @ op(B) + bias) + residual.
 * A (M, K) row stride lda; B (K, N) row stride ldb, or (N, K) with trans_b = 1;
 * bias (N) or NULL; residual (M, N dense) or NULL; act 0 none, 1 GELU (tanh).
 * mode 0 TF32, 1 3xTF32, 3 TF32 with C rounded to the nearest TF32 value (for a C read only
 * by TF32 products).  C 16-byte aligned, N a multiple of 4. */
int wxx_linear(float* C, const float* A, const float* B, const float* bias,
               const float* residual, int64_t M, int64_t N, int64_t K, int64_t lda,
               int64_t ldb, int trans_b, int act, float alpha, int mode);
/* Row-wise argmax of op(A) @ op(B) without storing the product (GPT2's forward when its output
 * is the next-token id of every position): idx[b*M + m] (u32) and vals (or NULL) get the index
 * and value wxx_argminmax (op 0) would return on the stored product; arguments as wxx_matmul
 * (no bias, alpha 1, mode 0..2).  Large TMA-addressable products keep each row's maximum per
 * 256-column tile in the SM-pair GEMM's epilogue; others go through scratch. */
int wxx_matmul_argmax(uint32_t* idx, float* vals, const float* A, const float* B, int64_t batch,
                      int64_t M, int64_t N, int64_t K, int64_t a_bs, int64_t b_bs, int64_t lda,
                      int64_t ldb, int trans_a, int trans_b, int mode);
/* The decode step's LayerNorm -> linear (nn/gpt.py: ln1 -> q/k/v, ln2 -> fc1, ln_f -> head) in
 * one launch for 1 <= M <= 32 rows: C (M, N) = act(LayerNorm(A) @ W^T + bias) + residual with
 * W (N, K) K-major, gamma / beta (K), act 0 / 1 (GELU), round_out = 1 stores C rounded to the
 * nearest TF32 value; exact fp32.  WXX_E_UNSUPPORTED (nothing enqueued) outside N >= 64,
 * K >= 128, K / lda / ldw multiples of 4, 16-byte aligned A, W, gamma, beta. */
int wxx_ln_linear(float* C, const float* A, int64_t lda, const float* gamma, const float* beta,
                  float eps, const float* W, int64_t ldw, const float* bias,
                  const float* residual, int64_t M, int64_t N, int64_t K, int act,
                  int round_out);
/* nn/hyena.py:242 out_proj(z.transpose(1, 2)): wxx_linear over a batch whose A operand is a
 * strided view, A[b] at A + b*a_bs with row stride lda, transposed when trans_a (A[b] stored
 * (K, M)), B shared by the batch, residual (batch, M, N) dense or NULL; act 0 or 1. */
int wxx_linear_batched(float* C, const float* A, const float* B, const float* bias,
                       const float* residual, int64_t batch, int64_t M, int64_t N, int64_t K,
                       int64_t a_bs, int64_t lda, int trans_a, int64_t ldb, int trans_b, int act,
                       float alpha, int mode);
/* nn/hyena.py:227-234 (HyenaOperator.forward): v = short_conv(proj_v(x).transpose(1, 2)) and
 * the gates short_conv(chunk(proj_x(x))[i].transpose(1, 2)) in one tcgen05 GEMM whose epilogue
 * applies the causal taps (CausalShortConv1d, nn/hyena.py:77-99) and writes channels first.
 * Y (M, N) = A @ op(B) + bias with row = b * seq_len + n (M a multiple of seq_len);
 * out[b, c, n] (M/seq_len, N, seq_len dense) = conv_b[c'] + sum_{k < conv_k, k <= n}
 * conv_w[c', k] * Y[row - k, c], c' = c % conv_ch.  A (M, K) row stride lda; B (K, N) row
 * stride ldb, or (N, K) with trans_b; bias (N) or NULL; conv_k 1..4; mode 0 TF32, 1 3xTF32
 * (K <= 1024).  WXX_E_UNSUPPORTED, nothing enqueued, when A or B is not TMA-addressable. */
int wxx_linear_short_conv(float* out, const float* A, const float* B, const float* bias, int64_t M,
                          int64_t N, int64_t K, int64_t lda, int64_t ldb, int trans_b,
                          int64_t seq_len, const float* conv_w, const float* conv_b, int conv_ch,
                          int conv_k, int mode);
/* functional/convolution.py:658-729 conv2d (conv2d.wgsl), NCHW implicit GEMM on tcgen05.
 * mode 0 TF32, 1 or 2 3xTF32. */
int wxx_conv2d(float* Y, const float* X, const float* W, const float* bias, int B, int Cin,
               int H, int Wd, int Cout, int KH, int KW, int sh, int sw, int ph, int pw, int dh,
               int dw, int mode);
/* nn/resnet.py:31-79 ResBlock's conv -> BatchNorm (eval, functional/normalization.py:148-206)
 * (-> + shortcut) -> relu in the conv's epilogue: Y = relu?(bn(conv(X) + bias) + residual).
 * rm == NULL: no batchnorm; residual NCHW like Y or NULL; relu 0/1.  Same values as the
 * separate kernels. */
int wxx_conv2d_bn(float* Y, const float* X, const float* W, const float* bias, int B, int Cin,
                  int H, int Wd, int Cout, int KH, int KW, int sh, int sw, int ph, int pw, int dh,
                  int dw, int mode, const float* rm, const float* rv, const float* gamma,
                  const float* beta, float eps, const float* residual, int relu);
/* The same convolution + follow-up ops on channels-last tensors: X (B, H, W, Cin) NHWC,
 * W (Cout, Cin, KH, KW) as above, residual and Y (B, Ho, Wo, Cout) NHWC.  The A operand is
 * fetched by 4-D TMA boxes (one filter tap x 32 channels x a 128-pixel output tile per
 * K-block).  Needs Cin % 32 == 0, Cout % 4 == 0, 16-byte aligned X / Y and 128-pixel output
 * tiles that are boxes (Wo a multiple of 128, or Wo | 128 and Ho a multiple or divisor of
 * 128 / Wo); else WXX_E_ARG.  No reference counterpart for the layout (the reference is NCHW
 * throughout); ResNet uses it between its stem and its pooling. */
int wxx_conv2d_nhwc(float* Y, const float* X, const float* W, const float* bias, int B, int Cin,
                    int H, int Wd, int Cout, int KH, int KW, int sh, int sw, int ph, int pw,
                    int dh, int dw, int mode, const float* rm, const float* rv,
                    const float* gamma, const float* beta, float eps, const float* residual,
                    int relu);
/* wxx_conv2d_nhwc with Wp already in the convolution's K order, (Cout, KH*KW, Cin), as written
 * by wxx_conv_weight_pack: no per-call reorder launch. */
int wxx_conv2d_nhwc_packed(float* Y, const float* X, const float* Wp, const float* bias, int B,
                           int Cin, int H, int Wd, int Cout, int KH, int KW, int sh, int sw,
                           int ph, int pw, int dh, int dw, int mode, const float* rm,
                           const float* rv, const float* gamma, const float* beta, float eps,
                           const float* residual, int relu);
/* nn/resnet.py forward (channels-last stages): the weights of up to 24 convolutions
 * (nn/module.py Conv2d.W, (cout, cin, taps)) reordered to (cout, taps, cin) in one launch;
 * dst, src, cout, cin, taps are host arrays of n entries (device pointers for dst / src);
 * cin * taps <= 51200. */
int wxx_conv_weight_pack(float* const* dst, const float* const* src, const int* cout,
                         const int* cin, const int* taps, int n);
/* nn/resnet.py forward stem: conv 7x7 / stride 2 / pad 3 (Cin 1..4 -> 64, H, W <= 32) + bias
 * (or NULL) + eval batchnorm (rm == NULL: none) + ReLU (relu = 1) + max pool 3x3 / stride 2 /
 * pad 1, stored channels-last Y (B, Hp, Wp, 64); one launch, values equal to the separate ops.
 * Wt (64, Cin, 7, 7), or with packed = 1 transposed to (Cin * 49, 64), 16-byte aligned. */
int wxx_resnet_stem(float* Y, const float* X, const float* Wt, const float* bias,
                    const float* rm, const float* rv, const float* gamma, const float* beta,
                    float eps, int relu, int B, int Cin, int H, int W, int packed);

/* nn/module.py:460-495 MultiHeadAttention core fused (QK^T * scale (+ mask), softmax, PV)
 * on tcgen05.  Q (B, Sq, H, hd) row stride q_ld, K/V (B, Sk, H, hd) row stride kv_ld,
 * O (B, Sq, H, hd) row stride o_ld; hd 32 or 64; causal masks keys after the query.
 * mode 0: TF32 products; out_tf32 = 1 stores O rounded to the nearest TF32 value (an O read
 * only by TF32 products).  mode 1: 3xTF32 products (fp32-faithful), out_tf32 ignored. */
int wxx_attention(float* O, const float* Q, const float* K, const float* V, int B, int H, int Sq,
                  int Sk, int hd, int64_t q_ld, int64_t kv_ld, int64_t o_ld, float scale,
                  const float* mask, int64_t mask_ld, int causal, int out_tf32, int mode);

/* ---------------------------------------------------------------- pooling */

/* functional/convolution.py:60-125 maxpool2d (maxpool2d.wgsl); idx may be NULL */
int wxx_maxpool2d(float* Y, uint32_t* idx, const float* X, int B, int C, int H, int W, int KH,
                  int KW, int sh, int sw, int ph, int pw);
/* functional/convolution.py:490-543 adaptive_avgpool2d (adaptive_avgpool2d.wgsl) */
int wxx_adaptive_avgpool2d(float* Y, const float* X, int B, int C, int H, int W, int Ho, int Wo);

/* ---------------------------------------------------------------- FFT */

/* functional/fft.py:484-563 rfft (fft_bitrev_real / fft_stage / fft_copy_out / fft_wg_real) */
int wxx_rfft(void* X, int64_t out_ld, const float* x, int64_t in_ld, int64_t rows, int64_t in_len,
             int64_t n);
/* functional/fft.py:566-645 irfft (fft_bitrev_complex / fft_stage / ifft_write_real / fft_wg_inverse) */
int wxx_irfft(float* y, int64_t out_ld, const void* X, int64_t in_ld, int64_t rows,
              int64_t in_len, int64_t n);
/* nn/hyena.py:208-216 HyenaOperator.fft_conv1d = irfft(rfft(x, n) * H, n)[..., :out_len]
 * with a precomputed filter spectrum H (D, n/2+1). */
int wxx_fftconv_spectrum(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                         int64_t sl, const void* H, int64_t h_ld, int B, int D, int L, int64_t n,
                         int out_len);
/* nn/hyena.py:240 gates[i] * fft_conv1d(z, h) with a precomputed spectrum H (D rows of h_ld
 * complex values, n/2+1 used): wxx_fftconv_spectrum with the gate view of wxx_fftconv_gated
 * applied as the output is stored. */
int wxx_fftconv_spectrum_gated(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                               int64_t sl, const void* H, int64_t h_ld, int B, int D, int L,
                               int64_t n, int out_len, const float* gate, int64_t g_off,
                               int64_t g_sb, int64_t g_sd, int64_t g_sl);
/* nn/hyena.py:208-216 fft_conv1d with a time-domain filter h (D, Lh) */
int wxx_fftconv(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd, int64_t sl,
                const float* h, int64_t h_ld, int Lh, int B, int D, int L, int64_t n, int out_len);
/* nn/hyena.py:240 z = gates[i] * fft_conv1d(z, h): wxx_fftconv whose output is
 * multiplied by a strided (B, D, out_len) gate view (element strides g_sb,
 * g_sd, g_sl from g_off) as it is stored. */
int wxx_fftconv_gated(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                      int64_t sl, const float* h, int64_t h_ld, int Lh, int B, int D, int L,
                      int64_t n, int out_len, const float* gate, int64_t g_off, int64_t g_sb,
                      int64_t g_sd, int64_t g_sl);
/* No counterpart in the reference.  wxx_fftconv without any allocation: the
 * filter spectrum lives in a fixed device array inside the library (32 MiB +
 * 4 KiB, rows n/2+2 complex values apart).  Limits: n <= 32768,
 * D*(n/2+2) <= 4194816 complex values (256 rows at n = 32768) and
 * 0 <= out_len <= n, else WXX_E_ARG and nothing is launched.  The scratch needs no zeroing (each call writes it
 * before reading it).  One array per device: calls that overlap on the device
 * (other streams or threads) race on it.  The first call on a device looks up
 * the array's address (cudaGetSymbolAddress, may load device code); make it
 * before any stream capture. */
int wxx_fftconv_static(float* y, const float* x, int64_t x_off, int64_t sb, int64_t sd,
                       int64_t sl, const float* h, int64_t h_ld, int Lh, int B, int D, int L,
                       int64_t n, int out_len);

/* ---------------------------------------------------------------- generation
 * nn/gpt.py:108-170 GPT2.generate, on the device: a prefill forward fills per-layer K / V
 * caches (B, max_len, D); each later token is one decode step of the new position, replayed
 * from a CUDA graph, with the current length *cur_len (an int in device memory) read and
 * advanced on the device. */
/* out (B, D) = tok_emb[ids[b, p]] + pos_emb[p], p = *cur_len - 1 (nn/gpt.py:101-103 for the
 * last position); ids row stride ids_ld. */
int wxx_decode_embed(float* out, const uint32_t* ids, int64_t ids_ld, const int* cur_len,
                     const float* tok_emb, const float* pos_emb, int B, int D, int vocab,
                     int max_len);
/* nn/module.py:460-495 for one query row per sequence: appends position p = *cur_len - 1's
 * k_new / v_new (row b at b * qkv_ld) to Kc / Vc (B, max_len, D = H * hd, batch stride
 * cache_bs), then O[b] (row stride o_ld) = softmax(scale q . K^T) V over positions 0..p in
 * exact fp32; hd 32 or 64; out_tf32 = 1 stores O rounded to the nearest TF32 value. */
int wxx_decode_attention(float* O, int64_t o_ld, const float* q, const float* k_new,
                         const float* v_new, int64_t qkv_ld, float* Kc, float* Vc,
                         int64_t cache_bs, int B, int H, int hd, const int* cur_len, int max_len,
                         float scale, int out_tf32);
/* nn/gpt.py:147-163 next-token choice for B rows of logits (row stride ld, V entries):
 * temperature 0 -> first index of the maximum; else top_k (0 = none; values below the k-th
 * largest dropped) and the first index whose float64 softmax cumulative probability exceeds
 * draws[b] (0 if none).  Writes ids[b, *cur_len] and advances *cur_len; done_count is a device
 * counter that starts at 0 and is left at 0. */
int wxx_sample_tokens(uint32_t* ids, int64_t ids_ld, int* cur_len, unsigned* done_count,
                      const float* logits, int64_t ld, int B, int V, float temperature, int top_k,
                      const double* draws, int max_len);

/* ---------------------------------------------------------------- training
 * Backward passes, loss and optimiser of GPT2 training (src/wxx/autograd/*.py backward
 * methods); matmul / linear gradients use wxx_matmul, bias and affine gradients wxx_reduce. */
/* gelubackwards.wgsl times grad_output: dx = dy * gelu'(x) (tanh form, +-10 clamps). */
int wxx_gelu_backward(float* dx, const float* dy, const float* x, int64_t n);
/* softmaxbackwards.wgsl over the last axis: dx = y * (dy - sum(dy * y)); rows of n <= 1024. */
int wxx_softmax_backward(float* dx, const float* dy, const float* y, int64_t rows, int64_t n);
/* meanvarnormdx / meanvarnormdg (autograd/normalization.py meanvarnorm.backward): dx from the
 * saved mean and inv_std, and dyxhat = dy * xhat whose column sums are d gamma; n <= 1024. */
int wxx_layernorm_backward(float* dx, float* dyxhat, const float* dy, const float* x,
                           const float* mean, const float* inv, const float* gamma, int64_t rows,
                           int64_t n);
/* embeddx.wgsl (autograd/layers.py Embedding.backward): dW (vocab, D) = scatter-add of dY rows. */
int wxx_embedding_backward(float* dW, const uint32_t* ids, const float* dY, int64_t n_tokens,
                           int D, int vocab);
/* functional/loss.py:20 cceloss (cceloss.wgsl): per-row loss and dZ = softmax - onehot. */
int wxx_cceloss(float* loss, float* dZ, const float* Z, const uint32_t* targets, int64_t rows,
                int K);
/* nn/optimizer.py:38-84 AdamW.step / adamw.wgsl: one step over n parameters in place. */
int wxx_adamw(float* p, const float* g, float* m, float* v, int64_t n, float lr, float beta1,
              float beta2, float eps, float weight_decay, float bc1, float bc2);
/* nn/optimizer.py AdamW.step with device-resident bias corrections (bc: two floats
 * {bc1, bc2}), so a training step recorded as a CUDA graph replays with each step's own. */
int wxx_adamw_device(float* p, const float* g, float* m, float* v, int64_t n, float lr,
                     float beta1, float beta2, float eps, float weight_decay, const float* bc);
/* wxx_adamw_device over n parameters, one launch per 128 of them: p, g, m, v are host arrays
 * of n device pointers, len their element counts; the pointers are kernel arguments, so a
 * step recorded in a CUDA graph replays with the same tensors. */
int wxx_adamw_device_multi(int n, float* const* p, const float* const* g, float* const* m,
                           float* const* v, const int64_t* len, float lr, float beta1,
                           float beta2, float eps, float weight_decay, const float* bc);
/* step (one device int) += 1, then bc = {1 - beta1^step, 1 - beta2^step} (computed in double). */
int wxx_adamw_advance(int* step, float* bc, double beta1, double beta2);

/* ---------------------------------------------------------------- NCCL
 * No reference counterpart (the reference drives one WebGPU device): the
 * all-gather of batch-sharded outputs across the GPUs of one node. */
int wxx_nccl_unique_id(uint8_t* out128);
int wxx_nccl_init(const uint8_t* id128, int nranks, int rank);
int wxx_nccl_allgather(void* recv, const void* send, uint64_t nbytes);
/* The all-gather on a separate communication stream, ordered after the work already on the
 * library stream; the library stream keeps computing.  wxx_nccl_wait(slot) makes the library
 * stream wait for the last gather issued with that slot (0..3).  Both buffers must stay
 * allocated until that wait is enqueued. */
int wxx_nccl_allgather_async(void* recv, const void* send, uint64_t nbytes, int slot);
int wxx_nccl_wait(int slot);
int wxx_nccl_async_error(int* code);
int wxx_nccl_destroy(int abort);

#ifdef __cplusplus
}
#endif

#endif /* WXX_CUDA_H */
