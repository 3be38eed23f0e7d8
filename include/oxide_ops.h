/*
 * oxide_ops.h -- C ABI of the B200 (sm_100a) tensor-op library.
 *
 * Drop-in boundary for mistralrs-oxide's tensor-op hot path: the elementwise,
 * broadcast and row-reduction ops in src/ops that src/layers calls for every
 * Mistral decoder layer, and the launch_* methods of
 * src/cuda_backend/kernels.rs (KernelManager) that were meant to run them on
 * the GPU.  A Rust (or any C-FFI) caller binds these symbols directly.
 *
 * Conventions (all entry points):
 *   - Pointers are device pointers unless the name says `host`.  The caller
 *     owns every buffer; nothing here allocates, frees or synchronises.
 *   - Work is enqueued on `stream` (NULL = legacy default stream) and returns
 *     immediately, like cudarc's CudaFunction::launch.
 *   - Tensors are contiguous row-major.  bf16 tensors are raw 16-bit
 *     patterns (`oxide_bf16`).
 *   - A size of 0 elements or rows is a valid no-op.
 *   - The return value is an oxide_status: 0 on success, a negative code
 *     otherwise; oxide_last_error() gives the message of the calling thread's
 *     last failure.  No entry point aborts the process.
 *   - Outputs may alias inputs element-for-element (in-place use) unless the
 *     entry point says otherwise.
 *   - Arithmetic follows the reference's sequential f32 formulas with IEEE
 *     rounding at every step (no FMA contraction, IEEE divide and sqrt).  bf16
 *     operands are widened to f32, and each tensor the reference materialises
 *     is rounded to bf16 (nearest-even) once at its store.
 */
#ifndef OXIDE_OPS_H
#define OXIDE_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* oxide_stream_t; /* identical to cudaStream_t */
typedef uint16_t oxide_bf16;

/* Status codes.  They mirror the error classes of
 * src/cuda_backend/errors.rs:10-31 (CudaError) and src/error.rs:3-45
 * (OxideError::InvalidArgument / UnsupportedOperation / CudaError). */
typedef enum {
    OXIDE_OK = 0,
    OXIDE_ERR_INVALID_ARG = -1,  /* null pointer, bad size, size overflow      */
    OXIDE_ERR_LAUNCH = -2,       /* kernel launch failed (cudaGetLastError)   */
    OXIDE_ERR_UNSUPPORTED = -3,  /* shape or device this build cannot run     */
    OXIDE_ERR_CUDA = -4,         /* other CUDA runtime error                  */
    OXIDE_ERR_WORKSPACE = -5,    /* workspace missing or too small            */
    OXIDE_ERR_INJECTED = -6,     /* failure injected by oxide_debug_fail_next */
    OXIDE_ERR_TIMEOUT = -7       /* bounded host wait expired                 */
} oxide_status;

/* Binary operator selector for oxide_binary_*. */
typedef enum { OXIDE_ADD = 0, OXIDE_SUB = 1, OXIDE_MUL = 2, OXIDE_DIV = 3 } oxide_binop;

/* Reduction selector for oxide_reduce_*. */
typedef enum { OXIDE_RED_SUM = 0, OXIDE_RED_MAX = 1, OXIDE_RED_SUMSQ = 2 } oxide_redop;

/* Unary operator selector for oxide_unary_*. */
typedef enum {
    OXIDE_RELU = 0,       /* max(x, 0); NaN -> 0 like f32::max          */
    OXIDE_GELU = 1,       /* tanh form, src/ops/activation.rs:39-56     */
    OXIDE_GELU_QUICK = 2, /* x * sigmoid(1.702 x), activation.rs:58-74  */
    OXIDE_SIGMOID = 3,    /* 1 / (1 + exp(-x)), activation.rs:126-140   */
    OXIDE_TANH = 4,       /* activation.rs:142-156                      */
    OXIDE_EXP = 5,        /* src/ops/math.rs:4-19                       */
    OXIDE_LOG = 6,        /* natural log, math.rs:21-36                 */
    OXIDE_SQRT = 7,       /* math.rs:38-53                              */
    OXIDE_POW = 8,        /* powf(x, a), math.rs:55-70                  */
    OXIDE_CLAMP = 9,      /* clamp(x, a, b), a <= b, math.rs:72-87      */
    OXIDE_NEG = 10,       /* math.rs:89-104                             */
    OXIDE_ABS = 11        /* math.rs:106-121                            */
} oxide_unop;

/* ---- library / status --------------------------------------------------- */

/* Human-readable name of a status code (never NULL). */
const char* oxide_status_string(int status);
/* Message of the calling thread's most recent failure ("" if none). */
const char* oxide_last_error(void);
/* Library version string. */
const char* oxide_version(void);
/* Self-test of the row-shared division used by RMSNorm and softmax (a
 * correctly rounded reciprocal plus FMA residual corrections): compares it
 * with the IEEE quotient a[i] / b[j] for every pair.  out (device, 2 x u64)
 * must hold {0, UINT64_MAX}; it receives the mismatch count and the smallest
 * mismatching pair index i * nb + j.  Diagnostic; no reference counterpart. */
int oxide_selftest_rowdiv(const float* a, uint64_t na, const float* b, uint64_t nb,
                          unsigned long long* out, oxide_stream_t stream);
/* Host-side fault injection for tests: the next call of entry point `op`
 * (e.g. "oxide_rms_norm_f32"; "*" = any) made by any thread returns
 * OXIDE_ERR_INJECTED before launching anything.  NULL clears. */
void oxide_debug_fail_next(const char* op);

/* ---- elementwise binary with broadcast ------------------------------------
 * Replaces src/ops/matmul.rs:74-134 (add/mul/sub/div) whose loop body is
 * elementwise_op_cpu, src/ops/matmul.rs:136-158:
 *     out[i] = a[i % na] op b[i % nb],  i in [0, n)
 * and KernelManager::launch_vecadd / launch_sub / launch_mul / launch_div
 * (src/cuda_backend/kernels.rs:75-156, na = nb = n).  A row-broadcast
 * multiply x[rows, cols] * s[cols] is na = rows*cols, nb = cols. */
int oxide_binary_f32(int op, const float* a, uint64_t na, const float* b, uint64_t nb,
                     float* out, uint64_t n, oxide_stream_t stream);
int oxide_binary_bf16(int op, const oxide_bf16* a, uint64_t na, const oxide_bf16* b,
                      uint64_t nb, oxide_bf16* out, uint64_t n, oxide_stream_t stream);

/* Named forms of oxide_binary_* with na = nb = n for add, sub and div
 * (KernelManager::launch_vecadd/sub/div, kernels.rs:75,96,138) and the
 * trailing-dimension broadcast for mul (ops::mul(x[rows,cols], s[cols]),
 * matmul.rs:97-108; launch_mul kernels.rs:117 is rows = 1). */
int oxide_add_f32(const float* a, const float* b, float* out, uint64_t n, oxide_stream_t stream);
int oxide_add_bf16(const oxide_bf16* a, const oxide_bf16* b, oxide_bf16* out, uint64_t n,
                   oxide_stream_t stream);
int oxide_sub_f32(const float* a, const float* b, float* out, uint64_t n, oxide_stream_t stream);
int oxide_div_f32(const float* a, const float* b, float* out, uint64_t n, oxide_stream_t stream);
int oxide_mul_rowbcast_f32(const float* x, const float* s, float* out, uint64_t rows,
                           uint64_t cols, oxide_stream_t stream);
int oxide_mul_rowbcast_bf16(const oxide_bf16* x, const oxide_bf16* s, oxide_bf16* out,
                            uint64_t rows, uint64_t cols, oxide_stream_t stream);
/* out = (a + b) * s[col] over a, b [rows, cols]: the residual add followed by
 * the row-broadcast multiply (ops::add then ops::mul, matmul.rs:74-108) in one
 * pass.  The sum is rounded to the I/O type before the multiply, so the result
 * equals oxide_add_* then oxide_mul_rowbcast_* bit for bit; the sum is not
 * stored.  out may alias a or b (in place); it must not overlap s, which
 * every row reads again. */
int oxide_add_mul_rowbcast_f32(const float* a, const float* b, const float* s, float* out, uint64_t rows,
                               uint64_t cols, oxide_stream_t stream);
int oxide_add_mul_rowbcast_bf16(const oxide_bf16* a, const oxide_bf16* b, const oxide_bf16* s,
                                oxide_bf16* out, uint64_t rows, uint64_t cols, oxide_stream_t stream);

/* out = x * scale.  Replaces KernelManager::launch_scale
 * (src/cuda_backend/kernels.rs:159-177; PTX scale_f32 build.rs:240-276). */
int oxide_scale_f32(const float* x, float* out, float scale, uint64_t n, oxide_stream_t stream);
int oxide_scale_bf16(const oxide_bf16* x, oxide_bf16* out, float scale, uint64_t n,
                     oxide_stream_t stream);

/* ---- activations -----------------------------------------------------------
 * out = x * (1 / (1 + exp(-x))).  Replaces ops::silu
 * (src/ops/activation.rs:21-37) and KernelManager::launch_silu
 * (src/cuda_backend/kernels.rs:231-248). */
int oxide_silu_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream);
int oxide_silu_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t n, oxide_stream_t stream);

/* out = silu(gate) * up in one pass.  Replaces the pair
 * silu(&gate) then ops::mul(&gated, &up) of MLP::forward
 * (src/layers/attention.rs:144-145).  The bf16 form rounds silu(gate) to
 * bf16 before the multiply, as the composed pair would, and rounds the exact
 * product of the two bf16 values once; the pair's f32 multiply rounds it
 * twice where that product is an f32 subnormal (|p| < 2^-126), so the two
 * can differ there by one bf16 ulp. */
int oxide_silu_mul_f32(const float* gate, const float* up, float* out, uint64_t n,
                       oxide_stream_t stream);
int oxide_silu_mul_bf16(const oxide_bf16* gate, const oxide_bf16* up, oxide_bf16* out,
                        uint64_t n, oxide_stream_t stream);

/* ---- unary ops -----------------------------------------------------------------
 * out[i] = op(x[i]) for the oxide_unop selector, with the scalar parameters a
 * (pow exponent, clamp minimum) and b (clamp maximum); each step rounded as the
 * reference's f32 expression (transcendentals are CUDA's expf/logf/tanhf/powf).
 * CLAMP with a > b (or a NaN bound) is OXIDE_ERR_INVALID_ARG, where the
 * reference's f32::clamp panics.  Replaces src/ops/activation.rs relu / gelu /
 * gelu_quick / sigmoid / tanh and src/ops/math.rs exp / log / sqrt / pow / clamp
 * / neg / abs; the named f32 forms replace KernelManager::launch_relu, launch_gelu,
 * launch_sigmoid and launch_tanh (src/cuda_backend/kernels.rs:211-309). */
int oxide_unary_f32(int op, const float* x, float* out, uint64_t n, float a, float b,
                    oxide_stream_t stream);
int oxide_unary_bf16(int op, const oxide_bf16* x, oxide_bf16* out, uint64_t n, float a, float b,
                     oxide_stream_t stream);
int oxide_relu_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream);
int oxide_gelu_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream);
int oxide_sigmoid_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream);
int oxide_tanh_f32(const float* x, float* out, uint64_t n, oxide_stream_t stream);

/* ---- normalisation ----------------------------------------------------------
 * Per row of x[rows, cols]: rms = sqrt(sum(x*x) / cols + eps);
 * out = (x / rms) * w.  Replaces ops::rms_norm (src/ops/norm.rs:4-51) and
 * KernelManager::launch_rms_norm (src/cuda_backend/kernels.rs:311-331). */
int oxide_rms_norm_f32(const float* x, const float* w, float* out, uint64_t rows,
                       uint64_t cols, float eps, oxide_stream_t stream);
int oxide_rms_norm_bf16(const oxide_bf16* x, const oxide_bf16* w, oxide_bf16* out,
                        uint64_t rows, uint64_t cols, float eps, oxide_stream_t stream);

/* h = x + r (stored: it is the next residual), then y = rms_norm(h, w, eps).
 * Replaces ops::add (src/layers/transformer.rs:64) followed by
 * post_attention_layernorm (transformer.rs:67); fusion intent of
 * rms_norm_fused_add_f32 (src/kernels/normalization.rs:41-77).  The norm reads
 * h as stored (bf16-rounded in the bf16 form).  h and y must not alias. */
int oxide_add_rms_norm_f32(const float* x, const float* r, const float* w, float* h, float* y,
                           uint64_t rows, uint64_t cols, float eps, oxide_stream_t stream);
int oxide_add_rms_norm_bf16(const oxide_bf16* x, const oxide_bf16* r, const oxide_bf16* w,
                            oxide_bf16* h, oxide_bf16* y, uint64_t rows, uint64_t cols,
                            float eps, oxide_stream_t stream);

/* Per row of x[rows, cols]: mean = sum(x) / cols; var = sum((x - mean)^2) / cols;
 * out = (x - mean) / sqrt(var + eps) * w + b.  Replaces ops::layer_norm
 * (src/ops/norm.rs:53-117) and KernelManager::launch_layer_norm
 * (src/cuda_backend/kernels.rs:334-356). */
int oxide_layer_norm_f32(const float* x, const float* w, const float* b, float* out, uint64_t rows,
                         uint64_t cols, float eps, oxide_stream_t stream);
int oxide_layer_norm_bf16(const oxide_bf16* x, const oxide_bf16* w, const oxide_bf16* b,
                          oxide_bf16* out, uint64_t rows, uint64_t cols, float eps,
                          oxide_stream_t stream);

/* out = layer_norm(x + r) with the same w, b and eps: the fused form of
 * layer_norm_fused_add_f32 (src/kernels/normalization.rs:123-167), one pass
 * over x and r.  The sum is rounded to the I/O type before the normalisation
 * (exact for f32), so the result equals oxide_add_* followed by
 * oxide_layer_norm_*; the sum itself is not stored.  out may alias x or r. */
int oxide_add_layer_norm_f32(const float* x, const float* r, const float* w, const float* b, float* out,
                             uint64_t rows, uint64_t cols, float eps, oxide_stream_t stream);
int oxide_add_layer_norm_bf16(const oxide_bf16* x, const oxide_bf16* r, const oxide_bf16* w,
                              const oxide_bf16* b, oxide_bf16* out, uint64_t rows, uint64_t cols, float eps,
                              oxide_stream_t stream);

/* ---- softmax ---------------------------------------------------------------
 * softmax(x, dim) of a tensor viewed as [outer, dim, inner] (inner = product
 * of the dims after `dim`).  Replaces ops::softmax (src/ops/activation.rs:76-124)
 * and KernelManager::launch_softmax (src/cuda_backend/kernels.rs:358-376,
 * inner = 1).  out must not alias x when inner > 1. */
int oxide_softmax_f32(const float* x, float* out, uint64_t outer, uint64_t dim, uint64_t inner,
                      oxide_stream_t stream);
int oxide_softmax_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t outer, uint64_t dim,
                       uint64_t inner, oxide_stream_t stream);

/* Scale + mask + softmax over rows of x[rows, cols] (raw attention scores):
 *     s_j = x_j * scale;  s_j += mask[j % mask_len]  (if mask != NULL);
 *     s_j = -inf for j >= L_r;   out = softmax(s)
 * the scale/mask/softmax block of scaled_dot_product_attention
 * (src/ops/attention.rs:41,60,63-79).  L_r (API addition) is cols, lowered
 * to lens[r / rows_per_len] when lens != NULL (per-sequence KV length) and to
 * (r % causal_q_len) + 1 + cols - causal_q_len when causal_q_len > 0 (causal
 * mask, query r % causal_q_len of a q_len-row block).  Keys j >= L_r are
 * written as 0 without being read; a row with L_r = 0 is all zeros. */
int oxide_scale_mask_softmax_f32(const float* x, float* out, uint64_t rows, uint64_t cols,
                                 float scale, const float* mask, uint64_t mask_len,
                                 const int32_t* lens, uint64_t rows_per_len,
                                 uint64_t causal_q_len, oxide_stream_t stream);
int oxide_scale_mask_softmax_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t rows,
                                  uint64_t cols, float scale, const float* mask,
                                  uint64_t mask_len, const int32_t* lens,
                                  uint64_t rows_per_len, uint64_t causal_q_len,
                                  oxide_stream_t stream);

/* ---- rotary embedding --------------------------------------------------------
 * Rotate-half RoPE of q and (optionally) k in one launch, replacing the two
 * apply_rotary_emb calls of MultiHeadAttention::forward
 * (src/layers/attention.rs:88-94; op body src/ops/attention.rs:139-155):
 *     o[d] = x1*c - x2*s,  o[d+half] = x1*s + x2*c,  d < half = head_dim/2
 * with c = cos[p, d], s = sin[p, d] from f32 tables [table_rows, half] and
 * p = positions[t] (positions may be NULL: p = t).
 * layout 0 = token-major [tokens, heads, head_dim] (src/kernels/attention.rs:91-118),
 * layout 1 = head-major [heads, tokens, head_dim] (src/ops/attention.rs:139-144).
 * k may be NULL (k_heads ignored).  Outputs may alias their inputs. */
int oxide_rope_f32(const float* q, float* q_out, uint64_t q_heads, const float* k, float* k_out,
                   uint64_t k_heads, const float* cos_t, const float* sin_t, uint64_t table_rows,
                   const int32_t* positions, uint64_t tokens, uint64_t head_dim, int layout,
                   oxide_stream_t stream);
int oxide_rope_bf16(const oxide_bf16* q, oxide_bf16* q_out, uint64_t q_heads,
                    const oxide_bf16* k, oxide_bf16* k_out, uint64_t k_heads,
                    const float* cos_t, const float* sin_t, uint64_t table_rows,
                    const int32_t* positions, uint64_t tokens, uint64_t head_dim, int layout,
                    oxide_stream_t stream);

/* Host-side table build with the formula of precompute_rope_cache
 * (src/models/mistral.rs:91-115): freq_i = theta^(-2i/head_dim) (powf),
 * angle = pos * freq_i, cos/sin into host arrays [max_pos, head_dim/2].
 * Model set-up, not a per-layer op; host pointers. */
int oxide_rope_table_host_f32(float theta, uint64_t head_dim, uint64_t max_pos,
                              float* cos_host, float* sin_host);

/* ---- weight decoding (safetensors element bytes) ---------------------------------
 * SafetensorsLoader::load_tensor_from_view (src/loading/safetensors.rs:48-82)
 * on the device: n little-endian elements of src_dtype (device memory, aligned
 * to the element size) -> out.  F32 is copied; F16 is converted exactly as the
 * half crate does (NaN: quiet bit set, payload kept); BF16 is decoded as the
 * high half of an f32 -- the reference decodes BF16 bytes as f16, a bug this
 * entry point fixes.  The bf16 form rounds the decoded value to nearest-even
 * bf16 (exact for BF16 sources; a NaN becomes the canonical bf16 NaN). */
enum oxide_wdtype { OXIDE_WDT_F32 = 0, OXIDE_WDT_F16 = 1, OXIDE_WDT_BF16 = 2 };
int oxide_decode_weights_f32(const void* src, uint64_t n, int src_dtype, float* out, oxide_stream_t stream);
int oxide_decode_weights_bf16(const void* src, uint64_t n, int src_dtype, oxide_bf16* out, oxide_stream_t stream);

/* ---- KV cache and grouped-query heads -------------------------------------------
 * repeat_kv (src/ops/attention.rs:161-201): x [batch, kv_heads, seq_len,
 * head_dim] -> out [batch, kv_heads * n_rep, seq_len, head_dim],
 * out[b, h * n_rep + r] = x[b, h] (bit-exact copy; out must not alias x). */
int oxide_repeat_kv_f32(const float* x, float* out, uint64_t batch, uint64_t kv_heads, uint64_t seq_len,
                        uint64_t head_dim, uint64_t n_rep, oxide_stream_t stream);
int oxide_repeat_kv_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t batch, uint64_t kv_heads,
                         uint64_t seq_len, uint64_t head_dim, uint64_t n_rep, oxide_stream_t stream);

/* KVCache::update (src/cache/kv_cache.rs:55-85; kernel intent kv_cache_update_f32,
 * src/kernels/attention.rs:121-158): k, v [batch, kv_heads, new_len, head_dim]
 * are copied to positions [cur_len, cur_len + new_len) of the caches
 * [batch, kv_heads, max_seq, head_dim], both in one launch.  cur_len + new_len
 * > max_seq is OXIDE_ERR_INVALID_ARG ("KV cache overflow"), nothing written. */
int oxide_kv_cache_append_f32(float* k_cache, float* v_cache, const float* k, const float* v, uint64_t batch,
                              uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, uint64_t cur_len,
                              uint64_t new_len, oxide_stream_t stream);
int oxide_kv_cache_append_bf16(oxide_bf16* k_cache, oxide_bf16* v_cache, const oxide_bf16* k,
                               const oxide_bf16* v, uint64_t batch, uint64_t kv_heads, uint64_t max_seq,
                               uint64_t head_dim, uint64_t cur_len, uint64_t new_len, oxide_stream_t stream);

/* ---- decode attention ---------------------------------------------------------
 * One query token per (batch, head) against KV caches [batch, kv_heads,
 * max_seq, head_dim]: the inline attention of scaled_dot_product_attention
 * (src/ops/attention.rs:41-87) with q_len = 1 -- s_j = (q . k_j) * scale,
 * softmax over j < lens[b] (lens NULL: every position), out = sum_j p_j v_j --
 * where query head h reads kv head h / (q_heads / kv_heads) (repeat_kv's head
 * map, attention.rs:161-201, without materialising it).  q, out [batch,
 * q_heads, head_dim].  A sequence of length 0 gives zeros.  Pass the
 * reference's scale, (head_dim as f32).sqrt().recip().  `workspace` is device
 * memory of at least oxide_decode_attention_workspace_bytes(...) bytes,
 * 16-byte aligned, for the split-K partials.  API addition (flash-decoding);
 * the reference computes it through repeat_kv + matmul + softmax + matmul. */
uint64_t oxide_decode_attention_workspace_bytes(uint64_t batch, uint64_t q_heads, uint64_t max_seq,
                                                uint64_t head_dim);
/* Kernel choice of oxide_decode_attention_bf16 (diagnostic; no reference
 * counterpart): 0 (default) = the tcgen05 / TMA kernel wherever it applies
 * (sm_100, head_dim 128, q_heads / kv_heads in {1, 2, 4, 8}, batch <= 1024,
 * max_seq >= 256), else the split-K mma.sync kernel; 1 = always the split-K
 * kernel; 2 = the tcgen05 kernel with its tile loads withheld, so that every
 * bounded wait in it runs out (about two seconds) and the launch ends with
 * NaN outputs and OXIDE_DEVICE_WAIT_TIMEOUT raised -- for failure-detection
 * tests only.  Process-wide; set it between calls, not while one is
 * enqueued. */
void oxide_debug_decode_attention_path(int path);

/* Device-side failure flags (no reference counterpart: the reference has no
 * device waits).  A kernel whose bounded wait runs out -- a copy or product
 * that never completes -- stops, writes NaN outputs and raises a flag in a
 * per-device word instead of hanging; the flags are sticky, like CUDA's own
 * errors, until reset.  oxide_device_status waits for the calling thread's
 * current device to finish its work, stores the flags raised since the last
 * reset in *flags and clears them if reset != 0. */
#define OXIDE_DEVICE_WAIT_TIMEOUT 1u
int oxide_device_status(int reset, uint32_t* flags);
int oxide_decode_attention_f32(const float* q, const float* k_cache, const float* v_cache, const int32_t* lens,
                               float* out, uint64_t batch, uint64_t q_heads, uint64_t kv_heads, uint64_t max_seq,
                               uint64_t head_dim, float scale, void* workspace, uint64_t workspace_bytes,
                               oxide_stream_t stream);
int oxide_decode_attention_bf16(const oxide_bf16* q, const oxide_bf16* k_cache, const oxide_bf16* v_cache,
                                const int32_t* lens, oxide_bf16* out, uint64_t batch, uint64_t q_heads,
                                uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, float scale,
                                void* workspace, uint64_t workspace_bytes, oxide_stream_t stream);

/* ---- token sampling ----------------------------------------------------------
 * sample_next_token (src/pipeline.rs:181-205) for each row of logits
 * [rows, vocab] (vocab <= 262144): probs = softmax_with_temperature(row,
 * temperature) (src/tokenizer.rs:166-180: x / T, max, sum of exp(s - max),
 * exp(s - max) / sum); then, if top_p < 1, sample_top_p (:182-211: the
 * shortest prefix of the probabilities sorted in descending order whose
 * running sum reaches top_p), else sample_top_k (:213-232: the first
 * min(top_k, vocab)); r = uniforms[r] * (the prefix's sum), and tokens[row] =
 * the first index of the prefix whose running sum reaches r.  Equal
 * probabilities keep ascending index order (the reference's stable sort).
 * uniforms[rows] (device, f32 in [0, 1)) are the draws the reference takes
 * from fastrand::f32(), so the caller keeps the reference's generator.
 * tokens[row] = OXIDE_SAMPLE_INVALID when the row's probabilities hold a NaN
 * (a NaN logit, a scaled logit of +-inf, an all -inf row; the reference's
 * sort panics there); vocab == 1 gives 0; top_k == 0 gives 0 (the reference's
 * empty prefix).  probs (device f32 [rows, vocab]) may be NULL; tokens may be
 * NULL when probs is not (softmax_with_temperature alone).  Running sums are
 * f64 sums of per-thread f32 sums, so an index can differ from the
 * reference's sequential f32 walk only when r falls within that walk's
 * rounding drift of a boundary between two running sums. */
#define OXIDE_SAMPLE_INVALID 0xFFFFFFFFu
int oxide_sample_f32(const float* logits, uint64_t rows, uint64_t vocab, float temperature, uint64_t top_k,
                     float top_p, const float* uniforms, uint32_t* tokens, float* probs, oxide_stream_t stream);
int oxide_sample_bf16(const oxide_bf16* logits, uint64_t rows, uint64_t vocab, float temperature, uint64_t top_k,
                      float top_p, const float* uniforms, uint32_t* tokens, float* probs, oxide_stream_t stream);
/* softmax_with_temperature (src/tokenizer.rs:166-180) alone: probs [rows, vocab] f32. */
int oxide_softmax_with_temperature_f32(const float* logits, float* probs, uint64_t rows, uint64_t vocab,
                                       float temperature, oxide_stream_t stream);
int oxide_softmax_with_temperature_bf16(const oxide_bf16* logits, float* probs, uint64_t rows, uint64_t vocab,
                                        float temperature, oxide_stream_t stream);

/* ---- argmax ----------------------------------------------------------------
 * Index of the largest element of each row of x[rows, cols] (cols < 2^32):
 * the lowest index among equal maxima (+0 == -0), NaN ranks below every
 * number.  API addition: the reference's only argmax-like path is
 * sample_top_k with k = 1 after a stable descending sort
 * (src/tokenizer.rs:213-232, called from src/pipeline.rs:181-205). */
int oxide_argmax_rows_f32(const float* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                          oxide_stream_t stream);
int oxide_argmax_rows_bf16(const oxide_bf16* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                           oxide_stream_t stream);

/* ---- reductions --------------------------------------------------------------
 * Per-row sum / max / sum of squares of x[rows, cols] into f32 out[rows].
 * API addition; the reference has them only inline (sum of squares
 * src/ops/norm.rs:36-40, max src/ops/activation.rs:99-103). */
int oxide_reduce_rows_f32(int op, const float* x, uint64_t rows, uint64_t cols, float* out,
                          oxide_stream_t stream);
int oxide_reduce_rows_bf16(int op, const oxide_bf16* x, uint64_t rows, uint64_t cols,
                           float* out, oxide_stream_t stream);

/* Whole-tensor sum / max / sum of squares of x[n] into one f64 at *out
 * (device pointer), deterministic for a given n: a fixed partition into at
 * most 1024 blocks, f32 lane sums inside a block, f64 above.  `workspace`
 * is caller-owned device memory of at least oxide_reduce_workspace_bytes(n)
 * bytes; it needs no initialisation.  Across GPUs, the per-GPU results are
 * combined with one NCCL allreduce (sum, or max) of a single f64. */
uint64_t oxide_reduce_workspace_bytes(uint64_t n);
int oxide_reduce_f32(int op, const float* x, uint64_t n, double* out, void* workspace,
                     uint64_t workspace_bytes, oxide_stream_t stream);
int oxide_reduce_bf16(int op, const oxide_bf16* x, uint64_t n, double* out, void* workspace,
                      uint64_t workspace_bytes, oxide_stream_t stream);

/* Whole-tensor reduction that allocates nothing and takes no workspace.
 * No counterpart in the reference: an addition for callers that cannot hand
 * over scratch memory, such as a launcher that receives only its input and
 * output buffers (the shape of KernelManager::launch_*), or a decode loop that
 * must not call cudaMalloc/cudaFree mid-step because they synchronise the
 * device.  Same result, bit for bit, as oxide_reduce_* for the same x and n.
 *
 * Scratch: a fixed array of OXIDE_REDUCE_STATIC_SLOTS f64 partials (8 KiB) in
 * the library's own device memory, one per device.  Every slot a call reads is
 * written earlier in the same call, so no slot has to start at zero and the
 * contents left by an earlier call do not matter.
 * Limit: n <= OXIDE_REDUCE_STATIC_MAX_N elements (2^24 per slot); larger n
 * returns OXIDE_ERR_INVALID_ARG without launching anything.
 * First call on a device: looks up the array's device address with the
 * calling thread's current device (cudaGetSymbolAddress), which may load the
 * library's device code; make that first call outside any stream capture.
 * The address is kept per CUDA context, so the first call after a
 * cudaDeviceReset (a new context) repeats the lookup and the same rule
 * applies to it.
 * Concurrency: all calls on one device share the one array, so two calls
 * that can overlap on the GPU (different streams without an ordering event
 * between them) race and return wrong results.  Order them on one stream, or
 * use oxide_reduce_* with separate workspaces. */
#define OXIDE_REDUCE_STATIC_SLOTS 1024
#define OXIDE_REDUCE_STATIC_MAX_N (((uint64_t)OXIDE_REDUCE_STATIC_SLOTS) << 24)
int oxide_reduce_static_f32(int op, const float* x, uint64_t n, double* out,
                            oxide_stream_t stream);
int oxide_reduce_static_bf16(int op, const oxide_bf16* x, uint64_t n, double* out,
                             oxide_stream_t stream);

/* ---- host-buffer pipeline ----------------------------------------------------
 * The reference's ops take host tensors and return host tensors
 * (src/ops: Tensor::zeros + as_f32_slice) and its GPU path copies through
 * CudaBackend::copy_host_to_device / copy_device_to_host
 * (src/cuda_backend/mod.rs:76-85).  A pipeline runs one op on host buffers:
 * it splits the rows into chunks and, on `depth` streams, overlaps the
 * host->device copy of chunk i+1, the kernel of chunk i and the device->host
 * copy of chunk i-1.  Host buffers should be page-locked (cudaHostRegister
 * or cudaMallocHost) for the copies to overlap.  The pipeline owns its
 * device staging buffers (allocated once by oxide_pipe_create); the op calls
 * allocate nothing and return after the output is in host memory. */
typedef struct oxide_pipe* oxide_pipe_t;
int oxide_pipe_create(int device, uint64_t chunk_bytes, int depth, oxide_pipe_t* out);
int oxide_pipe_destroy(oxide_pipe_t pipe);
int oxide_pipe_binary_f32(oxide_pipe_t pipe, int op, const float* a_host, uint64_t na,
                          const float* b_host, uint64_t nb, float* out_host, uint64_t n);
int oxide_pipe_silu_mul_f32(oxide_pipe_t pipe, const float* gate_host, const float* up_host,
                            float* out_host, uint64_t n);
int oxide_pipe_rms_norm_f32(oxide_pipe_t pipe, const float* x_host, const float* w_host,
                            float* out_host, uint64_t rows, uint64_t cols, float eps);

/* Deferred mode (on != 0): the op calls below return once their copies and
 * kernels are enqueued, so one op's uploads overlap the previous op's
 * downloads; oxide_pipe_sync waits for everything enqueued.  Host buffers must
 * stay valid, and outputs unread, until then.  Turning deferred mode off waits
 * as oxide_pipe_sync does.  A failing call still waits before returning. */
int oxide_pipe_defer(oxide_pipe_t pipe, int on);
int oxide_pipe_sync(oxide_pipe_t pipe);

/* h = a + b and y = h * s[col] (ops::add then the row-broadcast ops::mul,
 * src/ops/matmul.rs:74-108) from one upload of a, b and s: h is downloaded as
 * the next residual and not uploaded again for the multiply.  Results equal
 * oxide_add_f32 then oxide_mul_rowbcast_f32. */
int oxide_pipe_add_mul_rowbcast_f32(oxide_pipe_t pipe, const float* a_host, const float* b_host,
                                    const float* s_host, float* h_host, float* y_host, uint64_t rows,
                                    uint64_t cols);
/* oxide_add_rms_norm_* on host rows (src/layers/transformer.rs:64-67). */
int oxide_pipe_add_rms_norm_f32(oxide_pipe_t pipe, const float* x_host, const float* r_host,
                                const float* w_host, float* h_host, float* y_host, uint64_t rows,
                                uint64_t cols, float eps);
int oxide_pipe_add_rms_norm_bf16(oxide_pipe_t pipe, const oxide_bf16* x_host, const oxide_bf16* r_host,
                                 const oxide_bf16* w_host, oxide_bf16* h_host, oxide_bf16* y_host,
                                 uint64_t rows, uint64_t cols, float eps);
/* oxide_scale_mask_softmax_f32 on host rows (src/ops/attention.rs:41,60,63-79;
 * ops::softmax src/ops/activation.rs:76).  mask (mask_len f32) and lens
 * (int32, one per rows_per_len rows) are host arrays.  With lens, only the
 * first lens[g] keys of each row of group g are uploaded -- the kernel never
 * reads the others -- and the whole output row is downloaded.  A chunk holds
 * whole lens groups and whole causal blocks. */
int oxide_pipe_scale_mask_softmax_f32(oxide_pipe_t pipe, const float* x_host, float* out_host, uint64_t rows,
                                      uint64_t cols, float scale, const float* mask_host, uint64_t mask_len,
                                      const int32_t* lens_host, uint64_t rows_per_len, uint64_t causal_q_len);
/* oxide_argmax_rows_f32 on host rows; idx_host [rows]. */
int oxide_pipe_argmax_rows_f32(oxide_pipe_t pipe, const float* x_host, uint64_t rows, uint64_t cols,
                               uint32_t* idx_host);
/* oxide_rope_bf16, token-major layout, on host tensors: the two
 * apply_rotary_emb calls of MultiHeadAttention::forward
 * (src/layers/attention.rs:88-94; src/ops/attention.rs:96-159).  cos/sin
 * [table_rows, head_dim/2] f32 and positions [tokens] (may be NULL) are host
 * arrays; k may be NULL.  Outputs may alias inputs. */
int oxide_pipe_rope_bf16(oxide_pipe_t pipe, const oxide_bf16* q_host, oxide_bf16* q_out_host, uint64_t q_heads,
                         const oxide_bf16* k_host, oxide_bf16* k_out_host, uint64_t k_heads,
                         const float* cos_host, const float* sin_host, uint64_t table_rows,
                         const int32_t* positions_host, uint64_t tokens, uint64_t head_dim);

#ifdef __cplusplus
}
#endif
#endif /* OXIDE_OPS_H */
