/*
 * oxide_oracle.h -- CPU restatement of mistralrs-oxide's src/ops arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * kernels and the timed CPU baseline.  Only tests/, __graft_entry__.smoke()
 * and bench.py (its cpu_baseline leg and its `--impl reference` arm) may load
 * it.  No product code path links, imports or falls back to it.
 *
 * PARITY UNPINNED by the reference's own outputs: the reference is a Rust
 * crate that does not compile (and no Rust toolchain exists here), and it
 * ships no golden vectors or known-answer tests.  The restatement is pinned
 * instead by hand-derived known-answer tests (tests/test_oracle_kat.py) and
 * by an independent numpy restatement of the same loop bodies
 * (tests/test_oracle_numpy.py).
 *
 * Every function follows the sequential f32 order of the reference loop it
 * cites.  The threaded variants split the OUTER loop (elements or rows) over
 * OpenMP threads; the arithmetic of every output element is unchanged, so
 * results are bit-identical for any thread count.
 *
 * bf16 semantics (the reference has no bf16 arithmetic): a bf16 operand is
 * widened to f32, the reference formula runs in f32, and every tensor that the
 * reference would materialise is rounded to bf16 (round-to-nearest-even) once
 * at its store.
 */
#ifndef OXIDE_ORACLE_H
#define OXIDE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_ADD = 0, ORC_SUB = 1, ORC_MUL = 2, ORC_DIV = 3 };
enum { ORC_RED_SUM = 0, ORC_RED_MAX = 1, ORC_RED_SUMSQ = 2 };

float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);

/* src/ops/matmul.rs:136-158: out[i] = op(a[i % na], b[i % nb]) */
void orc_binary_f32(int op, const float* a, uint64_t na, const float* b, uint64_t nb,
                    float* out, uint64_t n, int threads);
void orc_binary_bf16(int op, const uint16_t* a, uint64_t na, const uint16_t* b, uint64_t nb,
                     uint16_t* out, uint64_t n, int threads);

/* build.rs:240-276 scale_f32 / src/cuda_backend/kernels.rs:159-177: out = x * s */
void orc_scale_f32(const float* x, float* out, float s, uint64_t n, int threads);
void orc_scale_bf16(const uint16_t* x, uint16_t* out, float s, uint64_t n, int threads);

/* src/ops/activation.rs:21-37: y = x * (1 / (1 + exp(-x))) */
void orc_silu_f32(const float* x, float* out, uint64_t n, int threads);
void orc_silu_bf16(const uint16_t* x, uint16_t* out, uint64_t n, int threads);

/* src/layers/attention.rs:144-145: mul(silu(gate), up) */
void orc_silu_mul_f32(const float* g, const float* u, float* out, uint64_t n, int threads);
void orc_silu_mul_bf16(const uint16_t* g, const uint16_t* u, uint16_t* out, uint64_t n,
                       int threads);

/* src/ops/norm.rs:33-47 */
void orc_rms_norm_f32(const float* x, const float* w, float* out, uint64_t rows,
                      uint64_t cols, float eps, int threads);
void orc_rms_norm_bf16(const uint16_t* x, const uint16_t* w, uint16_t* out, uint64_t rows,
                       uint64_t cols, float eps, int threads);

/* src/layers/transformer.rs:64-67 (add, then rms_norm of the sum) */
void orc_add_rms_norm_f32(const float* x, const float* r, const float* w, float* h,
                          float* y, uint64_t rows, uint64_t cols, float eps, int threads);
void orc_add_rms_norm_bf16(const uint16_t* x, const uint16_t* r, const uint16_t* w,
                           uint16_t* h, uint16_t* y, uint64_t rows, uint64_t cols, float eps,
                           int threads);

/* src/ops/activation.rs:76-124 softmax(x, dim) over [outer, dim, inner] */
void orc_softmax_f32(const float* x, float* out, uint64_t outer, uint64_t dim,
                     uint64_t inner, int threads);
void orc_softmax_bf16(const uint16_t* x, uint16_t* out, uint64_t outer, uint64_t dim,
                      uint64_t inner, int threads);

/* src/ops/attention.rs:41,60,63-79: s = x*scale; s += mask[j % mask_len];
 * softmax over the row.  lens (per group of rows_per_len rows) and
 * causal_q_len (row r is query r % q, keys j > r % q + cols - q masked) are
 * API additions that set s = -inf beyond the valid length; a row whose valid
 * length is 0 is written as zeros. */
void orc_scale_mask_softmax_f32(const float* x, float* out, uint64_t rows, uint64_t cols,
                                float scale, const float* mask, uint64_t mask_len,
                                const int32_t* lens, uint64_t rows_per_len,
                                uint64_t causal_q_len, int threads);
void orc_scale_mask_softmax_bf16(const uint16_t* x, uint16_t* out, uint64_t rows,
                                 uint64_t cols, float scale, const float* mask,
                                 uint64_t mask_len, const int32_t* lens,
                                 uint64_t rows_per_len, uint64_t causal_q_len, int threads);

/* src/models/mistral.rs:91-115 precompute_rope_cache: tables [max_pos, head_dim/2] */
void orc_rope_table_f32(float theta, uint64_t head_dim, uint64_t max_pos, float* cos_out,
                        float* sin_out);

/* src/ops/attention.rs:139-155 rotate-half RoPE.
 * layout 0: token-major [tokens, heads, head_dim] (src/kernels/attention.rs:91-118)
 * layout 1: head-major  [heads, tokens, head_dim] (src/ops/attention.rs:139-144)
 * positions (nullable) selects the table row of each token; NULL means row t. */
void orc_rope_f32(const float* x, float* out, uint64_t tokens, uint64_t heads,
                  uint64_t head_dim, int layout, const float* cos_t, const float* sin_t,
                  const int32_t* positions, int threads);
void orc_rope_bf16(const uint16_t* x, uint16_t* out, uint64_t tokens, uint64_t heads,
                   uint64_t head_dim, int layout, const float* cos_t, const float* sin_t,
                   const int32_t* positions, int threads);

/* argmax semantics of src/tokenizer.rs:213-232 with k = 1 (stable descending
 * sort: the lowest index among equal maxima); NaN ranks below every number. */
void orc_argmax_rows_f32(const float* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                         int threads);
void orc_argmax_rows_bf16(const uint16_t* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                          int threads);

/* Row reductions in the reference's inline sequential f32 order
 * (sum of squares: src/ops/norm.rs:36-40; max: src/ops/activation.rs:99-103). */
void orc_reduce_rows_f32(int op, const float* x, uint64_t rows, uint64_t cols, float* out,
                         int threads);
void orc_reduce_rows_bf16(int op, const uint16_t* x, uint64_t rows, uint64_t cols,
                          float* out, int threads);

/* Whole-tensor reductions accumulated in f64 (fixed 1 Mi-element chunks,
 * chunk partials summed in order; deterministic for any thread count). */
double orc_reduce_f32(int op, const float* x, uint64_t n, int threads);
double orc_reduce_bf16(int op, const uint16_t* x, uint64_t n, int threads);

/* The same whole-tensor reduction in the reference's naive sequential f32
 * order; reported for information only (it stalls for n ~ 1e8). */
float orc_reduce_seq_f32(int op, const float* x, uint64_t n);

/* Unary ops (op codes equal the C ABI's oxide_unop): relu, gelu (tanh form),
 * gelu_quick, sigmoid, tanh (src/ops/activation.rs) and exp, ln, sqrt, powf(a),
 * clamp(a, b), neg, abs (src/ops/math.rs). */
enum {
    ORC_RELU = 0, ORC_GELU = 1, ORC_GELU_QUICK = 2, ORC_SIGMOID = 3, ORC_TANH = 4, ORC_EXP = 5,
    ORC_LOG = 6, ORC_SQRT = 7, ORC_POW = 8, ORC_CLAMP = 9, ORC_NEG = 10, ORC_ABS = 11
};
void orc_unary_f32(int op, const float* x, float* out, uint64_t n, float a, float b, int threads);
void orc_unary_bf16(int op, const uint16_t* x, uint16_t* out, uint64_t n, float a, float b,
                    int threads);

/* src/ops/norm.rs:53-117: mean, variance of x - mean, (x - mean) / sqrt(var + eps) * w + b */
void orc_layer_norm_f32(const float* x, const float* w, const float* b, float* out, uint64_t rows,
                        uint64_t cols, float eps, int threads);
void orc_layer_norm_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* out,
                         uint64_t rows, uint64_t cols, float eps, int threads);

/* src/ops/attention.rs:161-201 repeat_kv and src/cache/kv_cache.rs:55-85 append
 * (byte copies; es = element size in bytes; append returns -1 on overflow). */
void orc_repeat_kv(const void* x, void* out, uint64_t batch, uint64_t heads, uint64_t seq,
                   uint64_t head_dim, uint64_t n_rep, uint64_t es);
int orc_kv_append(void* kc, void* vc, const void* k, const void* v, uint64_t batch, uint64_t heads,
                  uint64_t max_seq, uint64_t head_dim, uint64_t cur, uint64_t new_len, uint64_t es);

/* One-token (decode) attention, src/ops/attention.rs:41-87 with per-batch KV
 * lengths and grouped-query heads (kv head = q head / (q_heads / kv_heads)). */
void orc_decode_attention_f32(const float* q, const float* kc, const float* vc, const int32_t* lens,
                              float* out, uint64_t batch, uint64_t q_heads, uint64_t kv_heads,
                              uint64_t max_seq, uint64_t head_dim, float scale, int threads);
void orc_decode_attention_bf16(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                               const int32_t* lens, uint16_t* out, uint64_t batch, uint64_t q_heads,
                               uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, float scale,
                               int threads);

/* Token sampling, src/pipeline.rs:181-205 (sample_next_token) on one row of
 * logits: probs = softmax_with_temperature(row, T) (src/tokenizer.rs:166-180:
 * s = x / T, m = fold(-inf, f32::max), sum = sequential sum of exp(s - m),
 * p = exp(s - m) / sum), then top_p < 1 ? sample_top_p (:182-211) :
 * sample_top_k (:213-232): a stable descending sort by probability, the kept
 * prefix, total = its sequential f32 sum, r = u * total, and the first index
 * whose sequential cumulative sum reaches r.  u is the uniform draw the
 * reference takes from fastrand::f32().  A row whose probabilities hold a NaN
 * (vocab >= 2) yields ORC_SAMPLE_INVALID: the reference's sort panics there. */
#define ORC_SAMPLE_INVALID 0xFFFFFFFFu
void orc_softmax_temperature_f32(const float* x, uint64_t rows, uint64_t vocab, float temperature,
                                 float* probs, int threads);
void orc_softmax_temperature_bf16(const uint16_t* x, uint64_t rows, uint64_t vocab, float temperature,
                                  float* probs, int threads);
uint32_t orc_sample_probs(const float* probs, uint64_t vocab, uint64_t top_k, float top_p, float u);
void orc_sample_f32(const float* logits, uint64_t rows, uint64_t vocab, float temperature, uint64_t top_k,
                    float top_p, const float* uniforms, uint32_t* tokens, float* probs, int threads);
void orc_sample_bf16(const uint16_t* logits, uint64_t rows, uint64_t vocab, float temperature,
                     uint64_t top_k, float top_p, const float* uniforms, uint32_t* tokens, float* probs,
                     int threads);

/* src/loading/safetensors.rs:48-82 element decode: F32 copy, F16 through the
 * half crate's exact f16 -> f32 conversion, BF16 as the high half of an f32
 * (the reference runs BF16 bytes through the f16 conversion, a bug not
 * restated here; orc_decode_f16_bits_f32 gives what it computes). */
enum { ORC_WDT_F32 = 0, ORC_WDT_F16 = 1, ORC_WDT_BF16 = 2 };
void orc_decode_weights_f32(const void* src, uint64_t n, int dtype, float* out);
void orc_decode_weights_bf16(const void* src, uint64_t n, int dtype, uint16_t* out);
float orc_decode_f16_bits_f32(uint16_t h);

int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
