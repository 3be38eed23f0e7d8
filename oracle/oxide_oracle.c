/*
 * oxide_oracle.c -- CPU restatement of mistralrs-oxide's src/ops loop bodies.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); see
 * oxide_oracle.h for the contract, the bf16 convention and why parity is
 * unpinned by reference outputs.
 *
 * Build with -ffp-contract=off and without fast-math: Rust never contracts
 * a*b+c into an FMA and never reassociates, and neither may this file.
 * f32 transcendental calls go to glibc (expf, powf, cosf, sinf), which is what
 * Rust's f32::exp / powf / cos / sin lower to on Linux.
 */
#include "oxide_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OMP_FOR _Pragma("omp parallel for schedule(static) num_threads(threads)")

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
    return (uint16_t)(u >> 16);
}

#define B2F orc_bf16_to_f32
#define F2B orc_f32_to_bf16

static inline float apply_op(int op, float x, float y) {
    switch (op) {
        case ORC_ADD: return x + y;
        case ORC_SUB: return x - y;
        case ORC_MUL: return x * y;
        default: return x / y;
    }
}

/* ---- binary ops: src/ops/matmul.rs:136-158 (elementwise_op_cpu) --------- */
void orc_binary_f32(int op, const float* a, uint64_t na, const float* b, uint64_t nb,
                    float* out, uint64_t n, int threads) {
    if (na == n && nb == n) {
        OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = apply_op(op, a[i], b[i]);
        return;
    }
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = apply_op(op, a[i % na], b[i % nb]);
}

void orc_binary_bf16(int op, const uint16_t* a, uint64_t na, const uint16_t* b, uint64_t nb,
                     uint16_t* out, uint64_t n, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i)
        out[i] = F2B(apply_op(op, B2F(a[i % na]), B2F(b[i % nb])));
}

/* ---- scale: build.rs:240-276 / src/cuda_backend/kernels.rs:159-177 ------- */
void orc_scale_f32(const float* x, float* out, float s, uint64_t n, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = x[i] * s;
}

void orc_scale_bf16(const uint16_t* x, uint16_t* out, float s, uint64_t n, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = F2B(B2F(x[i]) * s);
}

/* ---- SiLU: src/ops/activation.rs:30-33 ---------------------------------- */
static inline float silu1(float x) {
    float e = expf(-x);
    float d = 1.0f + e;
    float r = 1.0f / d;
    return x * r;
}

void orc_silu_f32(const float* x, float* out, uint64_t n, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = silu1(x[i]);
}

void orc_silu_bf16(const uint16_t* x, uint16_t* out, uint64_t n, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = F2B(silu1(B2F(x[i])));
}

/* ---- SiLU * up: src/layers/attention.rs:144-145 (silu, then ops::mul) ---- */
void orc_silu_mul_f32(const float* g, const float* u, float* out, uint64_t n, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = silu1(g[i]) * u[i];
}

void orc_silu_mul_bf16(const uint16_t* g, const uint16_t* u, uint16_t* out, uint64_t n,
                       int threads) {
    /* The composed reference materialises silu(gate) as a bf16 tensor. */
    OMP_FOR for (uint64_t i = 0; i < n; ++i) {
        float gated = B2F(F2B(silu1(B2F(g[i]))));
        out[i] = F2B(gated * B2F(u[i]));
    }
}

/* ---- RMSNorm: src/ops/norm.rs:33-47 --------------------------------------- */
static inline float rms_of_row_f32(const float* x, uint64_t cols, float eps) {
    float ss = 0.0f;
    for (uint64_t i = 0; i < cols; ++i) {
        float v = x[i];
        ss += v * v;
    }
    return sqrtf(ss / (float)cols + eps);
}

void orc_rms_norm_f32(const float* x, const float* w, float* out, uint64_t rows,
                      uint64_t cols, float eps, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        float* orow = out + r * cols;
        float rms = rms_of_row_f32(xr, cols, eps);
        for (uint64_t i = 0; i < cols; ++i) {
            float normalized = xr[i] / rms;
            orow[i] = normalized * w[i];
        }
    }
}

void orc_rms_norm_bf16(const uint16_t* x, const uint16_t* w, uint16_t* out, uint64_t rows,
                       uint64_t cols, float eps, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * cols;
        uint16_t* orow = out + r * cols;
        float ss = 0.0f;
        for (uint64_t i = 0; i < cols; ++i) {
            float v = B2F(xr[i]);
            ss += v * v;
        }
        float rms = sqrtf(ss / (float)cols + eps);
        for (uint64_t i = 0; i < cols; ++i) {
            float normalized = B2F(xr[i]) / rms;
            orow[i] = F2B(normalized * B2F(w[i]));
        }
    }
}

/* ---- add + RMSNorm: src/layers/transformer.rs:64 then :67 ---------------- */
void orc_add_rms_norm_f32(const float* x, const float* r, const float* w, float* h,
                          float* y, uint64_t rows, uint64_t cols, float eps, int threads) {
    OMP_FOR for (uint64_t row = 0; row < rows; ++row) {
        const float* xr = x + row * cols;
        const float* rr = r + row * cols;
        float* hr = h + row * cols;
        float* yr = y + row * cols;
        for (uint64_t i = 0; i < cols; ++i) hr[i] = xr[i] + rr[i];
        float rms = rms_of_row_f32(hr, cols, eps);
        for (uint64_t i = 0; i < cols; ++i) {
            float normalized = hr[i] / rms;
            yr[i] = normalized * w[i];
        }
    }
}

void orc_add_rms_norm_bf16(const uint16_t* x, const uint16_t* r, const uint16_t* w,
                           uint16_t* h, uint16_t* y, uint64_t rows, uint64_t cols, float eps,
                           int threads) {
    OMP_FOR for (uint64_t row = 0; row < rows; ++row) {
        const uint16_t* xr = x + row * cols;
        const uint16_t* rr = r + row * cols;
        uint16_t* hr = h + row * cols;
        uint16_t* yr = y + row * cols;
        float ss = 0.0f;
        for (uint64_t i = 0; i < cols; ++i) {
            hr[i] = F2B(B2F(xr[i]) + B2F(rr[i]));
            float v = B2F(hr[i]);
            ss += v * v;
        }
        float rms = sqrtf(ss / (float)cols + eps);
        for (uint64_t i = 0; i < cols; ++i) {
            float normalized = B2F(hr[i]) / rms;
            yr[i] = F2B(normalized * B2F(w[i]));
        }
    }
}

/* ---- softmax(x, dim): src/ops/activation.rs:95-120 ------------------------ */
void orc_softmax_f32(const float* x, float* out, uint64_t outer, uint64_t dim,
                     uint64_t inner, int threads) {
    OMP_FOR for (uint64_t oi = 0; oi < outer * inner; ++oi) {
        uint64_t base = (oi / inner) * dim * inner + (oi % inner);
        float max_val = -INFINITY;
        for (uint64_t d = 0; d < dim; ++d) max_val = fmaxf(max_val, x[base + d * inner]);
        float sum = 0.0f;
        for (uint64_t d = 0; d < dim; ++d) {
            float e = expf(x[base + d * inner] - max_val);
            out[base + d * inner] = e;
            sum += e;
        }
        for (uint64_t d = 0; d < dim; ++d) out[base + d * inner] /= sum;
    }
}

void orc_softmax_bf16(const uint16_t* x, uint16_t* out, uint64_t outer, uint64_t dim,
                      uint64_t inner, int threads) {
    OMP_FOR for (uint64_t oi = 0; oi < outer * inner; ++oi) {
        uint64_t base = (oi / inner) * dim * inner + (oi % inner);
        float max_val = -INFINITY;
        for (uint64_t d = 0; d < dim; ++d) max_val = fmaxf(max_val, B2F(x[base + d * inner]));
        float sum = 0.0f;
        for (uint64_t d = 0; d < dim; ++d) sum += expf(B2F(x[base + d * inner]) - max_val);
        for (uint64_t d = 0; d < dim; ++d)
            out[base + d * inner] = F2B(expf(B2F(x[base + d * inner]) - max_val) / sum);
    }
}

/* ---- scale + mask + softmax: src/ops/attention.rs:41,60,63-79 ------------- */
static inline uint64_t valid_len(uint64_t r, uint64_t cols, const int32_t* lens,
                                 uint64_t rows_per_len, uint64_t causal_q_len) {
    uint64_t len = cols;
    if (lens) {
        int64_t l = lens[r / rows_per_len];
        if (l < 0) l = 0;
        if ((uint64_t)l < len) len = (uint64_t)l;
    }
    if (causal_q_len) {
        uint64_t q = r % causal_q_len;
        uint64_t lim = q + 1 + (cols - causal_q_len);
        if (lim < len) len = lim;
    }
    return len;
}

static void smax_row(const float* s_in, float* p, uint64_t cols, uint64_t len) {
    /* s_in already holds scaled+masked scores for j < len. */
    if (len == 0) {
        for (uint64_t j = 0; j < cols; ++j) p[j] = 0.0f;
        return;
    }
    float m = -INFINITY;
    for (uint64_t j = 0; j < len; ++j) m = fmaxf(m, s_in[j]);
    float sum = 0.0f;
    for (uint64_t j = 0; j < len; ++j) {
        p[j] = expf(s_in[j] - m);
        sum += p[j];
    }
    /* keys beyond len carry s = -inf: exp(-inf - m) = 0 contributes nothing */
    for (uint64_t j = 0; j < len; ++j) p[j] /= sum;
    for (uint64_t j = len; j < cols; ++j) p[j] = 0.0f;
}

void orc_scale_mask_softmax_f32(const float* x, float* out, uint64_t rows, uint64_t cols,
                                float scale, const float* mask, uint64_t mask_len,
                                const int32_t* lens, uint64_t rows_per_len,
                                uint64_t causal_q_len, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        float* pr = out + r * cols;
        uint64_t len = valid_len(r, cols, lens, rows_per_len, causal_q_len);
        for (uint64_t j = 0; j < len; ++j) {
            float s = xr[j] * scale;
            if (mask) s += mask[j % mask_len];
            pr[j] = s;
        }
        smax_row(pr, pr, cols, len);
    }
}

void orc_scale_mask_softmax_bf16(const uint16_t* x, uint16_t* out, uint64_t rows,
                                 uint64_t cols, float scale, const float* mask,
                                 uint64_t mask_len, const int32_t* lens,
                                 uint64_t rows_per_len, uint64_t causal_q_len, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * cols;
        uint16_t* orow = out + r * cols;
        uint64_t len = valid_len(r, cols, lens, rows_per_len, causal_q_len);
        float buf_stack[4096];
        float* buf = buf_stack;
        float* heap = 0;
        if (cols > 4096) {
            heap = (float*)__builtin_malloc(cols * sizeof(float));
            buf = heap;
        }
        for (uint64_t j = 0; j < len; ++j) {
            float s = B2F(xr[j]) * scale;
            if (mask) s += mask[j % mask_len];
            buf[j] = s;
        }
        smax_row(buf, buf, cols, len);
        for (uint64_t j = 0; j < cols; ++j) orow[j] = F2B(buf[j]);
        if (heap) __builtin_free(heap);
    }
}

/* ---- RoPE table: src/models/mistral.rs:102-108 ---------------------------- */
void orc_rope_table_f32(float theta, uint64_t head_dim, uint64_t max_pos, float* cos_out,
                        float* sin_out) {
    uint64_t half = head_dim / 2;
    for (uint64_t pos = 0; pos < max_pos; ++pos) {
        for (uint64_t i = 0; i < half; ++i) {
            float freq = powf(theta, (-2.0f * (float)i) / (float)head_dim);
            float angle = (float)pos * freq;
            cos_out[pos * half + i] = cosf(angle);
            sin_out[pos * half + i] = sinf(angle);
        }
    }
}

/* ---- RoPE: src/ops/attention.rs:139-155 ----------------------------------- */
static inline uint64_t rope_base(uint64_t t, uint64_t h, uint64_t tokens, uint64_t heads,
                                 uint64_t head_dim, int layout) {
    return layout == 0 ? (t * heads + h) * head_dim : (h * tokens + t) * head_dim;
}

void orc_rope_f32(const float* x, float* out, uint64_t tokens, uint64_t heads,
                  uint64_t head_dim, int layout, const float* cos_t, const float* sin_t,
                  const int32_t* positions, int threads) {
    uint64_t half = head_dim / 2;
    OMP_FOR for (uint64_t th = 0; th < tokens * heads; ++th) {
        uint64_t t = th / heads, h = th % heads;
        uint64_t base = rope_base(t, h, tokens, heads, head_dim, layout);
        uint64_t p = positions ? (uint64_t)positions[t] : t;
        for (uint64_t d = 0; d < half; ++d) {
            float x1 = x[base + d];
            float x2 = x[base + d + half];
            float c = cos_t[p * half + d];
            float s = sin_t[p * half + d];
            out[base + d] = x1 * c - x2 * s;
            out[base + d + half] = x1 * s + x2 * c;
        }
    }
}

void orc_rope_bf16(const uint16_t* x, uint16_t* out, uint64_t tokens, uint64_t heads,
                   uint64_t head_dim, int layout, const float* cos_t, const float* sin_t,
                   const int32_t* positions, int threads) {
    uint64_t half = head_dim / 2;
    OMP_FOR for (uint64_t th = 0; th < tokens * heads; ++th) {
        uint64_t t = th / heads, h = th % heads;
        uint64_t base = rope_base(t, h, tokens, heads, head_dim, layout);
        uint64_t p = positions ? (uint64_t)positions[t] : t;
        for (uint64_t d = 0; d < half; ++d) {
            float x1 = B2F(x[base + d]);
            float x2 = B2F(x[base + d + half]);
            float c = cos_t[p * half + d];
            float s = sin_t[p * half + d];
            float o1 = x1 * c - x2 * s;
            float o2 = x1 * s + x2 * c;
            out[base + d] = F2B(o1);
            out[base + d + half] = F2B(o2);
        }
    }
}

/* ---- argmax: src/tokenizer.rs:213-232 with k = 1 -------------------------- */
static inline uint32_t argmax_row(const float* v, uint64_t cols) {
    uint32_t bi = 0;
    float bv = v[0];
    for (uint64_t j = 1; j < cols; ++j) {
        float x = v[j];
        if (isnan(x)) continue;
        if (isnan(bv) || x > bv) {
            bv = x;
            bi = (uint32_t)j;
        }
    }
    return bi;
}

void orc_argmax_rows_f32(const float* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                         int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) idx[r] = argmax_row(x + r * cols, cols);
}

void orc_argmax_rows_bf16(const uint16_t* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                          int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * cols;
        uint32_t bi = 0;
        float bv = B2F(xr[0]);
        for (uint64_t j = 1; j < cols; ++j) {
            float v = B2F(xr[j]);
            if (isnan(v)) continue;
            if (isnan(bv) || v > bv) {
                bv = v;
                bi = (uint32_t)j;
            }
        }
        idx[r] = bi;
    }
}

/* ---- row reductions (reference inline loops) ------------------------------ */
static inline float reduce_step(int op, float acc, float v) {
    if (op == ORC_RED_SUM) return acc + v;
    if (op == ORC_RED_MAX) return fmaxf(acc, v);
    return acc + v * v;
}

void orc_reduce_rows_f32(int op, const float* x, uint64_t rows, uint64_t cols, float* out,
                         int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        float acc = op == ORC_RED_MAX ? -INFINITY : 0.0f;
        for (uint64_t j = 0; j < cols; ++j) acc = reduce_step(op, acc, x[r * cols + j]);
        out[r] = acc;
    }
}

void orc_reduce_rows_bf16(int op, const uint16_t* x, uint64_t rows, uint64_t cols,
                          float* out, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        float acc = op == ORC_RED_MAX ? -INFINITY : 0.0f;
        for (uint64_t j = 0; j < cols; ++j) acc = reduce_step(op, acc, B2F(x[r * cols + j]));
        out[r] = acc;
    }
}

/* ---- whole-tensor reductions in f64 --------------------------------------- */
#define ORC_CHUNK ((uint64_t)1 << 20)

static double combine_chunks(int op, const double* part, uint64_t nchunks) {
    double acc = op == ORC_RED_MAX ? -INFINITY : 0.0;
    for (uint64_t c = 0; c < nchunks; ++c)
        acc = op == ORC_RED_MAX ? fmax(acc, part[c]) : acc + part[c];
    return acc;
}

double orc_reduce_f32(int op, const float* x, uint64_t n, int threads) {
    uint64_t nchunks = (n + ORC_CHUNK - 1) / ORC_CHUNK;
    if (nchunks == 0) return op == ORC_RED_MAX ? -INFINITY : 0.0;
    double* part = (double*)__builtin_malloc(nchunks * sizeof(double));
    OMP_FOR for (uint64_t c = 0; c < nchunks; ++c) {
        uint64_t lo = c * ORC_CHUNK, hi = lo + ORC_CHUNK < n ? lo + ORC_CHUNK : n;
        double acc = op == ORC_RED_MAX ? -INFINITY : 0.0;
        for (uint64_t i = lo; i < hi; ++i) {
            double v = (double)x[i];
            if (op == ORC_RED_SUM) acc += v;
            else if (op == ORC_RED_MAX) acc = fmax(acc, v);
            else acc += v * v;
        }
        part[c] = acc;
    }
    double r = combine_chunks(op, part, nchunks);
    __builtin_free(part);
    return r;
}

double orc_reduce_bf16(int op, const uint16_t* x, uint64_t n, int threads) {
    uint64_t nchunks = (n + ORC_CHUNK - 1) / ORC_CHUNK;
    if (nchunks == 0) return op == ORC_RED_MAX ? -INFINITY : 0.0;
    double* part = (double*)__builtin_malloc(nchunks * sizeof(double));
    OMP_FOR for (uint64_t c = 0; c < nchunks; ++c) {
        uint64_t lo = c * ORC_CHUNK, hi = lo + ORC_CHUNK < n ? lo + ORC_CHUNK : n;
        double acc = op == ORC_RED_MAX ? -INFINITY : 0.0;
        for (uint64_t i = lo; i < hi; ++i) {
            double v = (double)B2F(x[i]);
            if (op == ORC_RED_SUM) acc += v;
            else if (op == ORC_RED_MAX) acc = fmax(acc, v);
            else acc += v * v;
        }
        part[c] = acc;
    }
    double r = combine_chunks(op, part, nchunks);
    __builtin_free(part);
    return r;
}

float orc_reduce_seq_f32(int op, const float* x, uint64_t n) {
    float acc = op == ORC_RED_MAX ? -INFINITY : 0.0f;
    for (uint64_t i = 0; i < n; ++i) acc = reduce_step(op, acc, x[i]);
    return acc;
}

/* ---- unary ops: src/ops/activation.rs (relu :4-19, gelu :39-56, gelu_quick
 * :58-74, sigmoid :126-140, tanh :142-156) and src/ops/math.rs (exp :4, ln :21,
 * sqrt :38, powf :55, clamp :72, neg :89, abs :106) --------------------------- */
static inline float unary1(int op, float x, float a, float b) {
    switch (op) {
        case ORC_RELU: return fmaxf(x, 0.0f); /* f32::max(x, 0.0): NaN -> 0 */
        case ORC_GELU: {
            /* 0.5 * x * (1.0 + ((2.0 / PI).sqrt() * (x + 0.044715 * x.powi(3))).tanh());
             * powi(3) evaluates (x * x) * x; every step rounded to f32. */
            const float k = sqrtf(2.0f / 3.14159265358979323846f);
            float half_x = 0.5f * x;
            float p = x * x;
            p = p * x;
            float t = 0.044715f * p;
            float u = x + t;
            float v = k * u;
            float th = tanhf(v);
            float w = 1.0f + th;
            return half_x * w;
        }
        case ORC_GELU_QUICK: {
            float n = -1.702f * x;
            float e = expf(n);
            float d = 1.0f + e;
            float r = 1.0f / d;
            return x * r;
        }
        case ORC_SIGMOID: {
            float e = expf(-x);
            float d = 1.0f + e;
            return 1.0f / d;
        }
        case ORC_TANH: return tanhf(x);
        case ORC_EXP: return expf(x);
        case ORC_LOG: return logf(x);
        case ORC_SQRT: return sqrtf(x);
        case ORC_POW: return powf(x, a);
        case ORC_CLAMP: { /* f32::clamp: x < min -> min; x > max -> max; NaN stays */
            float r = x;
            if (r < a) r = a;
            if (r > b) r = b;
            return r;
        }
        case ORC_NEG: return -x;
        default: return fabsf(x);
    }
}

void orc_unary_f32(int op, const float* x, float* out, uint64_t n, float a, float b, int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = unary1(op, x[i], a, b);
}

void orc_unary_bf16(int op, const uint16_t* x, uint16_t* out, uint64_t n, float a, float b,
                    int threads) {
    OMP_FOR for (uint64_t i = 0; i < n; ++i) out[i] = F2B(unary1(op, B2F(x[i]), a, b));
}

/* ---- LayerNorm: src/ops/norm.rs:92-113 -------------------------------------- */
static inline void layer_norm_row(const float* xr, const float* w, const float* bias, float* orow,
                                  uint64_t cols, float eps) {
    float sum = 0.0f;
    for (uint64_t i = 0; i < cols; ++i) sum += xr[i];
    float mean = sum / (float)cols;
    float sum_sq = 0.0f;
    for (uint64_t i = 0; i < cols; ++i) {
        float diff = xr[i] - mean;
        sum_sq += diff * diff;
    }
    float var = sum_sq / (float)cols;
    float sd = sqrtf(var + eps);
    for (uint64_t i = 0; i < cols; ++i) {
        float normalized = (xr[i] - mean) / sd;
        orow[i] = normalized * w[i] + bias[i];
    }
}

void orc_layer_norm_f32(const float* x, const float* w, const float* b, float* out, uint64_t rows,
                        uint64_t cols, float eps, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r)
        layer_norm_row(x + r * cols, w, b, out + r * cols, cols, eps);
}

void orc_layer_norm_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* out,
                         uint64_t rows, uint64_t cols, float eps, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        float* tmp = (float*)__builtin_malloc(4 * cols * sizeof(float));
        float *xf = tmp, *wf = tmp + cols, *bf = tmp + 2 * cols, *of = tmp + 3 * cols;
        for (uint64_t i = 0; i < cols; ++i) {
            xf[i] = B2F(x[r * cols + i]);
            wf[i] = B2F(w[i]);
            bf[i] = B2F(b[i]);
        }
        layer_norm_row(xf, wf, bf, of, cols, eps);
        for (uint64_t i = 0; i < cols; ++i) out[r * cols + i] = F2B(of[i]);
        __builtin_free(tmp);
    }
}

/* ---- repeat_kv: src/ops/attention.rs:184-198 (element size `es` bytes) --------- */
void orc_repeat_kv(const void* x, void* out, uint64_t batch, uint64_t heads, uint64_t seq,
                   uint64_t head_dim, uint64_t n_rep, uint64_t es) {
    const uint64_t per = seq * head_dim * es;
    for (uint64_t b = 0; b < batch; ++b)
        for (uint64_t h = 0; h < heads; ++h)
            for (uint64_t r = 0; r < n_rep; ++r) {
                const uint64_t src = (b * heads + h) * per;
                const uint64_t dst = (b * (heads * n_rep) + h * n_rep + r) * per;
                memcpy((char*)out + dst, (const char*)x + src, per);
            }
}

/* ---- KV-cache append: positions [cur, cur + new_len) of [batch, heads, max_seq, hd]
 * (src/cache/kv_cache.rs:55-85).  Returns -1 on overflow ("KV cache overflow"). -- */
int orc_kv_append(void* kc, void* vc, const void* k, const void* v, uint64_t batch, uint64_t heads,
                  uint64_t max_seq, uint64_t head_dim, uint64_t cur, uint64_t new_len, uint64_t es) {
    if (cur > max_seq || new_len > max_seq - cur) return -1;
    const uint64_t row = head_dim * es;
    for (uint64_t bh = 0; bh < batch * heads; ++bh) {
        memcpy((char*)kc + (bh * max_seq + cur) * row, (const char*)k + bh * new_len * row, new_len * row);
        memcpy((char*)vc + (bh * max_seq + cur) * row, (const char*)v + bh * new_len * row, new_len * row);
    }
    return 0;
}

/* ---- decode attention: the inline attention of scaled_dot_product_attention
 * (src/ops/attention.rs:41-87) for one query token per (batch, head), with the
 * keys of batch b limited to j < lens[b] (the decode KV length) and query head
 * qh reading kv head qh / (q_heads / kv_heads) (repeat_kv, attention.rs:161-201).
 * dot sequential in f32, * scale, max, exp(s - max) with a sequential sum, divide,
 * then out[d] = sum_j p_j * v[j][d] sequentially.  A batch with length 0 gives
 * zeros.  The caches are [batch, kv_heads, max_seq, head_dim]. ---------------- */
static void decode_attn_one(const float* q, const float* kc, const float* vc, float* out, uint64_t len,
                            uint64_t d, float scale, float* p) {
    if (len == 0) {
        for (uint64_t i = 0; i < d; ++i) out[i] = 0.0f;
        return;
    }
    float mx = -INFINITY;
    for (uint64_t j = 0; j < len; ++j) {
        float dot = 0.0f;
        for (uint64_t i = 0; i < d; ++i) dot += q[i] * kc[j * d + i];
        p[j] = dot * scale;
        mx = fmaxf(mx, p[j]);
    }
    float sum = 0.0f;
    for (uint64_t j = 0; j < len; ++j) {
        p[j] = expf(p[j] - mx);
        sum += p[j];
    }
    for (uint64_t j = 0; j < len; ++j) p[j] /= sum;
    for (uint64_t i = 0; i < d; ++i) {
        float acc = 0.0f;
        for (uint64_t j = 0; j < len; ++j) acc += p[j] * vc[j * d + i];
        out[i] = acc;
    }
}

void orc_decode_attention_f32(const float* q, const float* kc, const float* vc, const int32_t* lens,
                              float* out, uint64_t batch, uint64_t q_heads, uint64_t kv_heads,
                              uint64_t max_seq, uint64_t head_dim, float scale, int threads) {
    const uint64_t rep = q_heads / kv_heads;
    OMP_FOR for (uint64_t bh = 0; bh < batch * q_heads; ++bh) {
        const uint64_t b = bh / q_heads, h = bh % q_heads, kvh = h / rep;
        uint64_t len = max_seq;
        if (lens) len = lens[b] < 0 ? 0 : ((uint64_t)lens[b] < max_seq ? (uint64_t)lens[b] : max_seq);
        float* p = (float*)__builtin_malloc((max_seq ? max_seq : 1) * sizeof(float));
        const uint64_t kv_off = (b * kv_heads + kvh) * max_seq * head_dim;
        decode_attn_one(q + bh * head_dim, kc + kv_off, vc + kv_off, out + bh * head_dim, len, head_dim,
                        scale, p);
        __builtin_free(p);
    }
}

void orc_decode_attention_bf16(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                               const int32_t* lens, uint16_t* out, uint64_t batch, uint64_t q_heads,
                               uint64_t kv_heads, uint64_t max_seq, uint64_t head_dim, float scale,
                               int threads) {
    const uint64_t rep = q_heads / kv_heads;
    OMP_FOR for (uint64_t bh = 0; bh < batch * q_heads; ++bh) {
        const uint64_t b = bh / q_heads, h = bh % q_heads, kvh = h / rep;
        uint64_t len = max_seq;
        if (lens) len = lens[b] < 0 ? 0 : ((uint64_t)lens[b] < max_seq ? (uint64_t)lens[b] : max_seq);
        const uint64_t n = len * head_dim, kv_off = (b * kv_heads + kvh) * max_seq * head_dim;
        float* buf = (float*)__builtin_malloc((2 * n + 2 * head_dim + len + 1) * sizeof(float));
        float *kf = buf, *vf = buf + n, *qf = buf + 2 * n, *of = qf + head_dim, *p = of + head_dim;
        for (uint64_t i = 0; i < n; ++i) {
            kf[i] = B2F(kc[kv_off + i]);
            vf[i] = B2F(vc[kv_off + i]);
        }
        for (uint64_t i = 0; i < head_dim; ++i) qf[i] = B2F(q[bh * head_dim + i]);
        decode_attn_one(qf, kf, vf, of, len, head_dim, scale, p);
        for (uint64_t i = 0; i < head_dim; ++i) out[bh * head_dim + i] = F2B(of[i]);
        __builtin_free(buf);
    }
}

/* ---- token sampling (src/tokenizer.rs:166-232, src/pipeline.rs:181-205) ---- */
/* softmax_with_temperature, src/tokenizer.rs:166-180 */
static void softmax_temperature_row(const float* x, uint64_t n, float t, float* p) {
    float m = -INFINITY;
    for (uint64_t i = 0; i < n; ++i) m = fmaxf(m, x[i] / t); /* fold(NEG_INFINITY, f32::max) */
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; ++i) sum += expf(x[i] / t - m);
    for (uint64_t i = 0; i < n; ++i) p[i] = expf(x[i] / t - m) / sum;
}

void orc_softmax_temperature_f32(const float* x, uint64_t rows, uint64_t vocab, float temperature,
                                 float* probs, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r)
        softmax_temperature_row(x + r * vocab, vocab, temperature, probs + r * vocab);
}

void orc_softmax_temperature_bf16(const uint16_t* x, uint64_t rows, uint64_t vocab, float temperature,
                                  float* probs, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        float* row = probs + r * vocab;
        for (uint64_t i = 0; i < vocab; ++i) row[i] = B2F(x[r * vocab + i]); /* to_f32_vec */
        softmax_temperature_row(row, vocab, temperature, row);
    }
}

typedef struct {
    uint32_t idx;
    float p;
} orc_prob_t;

/* sort_by(|a, b| b.1.partial_cmp(&a.1)) is a stable sort: descending by
 * probability, equal probabilities keep ascending index order. */
static int prob_desc_cmp(const void* a, const void* b) {
    const orc_prob_t* x = (const orc_prob_t*)a;
    const orc_prob_t* y = (const orc_prob_t*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

uint32_t orc_sample_probs(const float* probs, uint64_t vocab, uint64_t top_k, float top_p, float u) {
    if (vocab >= 2)
        for (uint64_t i = 0; i < vocab; ++i)
            if (isnan(probs[i])) return ORC_SAMPLE_INVALID; /* partial_cmp(..).unwrap() panics */
    orc_prob_t* s = (orc_prob_t*)malloc((vocab ? vocab : 1) * sizeof(orc_prob_t));
    for (uint64_t i = 0; i < vocab; ++i) {
        s[i].idx = (uint32_t)i;
        s[i].p = probs[i];
    }
    qsort(s, vocab, sizeof(orc_prob_t), prob_desc_cmp);
    uint64_t keep;
    if (top_p < 1.0f) { /* sample_top_p, src/tokenizer.rs:182-211 */
        float cumsum = 0.0f;
        keep = vocab;
        for (uint64_t i = 0; i < vocab; ++i) {
            cumsum += s[i].p;
            if (cumsum >= top_p) {
                keep = i + 1;
                break;
            }
        }
    } else { /* sample_top_k, src/tokenizer.rs:213-232 */
        keep = top_k < vocab ? top_k : vocab;
    }
    float total = 0.0f;
    for (uint64_t i = 0; i < keep; ++i) total += s[i].p;
    const float r = u * total;
    uint32_t tok = keep ? s[keep - 1].idx : 0u; /* last().map(..).unwrap_or(0) */
    float cum = 0.0f;
    for (uint64_t i = 0; i < keep; ++i) {
        cum += s[i].p;
        if (cum >= r) {
            tok = s[i].idx;
            break;
        }
    }
    free(s);
    return tok;
}

void orc_sample_f32(const float* logits, uint64_t rows, uint64_t vocab, float temperature, uint64_t top_k,
                    float top_p, const float* uniforms, uint32_t* tokens, float* probs, int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        float* p = probs ? probs + r * vocab : (float*)malloc((vocab ? vocab : 1) * sizeof(float));
        softmax_temperature_row(logits + r * vocab, vocab, temperature, p);
        tokens[r] = orc_sample_probs(p, vocab, top_k, top_p, uniforms[r]);
        if (!probs) free(p);
    }
}

void orc_sample_bf16(const uint16_t* logits, uint64_t rows, uint64_t vocab, float temperature,
                     uint64_t top_k, float top_p, const float* uniforms, uint32_t* tokens, float* probs,
                     int threads) {
    OMP_FOR for (uint64_t r = 0; r < rows; ++r) {
        float* p = probs ? probs + r * vocab : (float*)malloc((vocab ? vocab : 1) * sizeof(float));
        for (uint64_t i = 0; i < vocab; ++i) p[i] = B2F(logits[r * vocab + i]);
        softmax_temperature_row(p, vocab, temperature, p);
        tokens[r] = orc_sample_probs(p, vocab, top_k, top_p, uniforms[r]);
        if (!probs) free(p);
    }
}

/* ---- weight decoding (src/loading/safetensors.rs:48-82) -------------------- */
/* half::f16 -> f32: exact; NaN keeps its payload with the quiet bit set */
float orc_decode_f16_bits_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            float v = (float)man * 0x1p-24f; /* subnormal half: exact in f32 */
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = man == 0 ? (sign | 0x7F800000u) : (sign | 0x7FC00000u | (man << 13));
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float decode_elem(const unsigned char* s, uint64_t i, int dtype) {
    if (dtype == ORC_WDT_F32) {
        float f;
        memcpy(&f, s + 4 * i, 4); /* f32::from_le_bytes on a little-endian host */
        return f;
    }
    uint16_t h;
    memcpy(&h, s + 2 * i, 2);
    if (dtype == ORC_WDT_F16) return orc_decode_f16_bits_f32(h);
    return B2F(h);
}

void orc_decode_weights_f32(const void* src, uint64_t n, int dtype, float* out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = decode_elem((const unsigned char*)src, i, dtype);
}

void orc_decode_weights_bf16(const void* src, uint64_t n, int dtype, uint16_t* out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(decode_elem((const unsigned char*)src, i, dtype));
}
