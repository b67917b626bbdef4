/*
 * kernrt_oracle.c — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of KernRT's scalar `reference` backend for the per-row
 * layer ops, used as the parity checker for the CUDA backend.  Nothing in the
 * product links or calls this file: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm load it, and only as the checker or
 * as the timed CPU baseline.
 *
 * Every function follows the reference loop for loop (KernRT is Rust; all
 * citations are paths inside that crate).  The arithmetic is f32 with no FMA
 * contraction (build with -ffp-contract=off, no fast-math), left-to-right
 * reductions, and the platform libm for powf/sinf/cosf/expf: Rust's std calls
 * the same glibc entry points on Linux and never contracts to FMA, so on one
 * host this file and the Rust `reference` backend produce identical bits.
 *
 * Parity pinning: the reference itself cannot be built here (Rust, no cargo),
 * so the restatement is pinned against the reference's own known-answer tests
 * (tests/test_oracle_golden.py restates them with their source lines).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>

#include <pthread.h>
#include <unistd.h>

#define KRO_Q8_BLOCK 32 /* src/ops/quant.rs:714 Q8_0_BLOCK */

/* ------------------------------------------------------------------ */
/* Number formats                                                       */
/* ------------------------------------------------------------------ */

static inline float f32_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* src/ops/dot.rs:222-224 bf16_to_f32: the bf16 pattern is the top half. */
float kro_bf16_to_f32(uint16_t bits) { return f32_from_bits((uint32_t)bits << 16); }

/* src/ops/quant.rs:707-711 f32_to_bf16_bits: round to nearest even on the
 * discarded low half (plain wrapping add, no NaN special case). */
uint16_t kro_f32_to_bf16_bits(float v) {
    uint32_t bits = f32_bits(v);
    uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

/* src/ops/quant.rs:722-758 f32_to_f16_bits: IEEE binary16, round to nearest
 * even, with subnormal and overflow handling; NaN keeps a quiet payload bit. */
uint16_t kro_f32_to_f16_bits(float value) {
    uint32_t bits = f32_bits(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exp = (int32_t)((bits >> 23) & 0xffu) - 127 + 15;
    uint32_t mant = bits & 0x007fffffu;
    if (((bits >> 23) & 0xffu) == 0xffu)
        return (uint16_t)(sign | 0x7c00u | (mant != 0 ? 0x0200u : 0u));
    if (exp <= 0) {
        if (exp < -10) return sign;
        uint32_t significand = mant | 0x00800000u;
        uint32_t shift = (uint32_t)(14 - exp);
        uint32_t base = significand >> shift;
        uint32_t rem = significand & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        uint32_t rounded = base + ((rem > halfway || (rem == halfway && (base & 1u))) ? 1u : 0u);
        return (uint16_t)(sign | (uint16_t)rounded);
    }
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t base = mant >> 13;
    uint32_t rem = mant & 0x1fffu;
    uint32_t rounded = base + ((rem > 0x1000u || (rem == 0x1000u && (base & 1u))) ? 1u : 0u);
    if (rounded == 0x400u) { exp += 1; rounded = 0; }
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | (uint16_t)(exp << 10) | (uint16_t)rounded);
}

/* src/ops/quant.rs:764-769 f16_scale_to_f32: the fast widening used for
 * Q8_0x4 scales.  It assumes a normal half, so a zero scale widens to 2^-15
 * (harmless: that block's quants are all zero). */
float kro_f16_scale_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits >> 15) << 31;
    uint32_t exp = (uint32_t)((bits >> 10) & 0x1fu);
    uint32_t mant = (uint32_t)(bits & 0x03ffu);
    return f32_from_bits(sign | ((exp + 112u) << 23) | (mant << 13));
}

/* Rust `f32::round` then `clamp(-127, 127)` then `as i8` (saturating, NaN -> 0),
 * as written at src/ops/quant.rs:871. */
static inline int8_t q8_code(float v) {
    float r = roundf(v);
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    if (r != r) return 0;
    return (int8_t)(int)r;
}

/* ------------------------------------------------------------------ */
/* Q8_0 activation quantisation                                         */
/* ------------------------------------------------------------------ */

/* src/ops/quant.rs:856-874 Q8Vec::quantize_into.  `quants` holds
 * ceil(n/32)*32 entries (the tail block is zero padded), `scales` and
 * `scales_f16` one entry per block.  `scales_f16` may be NULL. */
void kro_q8_quantize_into(const float *x, size_t n, int8_t *quants, float *scales,
                          uint16_t *scales_f16) {
    size_t blocks = (n + KRO_Q8_BLOCK - 1) / KRO_Q8_BLOCK;
    memset(quants, 0, blocks * KRO_Q8_BLOCK);
    for (size_t b = 0; b < blocks; ++b) {
        size_t lo = b * KRO_Q8_BLOCK;
        size_t hi = lo + KRO_Q8_BLOCK < n ? lo + KRO_Q8_BLOCK : n;
        float amax = 0.0f;
        for (size_t i = lo; i < hi; ++i) amax = fmaxf(amax, fabsf(x[i]));
        float d = amax / 127.0f;
        float inv = d > 0.0f ? 1.0f / d : 0.0f;
        scales[b] = d;
        if (scales_f16) scales_f16[b] = kro_f32_to_f16_bits(d);
        for (size_t i = lo; i < hi; ++i) quants[i] = q8_code(x[i] * inv);
    }
}

/* src/ops/quant.rs:124-165 Q8_0x4::from_f32: quantise [out, in] f32 weights
 * four rows at a time into 136-byte blocks {u16 scales[4]; i8 quants[128]},
 * quants interleaved in 4-byte lanes.  Used by tests to build Q8_0x4 tables. */
int kro_q8_0x4_pack(const float *w, size_t out_dim, size_t in_dim, uint8_t *blocks_out) {
    if (in_dim % KRO_Q8_BLOCK != 0 || out_dim % 4 != 0) return -1;
    size_t groups = out_dim / 4, blocks = in_dim / KRO_Q8_BLOCK;
    for (size_t g = 0; g < groups; ++g) {
        for (size_t b = 0; b < blocks; ++b) {
            uint8_t *blk = blocks_out + (g * blocks + b) * 136;
            uint16_t *sc = (uint16_t *)blk;
            int8_t *qs = (int8_t *)(blk + 8);
            memset(blk, 0, 136);
            for (size_t rig = 0; rig < 4; ++rig) {
                const float *src = w + (g * 4 + rig) * in_dim + b * KRO_Q8_BLOCK;
                float amax = 0.0f;
                for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));
                float scale = amax / 127.0f;
                sc[rig] = kro_f32_to_f16_bits(scale);
                float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
                for (int seg = 0; seg < 8; ++seg)
                    for (int lane = 0; lane < 4; ++lane)
                        qs[seg * 16 + rig * 4 + lane] = q8_code(src[seg * 4 + lane] * inv);
            }
        }
    }
    return 0;
}

/* src/ops/quant.rs:198-220 Q8_0x4::to_row_major: de-interleave to row-major
 * Q8_0 (int8 [out*in] + f32 scales [out*in/32]), scales widened with
 * f16_scale_to_f32. */
void kro_q8_0x4_to_row_major(const uint8_t *blocks_in, size_t out_dim, size_t in_dim,
                             int8_t *quants, float *scales) {
    size_t blocks = in_dim / KRO_Q8_BLOCK;
    for (size_t g = 0; g < out_dim / 4; ++g) {
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *blk = blocks_in + (g * blocks + b) * 136;
            uint16_t sc[4];
            memcpy(sc, blk, 8);
            const int8_t *qs = (const int8_t *)(blk + 8);
            for (size_t rig = 0; rig < 4; ++rig) {
                size_t row = g * 4 + rig;
                scales[row * blocks + b] = kro_f16_scale_to_f32(sc[rig]);
                int8_t *dst = quants + row * in_dim + b * KRO_Q8_BLOCK;
                for (int seg = 0; seg < 8; ++seg)
                    for (int lane = 0; lane < 4; ++lane)
                        dst[seg * 4 + lane] = qs[seg * 16 + rig * 4 + lane];
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* Embedding rows: Matrix::decode_row                                   */
/* ------------------------------------------------------------------ */

/* src/ops/quant.rs:659-693 decode_row, F32 arm. */
void kro_decode_row_f32(const float *table, size_t in_dim, size_t index, float *out) {
    memcpy(out, table + index * in_dim, in_dim * sizeof(float));
}

/* src/ops/quant.rs:666-669 decode_row, Bf16 arm. */
void kro_decode_row_bf16(const uint16_t *table, size_t in_dim, size_t index, float *out) {
    const uint16_t *row = table + index * in_dim;
    for (size_t i = 0; i < in_dim; ++i) out[i] = kro_bf16_to_f32(row[i]);
}

/* src/ops/quant.rs:670-690 decode_row, Q8_0 arm: one f32 multiply per value. */
void kro_decode_row_q8_0(const int8_t *quants, const float *scales, size_t in_dim, size_t index,
                         float *out) {
    size_t blocks = in_dim / KRO_Q8_BLOCK;
    const int8_t *qs = quants + index * in_dim;
    const float *ss = scales + index * blocks;
    for (size_t b = 0; b < blocks; ++b)
        for (size_t i = 0; i < KRO_Q8_BLOCK; ++i)
            out[b * KRO_Q8_BLOCK + i] = (float)qs[b * KRO_Q8_BLOCK + i] * ss[b];
}

/* src/ops/quant.rs:174-190 Q8_0x4::row (decode_row's Q8_0x4 arm, :691). */
void kro_decode_row_q8_0x4(const uint8_t *blocks_in, size_t in_dim, size_t index, float *out) {
    size_t blocks = in_dim / KRO_Q8_BLOCK;
    size_t g = index / 4, rig = index % 4;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = blocks_in + (g * blocks + b) * 136;
        uint16_t sc[4];
        memcpy(sc, blk, 8);
        const int8_t *qs = (const int8_t *)(blk + 8);
        float scale = kro_f16_scale_to_f32(sc[rig]);
        for (int seg = 0; seg < 8; ++seg)
            for (int lane = 0; lane < 4; ++lane)
                out[b * KRO_Q8_BLOCK + seg * 4 + lane] = (float)qs[seg * 16 + rig * 4 + lane] * scale;
    }
}

/* ------------------------------------------------------------------ */
/* Row ops: src/backends/reference.rs                                   */
/* ------------------------------------------------------------------ */

/* One row of reference.rs:161-178 rms_norm: sequential sum of squares,
 * divide by dim, add eps, 1/sqrt, then w * (scale * x). */
static void rms_norm_row(float *dst, const float *src, const float *w, size_t dim, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < dim; ++i) ss += src[i] * src[i];
    ss /= (float)dim;
    ss += eps;
    float scale = 1.0f / sqrtf(ss);
    for (size_t i = 0; i < dim; ++i) dst[i] = w[i] * (scale * src[i]);
}

/* src/backends/reference.rs:161-178 rms_norm over `rows` rows of `dim`. */
void kro_rms_norm(float *out, const float *x, const float *w, size_t rows, size_t dim, float eps) {
    for (size_t r = 0; r < rows; ++r) rms_norm_row(out + r * dim, x + r * dim, w, dim, eps);
}

/* One row of reference.rs:180-207 qk_norm: rms_norm per head slice, in place. */
static void qk_norm_row(float *v, size_t width, size_t head, const float *w, float eps) {
    for (size_t h = 0; h < width / head; ++h) {
        float *at = v + h * head;
        float ss = 0.0f;
        for (size_t i = 0; i < head; ++i) ss += at[i] * at[i];
        ss /= (float)head;
        ss += eps;
        float scale = 1.0f / sqrtf(ss);
        for (size_t i = 0; i < head; ++i) at[i] = w[i] * (scale * at[i]);
    }
}

/* src/backends/reference.rs:180-207 qk_norm. */
void kro_qk_norm(float *v, size_t rows, size_t width, size_t head, const float *w, float eps) {
    for (size_t r = 0; r < rows; ++r) qk_norm_row(v + r * width, width, head, w, eps);
}

/* One row of reference.rs:209-257 rope.  The frequency, angle and sin/cos are
 * recomputed per element exactly as the reference does. */
static void rope_row(float *q, float *k, size_t q_width, size_t kv_width, uint64_t pos,
                     size_t head, float theta, int interleaved) {
    if (interleaved) {
        size_t i = 0;
        while (i + 1 < q_width) {
            size_t head_dim = i % head;
            float freq = 1.0f / powf(theta, (float)head_dim / (float)head);
            float angle = (float)pos * freq;
            float s = sinf(angle), c = cosf(angle);
            float q0 = q[i], q1 = q[i + 1];
            q[i] = q0 * c - q1 * s;
            q[i + 1] = q0 * s + q1 * c;
            if (i < kv_width) {
                float k0 = k[i], k1 = k[i + 1];
                k[i] = k0 * c - k1 * s;
                k[i + 1] = k0 * s + k1 * c;
            }
            i += 2;
        }
    } else {
        size_t half = head / 2;
        float *vecs[2] = {q, k};
        size_t widths[2] = {q_width, kv_width};
        for (int t = 0; t < 2; ++t) {
            for (size_t h = 0; h < widths[t] / head; ++h) {
                float *at = vecs[t] + h * head;
                for (size_t i = 0; i < half; ++i) {
                    float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head);
                    float angle = (float)pos * freq;
                    float s = sinf(angle), c = cosf(angle);
                    float lo = at[i], hi = at[i + half];
                    at[i] = lo * c - hi * s;
                    at[i + half] = lo * s + hi * c;
                }
            }
        }
    }
}

/* src/backends/reference.rs:209-257 rope, `positions[r]` for row r. */
void kro_rope(float *q, float *k, size_t q_width, size_t kv_width, size_t rows,
              const uint64_t *positions, size_t head, float theta, int interleaved) {
    for (size_t r = 0; r < rows; ++r)
        rope_row(q + r * q_width, k + r * kv_width, q_width, kv_width, positions[r], head, theta,
                 interleaved);
}

/* src/backends/reference.rs:81-83 silu, used by silu_mul at :395-400. */
static inline float silu(float x) { return x / (1.0f + expf(-x)); }

/* src/backends/reference.rs:395-400 silu_mul: gate = silu(gate) * up. */
void kro_silu_mul(float *gate, const float *up, size_t len) {
    for (size_t i = 0; i < len; ++i) gate[i] = silu(gate[i]) * up[i];
}

/* src/backends/reference.rs:308-313 add_in_place. */
void kro_add_in_place(float *dst, const float *src, size_t len) {
    for (size_t i = 0; i < len; ++i) dst[i] += src[i];
}

/* src/backends/reference.rs:315-363 mul: out[oo+i] = a[ao+i] * b[bo+i] in
 * index order.  The pointers may alias (the caller passes the same base for a
 * shared buffer), so the sequential read-then-write order is part of the
 * semantics. */
void kro_mul(float *out, size_t out_off, const float *a, size_t a_off, const float *b,
             size_t b_off, size_t len) {
    for (size_t i = 0; i < len; ++i) {
        float x = a[a_off + i];
        float y = b[b_off + i];
        out[out_off + i] = x * y;
    }
}

/* src/backends/reference.rs:142-149 copy: copy_within (memmove) on one buffer. */
void kro_copy(const float *src, size_t src_off, float *dst, size_t dst_off, size_t len) {
    memmove(dst + dst_off, src + src_off, len * sizeof(float));
}

/* src/backends/reference.rs:490-503 conv_rows: causal depthwise conv,
 * out[r,i] = sum_j kernel[i*k+j] * x[r-k+1+j, i], zero padded, j order. */
void kro_conv_rows(const float *x, const float *kernel, float *out, size_t rows, size_t dim,
                   size_t k) {
    for (size_t r = 0; r < rows; ++r) {
        for (size_t i = 0; i < dim; ++i) {
            float acc = 0.0f;
            for (size_t j = 0; j < k; ++j) {
                long h = (long)r - ((long)k - 1) + (long)j;
                if (h >= 0) acc += kernel[i * k + j] * x[(size_t)h * dim + i];
            }
            out[r * dim + i] = acc;
        }
    }
}

/* src/backends/reference.rs:365-370 conv_prefill. */
void kro_conv_prefill(float *out, const float *x, const float *kernel, size_t rows, size_t dim,
                      size_t k) {
    kro_conv_rows(x, kernel, out, rows, dim, k);
}

/* src/backends/reference.rs:372-393 conv_decode: output is the last row of
 * conv_rows(state ++ x); then the ring drops its oldest row and gains x.
 * x is read in full before out is written, so out may alias x. */
void kro_conv_decode(float *out, const float *x, const float *kernel, float *state, size_t dim,
                     size_t k) {
    size_t hist_len = k - 1;
    float *hist = (float *)malloc(k * dim * sizeof(float));
    float *full = (float *)malloc(k * dim * sizeof(float));
    memcpy(hist, state, hist_len * dim * sizeof(float));
    memcpy(hist + hist_len * dim, x, dim * sizeof(float));
    kro_conv_rows(hist, kernel, full, k, dim, k);
    memcpy(out, full + (k - 1) * dim, dim * sizeof(float));
    if (hist_len > 0) {
        if (hist_len > 1) memmove(state, state + dim, (hist_len - 1) * dim * sizeof(float));
        memcpy(state + (hist_len - 1) * dim, hist + hist_len * dim, dim * sizeof(float));
    }
    free(hist);
    free(full);
}

/* ------------------------------------------------------------------ */
/* Embedding tables and the benchmark chains                            */
/* ------------------------------------------------------------------ */

/* Storage kinds, as src/ops/quant.rs:565-572 Matrix::kind names them. */
enum { KRO_F32 = 0, KRO_BF16 = 1, KRO_Q8_0 = 2, KRO_Q8_0X4 = 3 };

typedef struct {
    int kind;
    size_t vocab, dim;
    const void *data;     /* f32 / u16 bf16 / i8 quants / Q8_0x4 blocks */
    const float *scales;  /* Q8_0 block scales */
} kro_table;

/* src/backends/reference.rs:133-140 embed: decode_row of the token's row. */
void kro_embed(const kro_table *t, size_t token, float *out) {
    switch (t->kind) {
    case KRO_F32: kro_decode_row_f32((const float *)t->data, t->dim, token, out); break;
    case KRO_BF16: kro_decode_row_bf16((const uint16_t *)t->data, t->dim, token, out); break;
    case KRO_Q8_0:
        kro_decode_row_q8_0((const int8_t *)t->data, t->scales, t->dim, token, out);
        break;
    default: kro_decode_row_q8_0x4((const uint8_t *)t->data, t->dim, token, out); break;
    }
}

/* Flat-argument form for ctypes callers. */
void kro_embed_rows(int kind, const void *data, const float *scales, size_t vocab, size_t dim,
                    const int32_t *tokens, size_t rows, float *out) {
    kro_table t = {kind, vocab, dim, data, scales};
    for (size_t r = 0; r < rows; ++r) kro_embed(&t, (size_t)tokens[r], out + r * dim);
}

/*
 * The layer-op chain of a Llama-family attention block, with every stage in
 * the driver's order (src/arch/llm/llama.rs:734-770 prefill_rows; the row ops
 * only, contractions elided):
 *
 *   x    = embed(tokens)                 (optional: else x is an input)
 *   xb   = rms_norm(x, w_att)
 *   q, k = qk_norm(q, w_q), qk_norm(k, w_k)   (optional, Qwen3)
 *   q, k = rope(q, k, positions)
 *   gate = silu(gate) * up
 *   x    = x + resid
 *   codes, scales = Q8_0(rms_norm(x, w_final))  (optional, Qwen3 final norm;
 *                   quantisation as src/ops/quant.rs:856-874)
 *
 * Rows are independent, so one row is processed start to finish; the result
 * is identical to running each op over all rows in turn.
 */
typedef struct {
    size_t rows, dim, q_dim, kv_dim, hidden, head;
    float eps, theta, final_eps;
    int interleaved;
    kro_table table;          /* used when tokens != NULL */
    const int32_t *tokens;    /* [rows] or NULL */
    const uint64_t *positions;/* [rows] */
    const float *w_att;       /* [dim] */
    const float *w_q, *w_k;   /* [head] or NULL */
    const float *w_final;     /* [dim] or NULL */
    float *x;                 /* [rows, dim]: input when tokens == NULL; output x + resid */
    float *xb;                /* [rows, dim] out */
    float *q, *k;             /* [rows, q_dim], [rows, kv_dim] in/out */
    float *gate;              /* [rows, hidden] in/out */
    const float *up;          /* [rows, hidden] */
    const float *resid;       /* [rows, dim] */
    int8_t *codes;            /* [rows, ceil(dim/32)*32] out when w_final */
    float *scales;            /* [rows, ceil(dim/32)] out when w_final */
    uint16_t *scales_f16;     /* [rows, ceil(dim/32)] out, may be NULL */
} kro_chain;

static void chain_row(const kro_chain *c, size_t r, float *tmp) {
    size_t dim = c->dim;
    float *x = c->x + r * dim;
    if (c->tokens) kro_embed(&c->table, (size_t)c->tokens[r], x);
    rms_norm_row(c->xb + r * dim, x, c->w_att, dim, c->eps);
    float *q = c->q + r * c->q_dim, *k = c->k + r * c->kv_dim;
    if (c->w_q) qk_norm_row(q, c->q_dim, c->head, c->w_q, c->eps);
    if (c->w_k) qk_norm_row(k, c->kv_dim, c->head, c->w_k, c->eps);
    rope_row(q, k, c->q_dim, c->kv_dim, c->positions[r], c->head, c->theta, c->interleaved);
    kro_silu_mul(c->gate + r * c->hidden, c->up + r * c->hidden, c->hidden);
    kro_add_in_place(x, c->resid + r * dim, dim);
    if (c->w_final) {
        size_t blocks = (dim + KRO_Q8_BLOCK - 1) / KRO_Q8_BLOCK;
        rms_norm_row(tmp, x, c->w_final, dim, c->final_eps);
        kro_q8_quantize_into(tmp, dim, c->codes + r * blocks * KRO_Q8_BLOCK, c->scales + r * blocks,
                             c->scales_f16 ? c->scales_f16 + r * blocks : NULL);
    }
}

/* Single-threaded, like KernRT's cpu backend for these ops. */
void kro_chain_run(const kro_chain *c) {
    float *tmp = (float *)malloc(c->dim * sizeof(float));
    for (size_t r = 0; r < c->rows; ++r) chain_row(c, r, tmp);
    free(tmp);
}

/* Row-parallel over `threads` host threads (contiguous row ranges, one
 * pthread each).  Rows are independent, so the bits equal kro_chain_run's. */
typedef struct { const kro_chain *c; size_t lo, hi; } chain_span;

static void *chain_worker(void *arg) {
    const chain_span *s = (const chain_span *)arg;
    float *tmp = (float *)malloc(s->c->dim * sizeof(float));
    for (size_t r = s->lo; r < s->hi; ++r) chain_row(s->c, r, tmp);
    free(tmp);
    return NULL;
}

void kro_chain_run_mt(const kro_chain *c, int threads) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > c->rows) threads = c->rows ? (int)c->rows : 1;
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    chain_span *span = (chain_span *)malloc(sizeof(chain_span) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        span[t].c = c;
        span[t].lo = c->rows * (size_t)t / (size_t)threads;
        span[t].hi = c->rows * (size_t)(t + 1) / (size_t)threads;
        pthread_create(&tid[t], NULL, chain_worker, &span[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    free(span);
}

size_t kro_chain_struct_size(void) { return sizeof(kro_chain); }

/*
 * The LFM2 short-conv block's row ops in the driver's order
 * (src/arch/llm/lfm2.rs:584-624, contractions elided), over one sequence of
 * `rows` rows with bcx = [B | C | x] thirds per row (lfm2.rs:9-15):
 *
 *   h[r]  = B[r] * x[r]            (mul, once per row)
 *   co    = conv_prefill(h)        (causal, zero padded before row 0)
 *   ring  = last min(rows, k-1) rows of h, right-aligned   (copy)
 *   cy[r] = C[r] * co[r]           (mul, once per row)
 *
 * `h` and `co` are caller scratch of rows*dim each.
 */
void kro_lfm2_conv_block(const float *bcx, const float *kernel, float *ring, float *cy, float *h,
                         float *co, size_t rows, size_t dim, size_t k) {
    for (size_t r = 0; r < rows; ++r)
        kro_mul(h, r * dim, bcx, r * 3 * dim, bcx, r * 3 * dim + 2 * dim, dim);
    kro_conv_prefill(co, h, kernel, rows, dim, k);
    if (k > 1) {
        size_t take = rows < k - 1 ? rows : k - 1;
        kro_copy(h, (rows - take) * dim, ring, (k - 1 - take) * dim, take * dim);
    }
    for (size_t r = 0; r < rows; ++r) kro_mul(cy, r * dim, bcx, r * 3 * dim + dim, co, r * dim, dim);
}

/* Host threads available to this process. */
int kro_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

/* ------------------------------------------------------------------ */
/* Contractions (the reference backend's, src/backends/reference.rs)   */
/* ------------------------------------------------------------------ */

/* reference.rs:73-79 dot: one f32 accumulator, left to right, multiply then
 * add (no fused multiply-add). */
static float dot_seq(const float *a, const float *b, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += a[i] * b[i];
    return sum;
}

typedef struct {
    kro_table w;
    size_t out_dim, in_dim, rows, r0, r1;
    const float *x;
    float *y;
} kro_project_job;

static void *project_worker(void *arg) {
    kro_project_job *j = (kro_project_job *)arg;
    float *row = (float *)malloc(j->in_dim * sizeof(float));
    if (!row) return NULL;
    /* reference.rs:259-274: for each row, decode each weight row and dot it */
    for (size_t r = j->r0; r < j->r1; ++r)
        for (size_t o = 0; o < j->out_dim; ++o) {
            kro_embed(&j->w, o, row);
            j->y[r * j->out_dim + o] = dot_seq(row, j->x + r * j->in_dim, j->in_dim);
        }
    free(row);
    return NULL;
}

/* reference.rs:259-274 project (and :402-416 logits, one row): y[r, o] =
 * dot(decode_row(W, o), x[r]) with W of `kind` stored [out_dim, in_dim].
 * Rows split over `threads` host threads (each row is independent). */
void kro_project(int kind, const void *data, const float *scales, size_t out_dim, size_t in_dim,
                 const float *x, size_t rows, float *y, int threads) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > rows) threads = rows > 0 ? (int)rows : 1;
    kro_project_job jobs[64];
    pthread_t tid[64];
    if (threads > 64) threads = 64;
    for (int t = 0; t < threads; ++t) {
        kro_project_job *j = &jobs[t];
        j->w.kind = kind; j->w.vocab = out_dim; j->w.dim = in_dim; j->w.data = data; j->w.scales = scales;
        j->out_dim = out_dim; j->in_dim = in_dim; j->rows = rows; j->x = x; j->y = y;
        j->r0 = rows * (size_t)t / (size_t)threads;
        j->r1 = rows * (size_t)(t + 1) / (size_t)threads;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, project_worker, &jobs[t]);
    project_worker(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
}

/* reference.rs:151-159 kv_write: row i of k and v into slot slots[i] of
 * `layer` in caches laid out [layer][seq_len][kv_dim]. */
void kro_kv_write(float *key_cache, float *value_cache, size_t kv_dim, size_t seq_len, size_t layer,
                  const uint64_t *slots, size_t n_slots, const float *k, const float *v, size_t rows) {
    for (size_t row = 0; row < n_slots && row < rows; ++row) {
        size_t at = (layer * seq_len + (size_t)slots[row]) * kv_dim;
        memcpy(key_cache + at, k + row * kv_dim, kv_dim * sizeof(float));
        memcpy(value_cache + at, v + row * kv_dim, kv_dim * sizeof(float));
    }
}

/* One query row's window (src/backends/mod.rs:179-188): its own slots
 * att_start..=slot and the shared range [shared_start, shared_end). */
typedef struct {
    uint64_t att_start, slot, shared_start, shared_end;
} kro_window;

/* reference.rs:418-482 attention_rows for one query row. */
static void attention_row(const float *q, const float *key_cache, const float *value_cache, float *out,
                          float *att, size_t loff, const kro_window *w, size_t n_heads, size_t kv_mul,
                          size_t head_size, size_t kv_dim, size_t seq_len) {
    size_t n_shared = (size_t)(w->shared_end - w->shared_start);
    size_t count = n_shared + (size_t)(w->slot - w->att_start) + 1;
    float scale = 1.0f / sqrtf((float)head_size);
    for (size_t h = 0; h < n_heads; ++h) {
        const float *qh = q + h * head_size;
        float *scores = att + h * seq_len;
        size_t kv = (h / kv_mul) * head_size;
        size_t i = 0;
        for (uint64_t t = w->shared_start; t < w->shared_end; ++t, ++i)
            scores[i] = dot_seq(qh, key_cache + loff + (size_t)t * kv_dim + kv, head_size) * scale;
        for (uint64_t t = w->att_start; t <= w->slot; ++t, ++i)
            scores[n_shared + (size_t)(t - w->att_start)] =
                dot_seq(qh, key_cache + loff + (size_t)t * kv_dim + kv, head_size) * scale;
        float max = -INFINITY;
        for (size_t s = 0; s < count; ++s)
            if (scores[s] > max) max = scores[s];
        float sum = 0.0f;
        for (size_t s = 0; s < count; ++s) {
            scores[s] = expf(scores[s] - max);
            sum += scores[s];
        }
        for (size_t s = 0; s < count; ++s) scores[s] /= sum;
        float *o = out + h * head_size;
        for (size_t e = 0; e < head_size; ++e) o[e] = 0.0f;
        i = 0;
        for (uint64_t t = w->shared_start; t < w->shared_end; ++t, ++i) {
            const float *vv = value_cache + loff + (size_t)t * kv_dim + kv;
            float a = scores[i];
            for (size_t e = 0; e < head_size; ++e) o[e] += a * vv[e];
        }
        for (uint64_t t = w->att_start; t <= w->slot; ++t) {
            const float *vv = value_cache + loff + (size_t)t * kv_dim + kv;
            float a = scores[n_shared + (size_t)(t - w->att_start)];
            for (size_t e = 0; e < head_size; ++e) o[e] += a * vv[e];
        }
    }
}

/* reference.rs:276-306 attention: every window's row, scores at
 * att[row][head][seq_len], output [row][n_heads * head_size]. */
void kro_attention(const float *q, float *out, float *att, const float *key_cache, const float *value_cache,
                   size_t layer, const kro_window *windows, size_t n_windows, size_t n_heads, size_t kv_mul,
                   size_t head_size, size_t kv_dim, size_t seq_len) {
    size_t loff = layer * seq_len * kv_dim;
    size_t width = n_heads * head_size;
    for (size_t row = 0; row < n_windows; ++row)
        attention_row(q + row * width, key_cache, value_cache, out + row * width, att + row * n_heads * seq_len,
                      loff, &windows[row], n_heads, kv_mul, head_size, kv_dim, seq_len);
}
