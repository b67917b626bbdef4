// Launch interface between the host backend (backend.cu) and the sm_100a
// kernels (kernels.cu).  All pointers are device pointers; all launches are
// asynchronous on the given stream.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace krt {

// Bits of the device error word (checked by the host at every barrier).
enum : int { ERR_TOKEN = 1, ERR_POSITION = 2, ERR_TIMEOUT = 4 };

// Kernels this library has launched in this process, and the counter hook
// every launcher calls.
unsigned long long kernel_launches();
void count_launch();

// Storage kinds of an embedding table / source of the normalised row.
enum SrcKind : int { SRC_F32 = 0, SRC_BF16 = 1, SRC_Q8 = 2, SRC_X = 3 };

struct GatherArgs {
    const void *table;      // f32 / bf16 / int8 codes
    const float *tscales;   // q8_0 block scales
    int vocab, dim;
    const int32_t *tokens;  // [n]
    const int64_t *dst_off; // [n] element offsets into dst, or null: row r at r * dim
    float *dst;
    int n;
    int *err;
};
cudaError_t launch_embed_gather(int kind, bool vec, const GatherArgs &a, cudaStream_t s);

// The fused per-row-group kernel: every stage optional (null pointer = skip).
struct ChainArgs {
    int rows, dim, q_dim, kv_dim, hidden, head, half;
    float eps, final_eps;
    // source of the row being normalised
    const void *table; const float *tscales; int vocab; const int32_t *tokens; // SRC_F32/BF16/Q8
    const float *x_in;                                                          // SRC_X
    float *x_out;          // embed output, or x + resid
    float *xb; const float *w_att;
    float *q, *k; const float *w_q, *w_k;
    const int32_t *pos; const float *cos_t, *sin_t; int max_pos; int rope_mode; // 0 none 1 half 2 pair
    float *gate; const float *up;
    const float *resid;
    const float *w_final; int8_t *codes; float *scales; uint16_t *scales16;
    int *err;
    // The streams' work counter (one per stream that launches chains; zero
    // between launches), or null: the streams then split their work statically.
    unsigned *ticket;
    // Scratch of `rows` floats for the two-pass norm stage's row scales, or
    // null (the norm stage then runs as one pipeline).
    float *row_scale;
    // Tolerance mode, decode-sized norms (k_norm_small): the sum of squares
    // by a block reduction instead of one left-to-right chain.
    int tol;
};
// Optional callback around the kernels a chain launch issues: called with the
// stage about to launch, and with STAGE_END after the last one (the backend
// records CUDA events there when stage timing is on).
enum : int { STAGE_NORM = 0, STAGE_STREAM = 1, STAGE_FUSED = 2, STAGE_COUNT = 3, STAGE_END = -1 };
struct LaunchHook {
    void (*fn)(void *user, int stage);
    void *user;
};
// Chooses rows-per-CTA and shared memory, then launches.
// SM count of the current device (148 if it cannot be read).
int device_sms();
cudaError_t launch_chain(int src, const ChainArgs &a, cudaStream_t s, const LaunchHook *hook = nullptr);
// Shared memory a chain launch would need for one row group (to report limits).
size_t chain_smem_bytes(int src, const ChainArgs &a, int rows_per_cta);

cudaError_t launch_qk_norm(float *v, int rows, int width, int head, const float *w, float eps,
                           cudaStream_t s);
// x = x + resid, then xb = rms_norm(x) with weight w_att (a.x_in == a.x_out):
// the driver's add_in_place -> rms_norm pair in one pass.  dim % 8 == 0.
cudaError_t launch_add_rms_norm(const ChainArgs &a, cudaStream_t s);
// qk_norm(q), qk_norm(k) (either weight may be null), then rope(q, k).
cudaError_t launch_qk_rope(float *q, float *k, int q_width, int kv_width, int rows, int head, const float *wq,
                           const float *wk, float eps, const int32_t *pos, const float *cos_t, const float *sin_t,
                           int max_pos, int interleaved, int *err, cudaStream_t s);
// out[i*so + j] = a[i*sa + j] * b[i*sb + j] for i < count, j < len.
cudaError_t launch_mul_strided(float *out, const float *a, const float *b, long long so, long long sa, long long sb,
                               int len, int count, cudaStream_t s);
cudaError_t launch_rope(float *q, float *k, int q_width, int kv_width, int rows, int head,
                        const int32_t *pos, const float *cos_t, const float *sin_t, int max_pos,
                        int interleaved, int *err, cudaStream_t s);
// rope(q, k) and kv_write of k (rotated) and v into cache rows dst_rows (the
// layer's slots) in one launch; half-split RoPE, kv_width a whole number of
// heads and the cache's row width.
cudaError_t launch_rope_kv(float *q, float *k, int q_width, int kv_width, int rows, int head, const int32_t *pos,
                           const float *cos_t, const float *sin_t, int max_pos, int *err, const float *v, float *kc,
                           float *vc, const int32_t *dst_rows, cudaStream_t s);
cudaError_t launch_silu_mul(float *g, const float *u, size_t n, cudaStream_t s);
cudaError_t launch_add(float *d, const float *src, size_t n, cudaStream_t s);
cudaError_t launch_mul(float *o, const float *a, const float *b, size_t n, bool sequential,
                       cudaStream_t s);
cudaError_t launch_conv_prefill(float *out, const float *x, const float *w, int rows, int dim,
                                int k, cudaStream_t s);
cudaError_t launch_conv_decode(float *out, const float *x, const float *w, float *state, int dim,
                               int k, cudaStream_t s);
// The first `lead` (< k) of the `rows` rows of bcx are a shard's halo: they
// only feed the conv of the rows after them; cy gets rows - lead rows.  A null
// ring skips the ring update.
cudaError_t launch_lfm2_conv_block(const float *bcx, const float *w, float *ring, float *cy,
                                   int rows, int dim, int k, cudaStream_t s, int lead = 0);
cudaError_t launch_quantize_q8(const float *x, int rows, int dim, int8_t *codes, float *scales,
                               uint16_t *scales16, cudaStream_t s);
// Conversions for tables loaded from files (safetensors.rs / hf.rs): widen
// n bf16 (dtype 1) or f16 (dtype 2) patterns to f32; narrow f32 to bf16 by
// dropping the low half (hf.rs:182-188); widen f16 block scales the way
// Q8_0x4 reads them (quant.rs:764-769).
cudaError_t launch_widen_f32(int dtype, const uint16_t *src, float *dst, size_t n, cudaStream_t s);
// The bounded mbarrier wait run out on purpose (complete = 0) or satisfied
// (complete = 1), reporting through `err` like the pipelines' waits.
cudaError_t launch_wait_selftest(int *err, long long limit, int complete, cudaStream_t s);
cudaError_t launch_narrow_bf16(const float *src, uint16_t *dst, size_t n, cudaStream_t s);
cudaError_t launch_f16_scales_to_f32(const uint16_t *src, float *dst, size_t n, cudaStream_t s);
cudaError_t launch_q8x4_to_row_major(const uint8_t *blocks, int out_dim, int in_dim,
                                     int8_t *quants, float *scales, cudaStream_t s);


// ---- contractions (contract.cu) ----
// y[r, o] = dot(decode_row(W, o), x[r]) in the reference's order; W stored
// [out_dim, in_dim] as SRC_F32 / SRC_BF16 / SRC_Q8 (+ block scales).
cudaError_t launch_project(int src, const void *w, const float *wsc, int out_dim, int in_dim, const float *x,
                           int rows, float *y, int *err, cudaStream_t s);
// n (<= 3) projections of the same x and in_dim, one launch where the decode
// kernel takes them all (the trait's project_qkv / project_gate_up).
cudaError_t launch_project_set(int src, int n, const void *const *w, const float *const *wsc, const int *out_dim,
                               int in_dim, const float *x, int rows, float *const *y, int *err, cudaStream_t s);
// Tolerance-mode projections on the tensor cores (tc_project.cu): W bf16
// [out_dim, in_dim], in_dim % 8 == 0; x is first split into bf16 hi and lo
// halves ([rows, in_dim] each) by launch_split_bf16.
bool project_tc_supported(int out_dim, int in_dim, const void *w, const float *x, const float *y);
cudaError_t launch_split_bf16(const float *x, uint16_t *hi, uint16_t *lo, size_t n, cudaStream_t s);
cudaError_t launch_project_tc(const uint16_t *w, int out_dim, int in_dim, const uint16_t *hi, const uint16_t *lo,
                              int rows, float *y, int *err, cudaStream_t s);

// Tolerance mode, decode-sized calls: up to three bf16 matrices [out_dim[i],
// in_dim] over one x of 1..4 rows, y[i] = W[i] x, each output a warp-wide sum
// (not the reference's left-to-right order).  in_dim % 8 == 0, x and the
// matrices 16-byte aligned.
struct TolGemvSet {
    const uint16_t *w[3];
    float *y[3];
    int out_dim[3];
    int end[3];  // running totals of out_dim
    int n;
};
bool gemv_tol_supported(const void *w, const float *x, int in_dim, int rows);
cudaError_t launch_gemv_tol(int n, const uint16_t *const *w, const int *out_dim, int in_dim, const float *x, int rows,
                            float *const *y, cudaStream_t s);
// Row i of k and v into cache row dst_rows[i] of caches [rows_total, kv_dim].
cudaError_t launch_kv_write(float *kc, float *vc, int kv_dim, const int32_t *dst_rows, const float *k, const float *v,
                            int rows, cudaStream_t s);
// win: [n_rows][4] = att_start, slot, shared_start, shared_end; max_count the
// largest window; loff the layer's first cache element.
// raw: scratch of attention_scratch_floats() for the raw scores (null: the
// single-kernel form).
size_t attention_smem_bytes(int head_size, int max_count);
size_t attention_scratch_floats(int n_rows, int n_heads, int max_count);
// shared_map: every window maps window positions to the same cache slots (the
// same start and shared range; the rows of one sequence), so rows can share
// their key tiles.
cudaError_t launch_attention(const float *q, float *out, float *att, const float *kc, const float *vc,
                             const int32_t *win, int n_rows, int n_heads, int kv_mul, int head_size, int kv_dim,
                             int seq_len, size_t loff, int max_count, float *raw, bool shared_map, int *err,
                             cudaStream_t s);
// Tolerance mode: the window in chunks of 256 positions summed in parallel,
// then combined (not the reference's order).  part: scratch of
// attention_tol_scratch_floats() floats.
size_t attention_tol_scratch_floats(int n_rows, int n_heads, int head_size, int max_count);
cudaError_t launch_attention_tol(const float *q, float *out, float *att, const float *kc, const float *vc,
                                 const int32_t *win, int n_rows, int n_heads, int kv_mul, int head_size, int kv_dim,
                                 int seq_len, size_t loff, int max_count, float *part, cudaStream_t s);

}  // namespace krt
