/*
 * kernrt_cuda.h — C ABI of the B200 (sm_100a) `cuda` backend for KernRT's
 * per-row layer ops.
 *
 * The ABI mirrors KernRT's `Backend` trait (src/backends/mod.rs:264-404):
 * activations live in backend-owned device memory and cross the boundary as
 * opaque buffer handles (`kernrt_buf`, the trait's `Buf(usize)`,
 * mod.rs:40-42).  Work is enqueued on the backend's own CUDA stream and may be
 * deferred; `kernrt_cuda_read` is the barrier (mod.rs:8-15, 262-263, 280-282).
 *
 * Every function returns 0 on success and a nonzero KERNRT_E_* code on
 * failure; `kernrt_cuda_last_error()` then holds a message for the calling
 * thread.  The Rust side panics with that message, matching the reference's
 * panic-on-misuse convention (e.g. reference.rs:60-61 "buffers must be
 * distinct", reference.rs:135 "prepare() runs before compute").
 *
 * All sizes and offsets are in ELEMENTS of the buffer's element type (f32 for
 * buffers made by alloc/upload), exactly as in the trait.  Handles are only
 * valid for the context that made them.  A context is used by one host thread
 * at a time (the trait is Send, not Sync); it may migrate between threads.
 */
#ifndef KERNRT_CUDA_H
#define KERNRT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kernrt_cuda_ctx kernrt_cuda_ctx;
typedef uint64_t kernrt_buf;

enum {
    KERNRT_OK = 0,
    KERNRT_E_NO_DEVICE = 1,   /* no CUDA device / driver: BackendError.detail (mod.rs:192-213) */
    KERNRT_E_INVALID = 2,     /* bad handle, size, offset or aliasing: the reference panics */
    KERNRT_E_CUDA = 3,        /* a CUDA runtime call failed */
    KERNRT_E_DEVICE = 4,      /* a kernel reported a bad input (token / position out of range) */
    KERNRT_E_STATE = 5        /* call out of order (e.g. embed before prepare) */
};

/* Storage kinds of the token embedding, as Matrix::kind names them
 * (src/ops/quant.rs:565-572). */
enum { KERNRT_F32 = 0, KERNRT_BF16 = 1, KERNRT_Q8_0 = 2, KERNRT_Q8_0X4 = 3 };

/* Message for the last failing call on this thread ("" if none). */
const char *kernrt_cuda_last_error(void);

/* Kernels this library has launched in this process, over all contexts and
 * devices (for profiling and for checking what a timed region ran). */
int kernrt_cuda_kernel_launches(uint64_t *count);

/* Number of visible CUDA devices (0 when there is no driver or device). */
int kernrt_cuda_device_count(int *count);

/* Backend construction: replaces `Metal::new` in `backends::open`
 * (src/backends/mod.rs:228-244).  Fails with KERNRT_E_NO_DEVICE and the message
 * "no CUDA device" when none is present (the detail tests/backends.rs:335-348
 * checks for the Metal backend).  `device` < 0 selects KERNRT_CUDA_DEVICE or 0. */
int kernrt_cuda_create(int device, kernrt_cuda_ctx **out);
int kernrt_cuda_destroy(kernrt_cuda_ctx *ctx);

/* Backend::name (mod.rs:266) -> "cuda"; Backend::storage (mod.rs:269). */
const char *kernrt_cuda_name(const kernrt_cuda_ctx *ctx);
const char *kernrt_cuda_storage(const kernrt_cuda_ctx *ctx);

/* The device's CUDA stream (a cudaStream_t), for callers that time or order
 * work against it. */
int kernrt_cuda_stream(kernrt_cuda_ctx *ctx, void **stream);

/* --- Backend::prepare (mod.rs:272): upload the token embedding once. --------
 * The table is `[vocab, dim]` in the storage it was loaded at
 * (ModelWeights.token_embedding, mod.rs:131-145):
 *   f32   : float   [vocab*dim]
 *   bf16  : uint16  [vocab*dim]  (bf16 bit patterns)
 *   q8_0  : int8    [vocab*dim] + float scales [vocab*dim/32]  (quant.rs:509-515)
 *   q8_0x4: the 136-byte four-row blocks of Q8_0x4 (quant.rs:102-117),
 *           de-interleaved on the device to row-major Q8_0 (quant.rs:198-220). */
int kernrt_cuda_prepare_embedding(kernrt_cuda_ctx *ctx, int kind, const void *data,
                                  const float *scales, size_t vocab, size_t dim);

/* Self-test of the bounded waits (no counterpart in the reference: its CPU
 * backend has no device pipelines).  Every spin-wait in these kernels gives
 * up after a cycle limit, sets the device error word and returns, so a stuck
 * pipeline surfaces as KERNRT_E_DEVICE ("... timed out") at the next barrier
 * instead of hanging the GPU.  This runs that wait alone on an mbarrier phase
 * that nothing completes (complete = 0) for at most `cycles` SM cycles
 * (<= 2^31), or on one it completes first (complete = 1); the first returns
 * KERNRT_E_DEVICE and leaves the context usable, the second returns 0. */
int kernrt_cuda_selftest_wait(kernrt_cuda_ctx *ctx, uint64_t cycles, int complete);

/* --- Weights from a safetensors file (src/formats/safetensors.rs) ----------
 * A tensor's entry in a safetensors file, read and checked on the host only
 * (no device): the header is validated as read_with does
 * (safetensors.rs:161-257: header length, strict JSON, every entry's dtype,
 * shape and byte range), and the message of a failure is the reference's
 * SafeTensorsError text (safetensors.rs:46-68) in kernrt_cuda_last_error. */
enum { KERNRT_ST_F32 = 0, KERNRT_ST_BF16 = 1, KERNRT_ST_F16 = 2 };
typedef struct {
    int dtype;             /* KERNRT_ST_* */
    int rank;
    uint64_t shape[8];     /* the first min(rank, 8) dimensions */
    uint64_t file_offset;  /* byte offset of the payload in the file */
    uint64_t bytes;        /* payload bytes */
} kernrt_st_tensor;
int kernrt_cuda_safetensors_tensor(const char *path, const char *name, kernrt_st_tensor *out);

/* Backend::prepare's token embedding taken from a file, as the HF loaders take
 * "model.embed_tokens.weight" (take_matrix_raw, hf.rs:141-147, llama.rs:281,
 * lfm2.rs:174): the payload goes from the file to the device as stored and is
 * converted there by matrix_from_raw's rules (hf.rs:151-191) for `storage`
 * (KERNRT_F32 / _BF16 / _Q8_0 / _Q8_0X4): a bf16 payload is handed over as it
 * is for bf16 storage, and no f32 copy of it is made on the host.  The rank-2
 * tensor becomes the `[vocab, dim]` table kernrt_cuda_prepare_embedding would
 * install; kernrt_cuda_storage then names the storage the rules produced. */
int kernrt_cuda_prepare_embedding_file(kernrt_cuda_ctx *ctx, const char *path, const char *name, int storage);

/* --- buffers: Backend::alloc / upload / read (mod.rs:275-282) --------------- */
/* `len` f32 elements.  Zero-filled (the trait says uninitialised; zeroing is
 * what the LFM2 ring seeding relies on, lfm2.rs:311-318). */
int kernrt_cuda_alloc(kernrt_cuda_ctx *ctx, size_t len, kernrt_buf *out);
int kernrt_cuda_upload(kernrt_cuda_ctx *ctx, const float *data, size_t len, kernrt_buf *out);
/* Completes all deferred work, then copies `len` elements of `src` to the host. */
int kernrt_cuda_read(kernrt_cuda_ctx *ctx, kernrt_buf src, float *out, size_t len);
/* Extensions beyond the trait, for typed outputs (int8 codes, u16 scales, i32
 * ids): raw byte buffers, and a host->device write into an existing buffer. */
int kernrt_cuda_alloc_bytes(kernrt_cuda_ctx *ctx, size_t bytes, kernrt_buf *out);
int kernrt_cuda_write_bytes(kernrt_cuda_ctx *ctx, kernrt_buf dst, size_t dst_byte_off,
                            const void *src, size_t bytes);
int kernrt_cuda_read_bytes(kernrt_cuda_ctx *ctx, kernrt_buf src, size_t src_byte_off, void *dst,
                           size_t bytes);
/* Device address of a buffer (valid until destroy), for zero-copy interop. */
int kernrt_cuda_device_ptr(kernrt_cuda_ctx *ctx, kernrt_buf buf, void **ptr);
/* Wait for all deferred work. */
int kernrt_cuda_synchronize(kernrt_cuda_ctx *ctx);
/* Launch every deferred op (pending embeds, an op held for fusion) onto the
 * backend's stream without waiting for it. */
int kernrt_cuda_flush(kernrt_cuda_ctx *ctx);

/* --- the row ops ------------------------------------------------------------ */

/* Backend::embed (mod.rs:285): decode_row(token) into out[offset..offset+dim]
 * (reference.rs:133-140, quant.rs:659-693).  Deferred: consecutive calls are
 * coalesced into one gather launch at the next other op or read. */
int kernrt_cuda_embed(kernrt_cuda_ctx *ctx, size_t token, kernrt_buf out, size_t offset);

/* Backend::copy (mod.rs:288; reference.rs:142-149): memmove semantics within
 * one buffer. */
int kernrt_cuda_copy(kernrt_cuda_ctx *ctx, kernrt_buf src, size_t src_offset, kernrt_buf dst,
                     size_t dst_offset, size_t len);

/* Backend::rms_norm (mod.rs:290-291; reference.rs:161-178).  out != x. */
int kernrt_cuda_rms_norm(kernrt_cuda_ctx *ctx, kernrt_buf out, kernrt_buf x, kernrt_buf weight,
                         size_t rows, size_t dim, float eps);

/* Backend::qk_norm (mod.rs:294-302; reference.rs:180-207): per-head RMSNorm in
 * place over width/head_size full heads of each row. */
int kernrt_cuda_qk_norm(kernrt_cuda_ctx *ctx, kernrt_buf v, size_t rows, size_t width,
                        size_t head_size, kernrt_buf weight, float eps);

/* Backend::rope (mod.rs:306-315; reference.rs:209-257) with RopeSpec
 * (mod.rs:149-155) flattened: positions[i] (host, usize) for row i; like the
 * reference's `positions.iter().take(rows)`, min(rows, n_positions) rows are
 * rotated.  q != k.  head_size must be even. */
int kernrt_cuda_rope(kernrt_cuda_ctx *ctx, kernrt_buf q, kernrt_buf k, size_t q_width,
                     size_t kv_width, size_t rows, const uint64_t *positions,
                     size_t n_positions, size_t head_size, float theta, int interleaved);

/* Backend::add_in_place (mod.rs:361-362; reference.rs:308-313).  dst != src. */
int kernrt_cuda_add_in_place(kernrt_cuda_ctx *ctx, kernrt_buf dst, kernrt_buf src, size_t len);

/* Backend::mul (mod.rs:370-379; reference.rs:315-363): any aliasing allowed,
 * with the reference's in-order semantics. */
int kernrt_cuda_mul(kernrt_cuda_ctx *ctx, kernrt_buf out, size_t out_off, kernrt_buf a,
                    size_t a_off, kernrt_buf b, size_t b_off, size_t len);

/* Backend::conv_prefill (mod.rs:388; reference.rs:365-370, 490-503). */
int kernrt_cuda_conv_prefill(kernrt_cuda_ctx *ctx, kernrt_buf out, kernrt_buf x,
                             kernrt_buf kernel, size_t rows, size_t dim, size_t k);

/* Backend::conv_decode (mod.rs:397; reference.rs:372-393).  out may alias x. */
int kernrt_cuda_conv_decode(kernrt_cuda_ctx *ctx, kernrt_buf out, kernrt_buf x, kernrt_buf kernel,
                            kernrt_buf state, size_t dim, size_t k);

/* Backend::silu_mul (mod.rs:399-400; reference.rs:395-400).  gate != up. */
int kernrt_cuda_silu_mul(kernrt_cuda_ctx *ctx, kernrt_buf gate, kernrt_buf up, size_t len);

/* --- Q8_0 activation quantisation (beyond the trait) -------------------------
 * Q8Vec::quantize_into (src/ops/quant.rs:856-874) of each of `rows` rows of x:
 * codes int8 [rows, ceil(dim/32)*32] (tail zero padded), scales f32
 * [rows, ceil(dim/32)], scales_f16 u16 (same shape; 0 handle = skip).  The
 * code/scale buffers are byte buffers (kernrt_cuda_alloc_bytes). */
int kernrt_cuda_quantize_q8_0(kernrt_cuda_ctx *ctx, kernrt_buf x, size_t rows, size_t dim,
                              kernrt_buf codes, kernrt_buf scales, kernrt_buf scales_f16);

/* rms_norm fused with the quantisation that follows it on the CPU path
 * (cpu.rs:143-158, 361-369, 501-514 after llama.rs:740/765/858): the normalised
 * row never goes to HBM. */
int kernrt_cuda_rms_norm_q8_0(kernrt_cuda_ctx *ctx, kernrt_buf x, kernrt_buf weight, size_t rows,
                              size_t dim, float eps, kernrt_buf codes, kernrt_buf scales,
                              kernrt_buf scales_f16);

/* --- the fused layer-op chain ------------------------------------------------
 * One launch runs a Llama-family block's row ops for `rows` token rows in the
 * driver's order (llama.rs:734-770; row ops only, contractions elided):
 *   x = embed(tokens) (if tokens) | x (input);  xb = rms_norm(x, w_att);
 *   q,k = qk_norm (if w_q/w_k);  q,k = rope(positions);  gate = silu(gate)*up;
 *   x = x + resid (if resid);  codes/scales = Q8_0(rms_norm(x, w_final)) (if w_final).
 * Any stage whose buffer handle is 0 is skipped.  `tokens` and `positions`
 * are int32 byte buffers already on the device; tokens index the prepared
 * embedding.  The RoPE table must cover positions < rope_max_pos (see
 * kernrt_cuda_rope_prepare). */
typedef struct {
    size_t rows, dim, q_dim, kv_dim, hidden, head_size;
    float eps, theta, final_eps;
    int interleaved;
    kernrt_buf tokens;    /* int32 [rows] or 0 (then x is the input) */
    kernrt_buf positions; /* int32 [rows] */
    kernrt_buf x;         /* f32 [rows, dim]: output (embed) or input; x + resid written back */
    kernrt_buf xb;        /* f32 [rows, dim] out, or 0 */
    kernrt_buf w_att;     /* f32 [dim] */
    kernrt_buf q, k;      /* f32 [rows, q_dim], [rows, kv_dim] in place, or 0 */
    kernrt_buf w_q, w_k;  /* f32 [head_size] or 0 */
    kernrt_buf gate, up;  /* f32 [rows, hidden], or 0 */
    kernrt_buf resid;     /* f32 [rows, dim], or 0 */
    kernrt_buf w_final;   /* f32 [dim], or 0 */
    kernrt_buf codes, scales, scales_f16; /* Q8_0 outputs when w_final */
} kernrt_chain_args;

/* Build (or grow) the RoPE cos/sin table for (theta, head_size) to cover
 * positions [0, max_pos).  Row ops build it on demand; the chain needs it
 * prepared because its positions are already on the device. */
int kernrt_cuda_rope_prepare(kernrt_cuda_ctx *ctx, float theta, size_t head_size, size_t max_pos);

int kernrt_cuda_layer_chain(kernrt_cuda_ctx *ctx, const kernrt_chain_args *args);

/* The same chain on HOST buffers, for callers whose rows live in host memory:
 * the rows are processed in chunks of `chunk_rows` (0 = chosen by the
 * backend), each chunk's inputs copied to the device, run through the chain,
 * and its outputs copied back, with the copies in both directions and the
 * kernels of neighbouring chunks overlapping on three streams.  Returns when
 * every output is in host memory.  Page-locked host buffers give the overlap;
 * pageable ones still work, with the copies serialised.  Any input/output
 * pointer may be NULL to skip that stage (as a 0 handle does in
 * kernrt_chain_args); an output may alias its input (q_out == q_in, ...).
 * Token ids and positions are checked on the host; the RoPE table is built
 * or grown as needed.  Weights are device buffers (handles). */
typedef struct {
    size_t rows, dim, q_dim, kv_dim, hidden, head_size;
    float eps, theta, final_eps;
    int interleaved;
    size_t chunk_rows;
    const int32_t *tokens;     /* [rows], or NULL: then x_in is the input */
    const int32_t *positions;  /* [rows] */
    const float *x_in;         /* [rows, dim] when tokens == NULL */
    const float *q_in, *k_in;  /* [rows, q_dim], [rows, kv_dim] */
    const float *gate_in, *up; /* [rows, hidden] */
    const float *resid;        /* [rows, dim] */
    float *x_out, *xb_out;     /* [rows, dim] */
    float *q_out, *k_out;      /* [rows, q_dim], [rows, kv_dim] */
    float *gate_out;           /* [rows, hidden] */
    int8_t *codes;             /* [rows, ceil(dim/32)*32] when w_final */
    float *scales;             /* [rows, ceil(dim/32)] when w_final */
    uint16_t *scales_f16;      /* [rows, ceil(dim/32)] or NULL */
    kernrt_buf w_att, w_q, w_k, w_final;
} kernrt_chain_host_args;

int kernrt_cuda_layer_chain_host(kernrt_cuda_ctx *ctx, const kernrt_chain_host_args *args);

/* Stage timing (off by default): while enabled, every chain launch
 * (kernrt_cuda_rms_norm, _rms_norm_q8_0, _layer_chain) records a CUDA event
 * around each kernel it issues.  kernrt_cuda_stage_times completes pending
 * work and returns, per stage, the device milliseconds and launch count since
 * timing was enabled: [0] the norm stage (k_norm_rows for gathered rows,
 * k_norm_cols for f32 rows, k_norm_small for a few f32 rows, k_norm_pipe for
 * widths the bulk copies cannot take), [1] the RoPE/SwiGLU stream (k_stream), [2] the single
 * fused kernel (k_chain).  Enabling clears the record. */
int kernrt_cuda_stage_timing(kernrt_cuda_ctx *ctx, int enable);
int kernrt_cuda_stage_times(kernrt_cuda_ctx *ctx, double ms[3], uint64_t launches[3]);

/* The LFM2 short-conv block's row ops in one launch (lfm2.rs:584-624):
 * h = B*x; co = conv_prefill(h); ring <- last min(rows,k-1) rows of h;
 * cy = C*co, with bcx = [B | C | x] thirds per row (lfm2.rs:9-15). */
int kernrt_cuda_lfm2_conv_block(kernrt_cuda_ctx *ctx, kernrt_buf bcx, kernrt_buf kernel,
                                kernrt_buf ring, kernrt_buf cy, size_t rows, size_t dim, size_t k);

/* The same block for one shard of a sequence split across devices (no
 * counterpart in the reference: KernRT runs one device).  bcx holds `halo`
 * (< k) rows before the shard, staged by the caller from the preceding shard's
 * rows, then the shard's `rows` rows; the halo rows feed the conv of the
 * shard's first rows exactly as in the unsharded sequence and give no output,
 * so cy (`rows` rows) equals the unsharded block's rows of the shard bit for
 * bit.  halo = 0 is the sequence's first shard (zero padding, as
 * kernrt_cuda_lfm2_conv_block).  ring = 0 skips the ring update (a shard that
 * does not end the sequence); the last shard passes the ring, and then needs at
 * least k - 1 rows when halo > 0. */
int kernrt_cuda_lfm2_conv_block_halo(kernrt_cuda_ctx *ctx, kernrt_buf bcx, kernrt_buf kernel, kernrt_buf ring,
                                     kernrt_buf cy, size_t rows, size_t dim, size_t k, size_t halo);

/* --- Contractions: Backend::project / logits / kv_write / attention ----------
 * The reference backend's arithmetic order (reference.rs:73-79 dot, one f32
 * accumulator left to right, multiply then add): projections, logits and the
 * cache write are bit-identical to it; attention differs only through expf. */

/* A weight matrix prepared once (the weights Backend::prepare receives,
 * mod.rs:268-273): handle = index + 1. */
typedef uint64_t kernrt_mat;

/* Uploads W [out_dim, in_dim] in its stored format (kinds and layouts as for
 * kernrt_cuda_prepare_embedding; Matrix, quant.rs:502-520). */
int kernrt_cuda_prepare_matrix(kernrt_cuda_ctx *ctx, int kind, const void *data, const float *scales,
                               size_t out_dim, size_t in_dim, kernrt_mat *out);

/* Exact or tolerance mode of the projections (no counterpart in the
 * reference: its backends each have one arithmetic).  exact = 1 (the default)
 * keeps every projection in the reference's order, bit-identical to it.
 * exact = 0 runs bf16 projections of at least 16 rows (prefill) on the tensor
 * cores: x is split into bf16 hi + lo halves and both are multiplied by W
 * (tcgen05.mma, f32 accumulation), which keeps ~16 bits of each activation's
 * mantissa; results differ from the reference's sequential dot by the
 * reordered f32 sum (the bar tests/backends.rs:129-148 sets for a non-oracle
 * backend is 1e-3 on a model's logits).  bf16 projections of 1 to 4 rows
 * (decode, the classifier) sum each output across a warp instead of in one
 * chain, attention over at most 4 windows sums each window in chunks of 64
 * positions combined by their maxima, and rms_norm of at most 4 rows sums its
 * squares by a block reduction.  Larger calls and other storages stay exact.  KERNRT_CUDA_EXACT=0 in
 * the environment sets exact = 0 at kernrt_cuda_create. */
int kernrt_cuda_set_exact(kernrt_cuda_ctx *ctx, int exact);

/* Backend::project (mod.rs:318; reference.rs:259-274): y[r, o] =
 * dot(decode_row(W, o), x[r]) for rows r; x [rows, in_dim], y [rows, out_dim].
 * The trait's project_qkv / project_gate_up defaults (mod.rs:326-337) are
 * three / two of these calls. */
int kernrt_cuda_project(kernrt_cuda_ctx *ctx, kernrt_mat w, kernrt_buf x, kernrt_buf y, size_t rows);

/* Backend::project_qkv / project_gate_up (mod.rs:320-337): the same
 * projections of one x as three / two kernrt_cuda_project calls, in one
 * launch where the matrices share storage and in_dim (the override the
 * trait's comment invites: decode projections run side by side). */
int kernrt_cuda_project_qkv(kernrt_cuda_ctx *ctx, kernrt_mat wq, kernrt_mat wk, kernrt_mat wv, kernrt_buf x,
                            kernrt_buf q, kernrt_buf k, kernrt_buf v, size_t rows);
int kernrt_cuda_project_gate_up(kernrt_cuda_ctx *ctx, kernrt_mat wg, kernrt_mat wu, kernrt_buf x,
                                kernrt_buf gate, kernrt_buf up, size_t rows);

/* Backend::logits (mod.rs:403; reference.rs:402-416): the classifier W over
 * row 0 of x. */
int kernrt_cuda_logits(kernrt_cuda_ctx *ctx, kernrt_mat w, kernrt_buf x, kernrt_buf y);

/* The key/value caches of a KvSpec (mod.rs:169-177), [n_layers][seq_len]
 * [kv_dim] f32 each, zero-filled; Backend::prepare's cache half. */
int kernrt_cuda_kv_prepare(kernrt_cuda_ctx *ctx, size_t n_layers, size_t kv_dim, size_t seq_len);

/* Backend::kv_write (mod.rs:344; reference.rs:151-159): rows
 * min(rows, n_slots) of k and v [rows, kv_dim] into slots[i] of `layer`. */
int kernrt_cuda_kv_write(kernrt_cuda_ctx *ctx, size_t layer, const uint64_t *slots, size_t n_slots,
                         kernrt_buf k, kernrt_buf v, size_t rows);

/* One query row's causal window (Window, mod.rs:179-188): its own slots
 * att_start..=slot and the extra range [shared_start, shared_end). */
typedef struct {
    uint64_t att_start, slot, shared_start, shared_end;
} kernrt_window;

/* Backend::attention (mod.rs:351-359; reference.rs:276-306, 418-482) with
 * AttnSpec {n_heads, kv_mul, head_size, kv_dim, seq_len} (mod.rs:158-167):
 * q and out [n_windows, n_heads * head_size], att [n_windows, n_heads,
 * seq_len] (each head's first `count` scores are written). */
int kernrt_cuda_attention(kernrt_cuda_ctx *ctx, kernrt_buf q, kernrt_buf out, kernrt_buf att, size_t layer,
                          const kernrt_window *windows, size_t n_windows, size_t n_heads, size_t kv_mul,
                          size_t head_size, size_t kv_dim, size_t seq_len);

/* --- Embedding gather without allocation --------------------------------------
 * No counterpart in the reference: KernRT's backends allocate their own memory.
 * Some callers of this library cannot let it allocate device memory: a host
 * runtime that owns all of HBM through its own pre-reserved pool, or a serving
 * loop that must not hit the device-wide synchronisation cudaMalloc and
 * cudaFree can cause.  This entry point needs no context and calls no
 * allocator: it gathers rows `tokens[0..n)` (host int32 ids < vocab) of a
 * device-resident table into the caller's device rows `out[r*dim ..]`, on
 * `stream` (a cudaStream_t; NULL = the legacy default stream) of `device`.
 * The table is f32, bf16 or row-major Q8_0 (codes + f32 block scales), laid
 * out as for kernrt_cuda_prepare_embedding; results equal kernrt_cuda_embed's.
 *
 * The token ids go to a fixed scratch array compiled into the library:
 * KERNRT_NOALLOC_MAX_ROWS int32 ids (256 KiB), held on every GPU that loads
 * the library until the process exits.  Larger n is rejected with
 * KERNRT_E_INVALID; split the call.  All calls on a device share the array,
 * so calls that may overlap on the GPU (other streams, other threads) race
 * on the ids and must be ordered by the caller; a lost race gathers wrong
 * table rows but writes only inside each call's own `out`.  The first call
 * on each device does a one-time set-up: it looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture begins.  The ids are copied from host
 * memory with cudaMemcpyAsync on `stream`: pageable ids are read during the
 * call, page-locked ids must stay unchanged until the stream has passed this
 * call.  The caller's current device is unchanged on return. */
#define KERNRT_NOALLOC_MAX_ROWS 65536
int kernrt_cuda_embed_rows_noalloc(int device, int kind, const void *table, const float *scales,
                                   size_t vocab, size_t dim, const int32_t *tokens, size_t n,
                                   float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KERNRT_CUDA_H */
