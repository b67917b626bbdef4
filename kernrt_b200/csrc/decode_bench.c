/*
 * decode_bench: one decode step of configs[1] (SmolLM2-1.7B, one token at
 * position 511) through the C ABI, as a Rust caller of the `cuda` backend
 * issues it, with no Python in the loop: the row ops of a block in the
 * driver's order (llama.rs decode: embed, rms_norm, rope, add, rms_norm,
 * silu_mul, add; the contractions elided, their outputs fixed buffers) and one
 * read() per step, the timing convention of examples/decode_rate.rs:61-75.
 *
 *     kernrt_decode_bench [steps=300]
 *     kernrt_decode_bench model [layers=24] [tokens=50]
 *
 * The second form times whole decode tokens of SmolLM2-1.7B (bf16 matrices,
 * random; the KV cache filled to position 511): per layer rms_norm,
 * project_qkv, rope, kv_write, attention, project (o), add_in_place, rms_norm,
 * project_gate_up, silu_mul, project (down), add_in_place, then the final
 * rms_norm, logits and one read() (llama.rs decode order), once in exact mode
 * and once in tolerance mode (kernrt_cuda_set_exact(ctx, 0)); one JSON line
 * each.
 *
 * Prints one JSON line per mode (exact, then tolerance: kernrt_cuda_set_exact
 * (ctx, 0), the step's RMSNorms by block reduction): per step the host wall
 * time (issue + read barrier),
 * p10 and median; the host time to issue the ops before the barrier; the
 * device span from the step's first launch to its last (CUDA events on the
 * backend's stream); and the kernels launched per step.
 */
#include "../../include/kernrt_cuda.h"

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

enum { VOCAB = 49152, DIM = 2048, QD = 2048, KVD = 2048, HIDDEN = 8192, HEAD = 64, WARM = 20 };

static double now_us(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec * 1e6 + t.tv_nsec * 1e-3;
}

static void ok(int rc, const char *what) {
    if (rc != KERNRT_OK) {
        fprintf(stderr, "%s: %s\n", what, kernrt_cuda_last_error());
        exit(1);
    }
}

static void cuda_ok(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
        exit(1);
    }
}

/* tests/backends.rs:41-51's LCG, uniform in [-0.5, 0.5). */
static uint64_t lcg = 0x2545F4914F6CDD1Dull;
static float uniform(void) {
    lcg = lcg * 6364136223846793005ull + 1442695040888963407ull;
    return (float)(lcg >> 40) / (float)(1u << 24) - 0.5f;
}

static kernrt_buf random_buf(kernrt_cuda_ctx *ctx, size_t n) {
    float *h = malloc(n * sizeof(float));
    for (size_t i = 0; i < n; ++i) h[i] = uniform();
    kernrt_buf b = 0;
    ok(kernrt_cuda_upload(ctx, h, n, &b), "upload");
    free(h);
    return b;
}

static int cmp(const void *a, const void *b) {
    const double x = *(const double *)a, y = *(const double *)b;
    return x < y ? -1 : x > y;
}

/* Whole decode tokens through the C ABI (the second form above). */
static int model_decode(int n_layers, int tokens) {
    enum { Q = 2048, KV = 2048, SEQ = 4096, HEADS = 32, POS = 511 };
    kernrt_cuda_ctx *ctx = NULL;
    ok(kernrt_cuda_create(0, &ctx), "create");
    /* one host matrix per shape, uploaded into every layer's own device copy */
    uint16_t *h = malloc((size_t)VOCAB * DIM * sizeof(uint16_t));
    for (size_t i = 0; i < (size_t)VOCAB * DIM; ++i) {
        const float v = 0.04f * uniform();
        uint32_t bits;
        memcpy(&bits, &v, 4);
        h[i] = (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
    }
    ok(kernrt_cuda_prepare_embedding(ctx, KERNRT_BF16, h, NULL, VOCAB, DIM), "prepare");
    kernrt_mat cls;
    ok(kernrt_cuda_prepare_matrix(ctx, KERNRT_BF16, h, NULL, VOCAB, DIM, &cls), "classifier");
    kernrt_mat *m = malloc((size_t)n_layers * 7 * sizeof(kernrt_mat));
    const size_t shape[7][2] = {{Q, DIM}, {KV, DIM}, {KV, DIM}, {DIM, Q}, {HIDDEN, DIM}, {HIDDEN, DIM}, {DIM, HIDDEN}};
    for (int l = 0; l < n_layers; ++l)
        for (int j = 0; j < 7; ++j)  /* the table's first rows stand in for the weights */
            ok(kernrt_cuda_prepare_matrix(ctx, KERNRT_BF16, h, NULL, shape[j][0], shape[j][1], &m[7 * l + j]),
               "matrix");
    free(h);
    ok(kernrt_cuda_kv_prepare(ctx, (size_t)n_layers, KV, SEQ), "kv_prepare");
    kernrt_buf x, xb, q, k, v, ao, o, g, u, dn, att, lg, kf, vf;
    ok(kernrt_cuda_alloc(ctx, DIM, &x), "alloc");
    ok(kernrt_cuda_alloc(ctx, DIM, &xb), "alloc");
    ok(kernrt_cuda_alloc(ctx, Q, &q), "alloc");
    ok(kernrt_cuda_alloc(ctx, KV, &k), "alloc");
    ok(kernrt_cuda_alloc(ctx, KV, &v), "alloc");
    ok(kernrt_cuda_alloc(ctx, Q, &ao), "alloc");
    ok(kernrt_cuda_alloc(ctx, DIM, &o), "alloc");
    ok(kernrt_cuda_alloc(ctx, HIDDEN, &g), "alloc");
    ok(kernrt_cuda_alloc(ctx, HIDDEN, &u), "alloc");
    ok(kernrt_cuda_alloc(ctx, DIM, &dn), "alloc");
    ok(kernrt_cuda_alloc(ctx, (size_t)HEADS * SEQ, &att), "alloc");
    ok(kernrt_cuda_alloc(ctx, VOCAB, &lg), "alloc");
    kf = random_buf(ctx, (size_t)POS * KV);
    vf = random_buf(ctx, (size_t)POS * KV);
    uint64_t *slots = malloc(POS * sizeof(uint64_t));
    for (int i = 0; i < POS; ++i) slots[i] = (uint64_t)i;
    for (int l = 0; l < n_layers; ++l) ok(kernrt_cuda_kv_write(ctx, (size_t)l, slots, POS, kf, vf, POS), "kv_write");
    free(slots);
    float *ones = malloc(DIM * sizeof(float));
    for (int i = 0; i < DIM; ++i) ones[i] = 1.0f;
    kernrt_buf w;
    ok(kernrt_cuda_upload(ctx, ones, DIM, &w), "upload");
    free(ones);
    void *stream_ptr = NULL;
    ok(kernrt_cuda_stream(ctx, &stream_ptr), "stream");
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    cudaEvent_t ev0, ev1;
    cuda_ok(cudaEventCreate(&ev0), "event");
    cuda_ok(cudaEventCreate(&ev1), "event");
    const uint64_t pos = POS, slot = POS;
    const kernrt_window win = {0, POS, 0, 0};
    const float eps = 1e-5f, theta = 1.3e5f;
    float *out = malloc(VOCAB * sizeof(float));
    double *wall = malloc(tokens * sizeof(double)), *span = malloc(tokens * sizeof(double));
    for (int exact = 1; exact >= 0; --exact) {
        ok(kernrt_cuda_set_exact(ctx, exact), "set_exact");
        uint64_t l0 = 0, l1 = 0;
        for (int t = -3; t < tokens; ++t) {
            if (t == 0) ok(kernrt_cuda_kernel_launches(&l0), "launches");
            const double t0 = now_us();
            cuda_ok(cudaEventRecord(ev0, stream), "record");
            ok(kernrt_cuda_embed(ctx, 7, x, 0), "embed");
            for (int l = 0; l < n_layers; ++l) {
                const kernrt_mat *L = m + 7 * l;
                ok(kernrt_cuda_rms_norm(ctx, xb, x, w, 1, DIM, eps), "rms_norm");
                ok(kernrt_cuda_project_qkv(ctx, L[0], L[1], L[2], xb, q, k, v, 1), "project_qkv");
                ok(kernrt_cuda_rope(ctx, q, k, Q, KV, 1, &pos, 1, HEAD, theta, 0), "rope");
                ok(kernrt_cuda_kv_write(ctx, (size_t)l, &slot, 1, k, v, 1), "kv_write");
                ok(kernrt_cuda_attention(ctx, q, ao, att, (size_t)l, &win, 1, HEADS, 1, HEAD, KV, SEQ), "attention");
                ok(kernrt_cuda_project(ctx, L[3], ao, o, 1), "project o");
                ok(kernrt_cuda_add_in_place(ctx, x, o, DIM), "add");
                ok(kernrt_cuda_rms_norm(ctx, xb, x, w, 1, DIM, eps), "rms_norm");
                ok(kernrt_cuda_project_gate_up(ctx, L[4], L[5], xb, g, u, 1), "project_gate_up");
                ok(kernrt_cuda_silu_mul(ctx, g, u, HIDDEN), "silu_mul");
                ok(kernrt_cuda_project(ctx, L[6], g, dn, 1), "project down");
                ok(kernrt_cuda_add_in_place(ctx, x, dn, DIM), "add");
            }
            ok(kernrt_cuda_rms_norm(ctx, xb, x, w, 1, DIM, eps), "rms_norm");
            ok(kernrt_cuda_logits(ctx, cls, xb, lg), "logits");
            ok(kernrt_cuda_flush(ctx), "flush");
            cuda_ok(cudaEventRecord(ev1, stream), "record");
            ok(kernrt_cuda_read(ctx, lg, out, VOCAB), "read");
            const double t1 = now_us();
            if (t >= 0) {
                float ms = 0.0f;
                cuda_ok(cudaEventElapsedTime(&ms, ev0, ev1), "elapsed");
                wall[t] = t1 - t0;
                span[t] = ms * 1e3;
            }
        }
        ok(kernrt_cuda_kernel_launches(&l1), "launches");
        qsort(wall, tokens, sizeof(double), cmp);
        qsort(span, tokens, sizeof(double), cmp);
        printf("{\"name\": \"decode token, SmolLM2-1.7B (%d layers, bf16, pos %d), C ABI, %s\", \"tokens\": %d, "
               "\"wall_us_p10\": %.1f, \"wall_us_median\": %.1f, \"tokens_per_s\": %.1f, "
               "\"device_span_us_median\": %.1f, \"launches_per_token\": %.1f}\n",
               n_layers, POS, exact ? "exact" : "tolerance mode", tokens, wall[tokens / 10], wall[tokens / 2],
               1e6 / wall[tokens / 2], span[tokens / 2], (double)(l1 - l0) / tokens);
    }
    free(wall);
    free(span);
    free(out);
    free(m);
    ok(kernrt_cuda_destroy(ctx), "destroy");
    return 0;
}

int main(int argc, char **argv) {
    if (argc > 1 && strcmp(argv[1], "model") == 0) {
        const int layers = argc > 2 ? atoi(argv[2]) : 24, tokens = argc > 3 ? atoi(argv[3]) : 50;
        if (layers < 1 || tokens < 10) return fprintf(stderr, "layers >= 1, tokens >= 10\n"), 2;
        return model_decode(layers, tokens);
    }
    const int steps = argc > 1 ? atoi(argv[1]) : 300;
    if (steps < 10) return fprintf(stderr, "steps >= 10\n"), 2;
    kernrt_cuda_ctx *ctx = NULL;
    ok(kernrt_cuda_create(0, &ctx), "create");
    uint16_t *table = malloc((size_t)VOCAB * DIM * sizeof(uint16_t));
    for (size_t i = 0; i < (size_t)VOCAB * DIM; ++i) {
        const float v = 0.04f * uniform();
        uint32_t bits;
        memcpy(&bits, &v, 4);
        table[i] = (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16); /* round to nearest even */
    }
    ok(kernrt_cuda_prepare_embedding(ctx, KERNRT_BF16, table, NULL, VOCAB, DIM), "prepare");
    free(table);
    kernrt_buf x, xb;
    ok(kernrt_cuda_alloc(ctx, DIM, &x), "alloc");
    ok(kernrt_cuda_alloc(ctx, DIM, &xb), "alloc");
    const kernrt_buf q = random_buf(ctx, QD), k = random_buf(ctx, KVD), o = random_buf(ctx, DIM);
    const kernrt_buf g = random_buf(ctx, HIDDEN), u = random_buf(ctx, HIDDEN);
    float *ones = malloc(DIM * sizeof(float));
    for (int i = 0; i < DIM; ++i) ones[i] = 1.0f;
    kernrt_buf w;
    ok(kernrt_cuda_upload(ctx, ones, DIM, &w), "upload");
    free(ones);
    void *stream_ptr = NULL;
    ok(kernrt_cuda_stream(ctx, &stream_ptr), "stream");
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    cudaEvent_t ev0, ev1;
    cuda_ok(cudaEventCreate(&ev0), "event");
    cuda_ok(cudaEventCreate(&ev1), "event");
    const uint64_t pos = 511;
    const float eps = 1e-5f, theta = 1.3e5f;
    float out[DIM];
    double *wall = malloc(steps * sizeof(double)), *issue = malloc(steps * sizeof(double)),
           *span = malloc(steps * sizeof(double));
    for (int exact = 1; exact >= 0; --exact) {
        ok(kernrt_cuda_set_exact(ctx, exact), "set_exact");
        uint64_t l0 = 0, l1 = 0;
        for (int i = -WARM; i < steps; ++i) {
            if (i == 0) ok(kernrt_cuda_kernel_launches(&l0), "launches");
            const double t0 = now_us();
            cuda_ok(cudaEventRecord(ev0, stream), "record");
            ok(kernrt_cuda_embed(ctx, 7, x, 0), "embed");
            ok(kernrt_cuda_rms_norm(ctx, xb, x, w, 1, DIM, eps), "rms_norm");
            ok(kernrt_cuda_rope(ctx, q, k, QD, KVD, 1, &pos, 1, HEAD, theta, 0), "rope");
            ok(kernrt_cuda_add_in_place(ctx, x, o, DIM), "add");
            ok(kernrt_cuda_rms_norm(ctx, xb, x, w, 1, DIM, eps), "rms_norm");
            ok(kernrt_cuda_silu_mul(ctx, g, u, HIDDEN), "silu_mul");
            ok(kernrt_cuda_add_in_place(ctx, x, o, DIM), "add");
            ok(kernrt_cuda_flush(ctx), "flush");
            const double t_issued = now_us();
            cuda_ok(cudaEventRecord(ev1, stream), "record");
            ok(kernrt_cuda_read(ctx, x, out, DIM), "read");
            const double t1 = now_us();
            if (i >= 0) {
                float ms = 0.0f;
                cuda_ok(cudaEventElapsedTime(&ms, ev0, ev1), "elapsed");
                wall[i] = t1 - t0;
                issue[i] = t_issued - t0;
                span[i] = ms * 1e3;
            }
        }
        ok(kernrt_cuda_kernel_launches(&l1), "launches");
        qsort(wall, steps, sizeof(double), cmp);
        qsort(issue, steps, sizeof(double), cmp);
        qsort(span, steps, sizeof(double), cmp);
        printf("{\"name\": \"decode step, configs[1] row ops, C ABI%s\", \"steps\": %d, \"wall_us_p10\": %.2f, "
               "\"wall_us_median\": %.2f, \"issue_us_median\": %.2f, \"ops\": 7, \"issue_us_per_op\": %.2f, "
               "\"device_span_us_median\": %.2f, \"launches_per_step\": %.2f}\n",
               exact ? "" : ", tolerance mode", steps, wall[steps / 10], wall[steps / 2], issue[steps / 2],
               issue[steps / 2] / 7.0, span[steps / 2], (double)(l1 - l0) / steps);
    }
    free(wall);
    free(issue);
    free(span);
    ok(kernrt_cuda_destroy(ctx), "destroy");
    return 0;
}
