// The reference backend's contractions on the device, in its arithmetic order
// (src/backends/reference.rs:73-79, 151-159, 259-306, 402-482): projections
// and logits as y[r, o] = dot(decode_row(W, o), x[r]) with one f32 accumulator
// per output running over k left to right, multiply then add; the key/value
// cache write; causal attention with the reference's score, softmax and
// weighted-sum order.  Every operation is an explicit _rn intrinsic (the
// library builds with -fmad=false), so projections, logits and the cache are
// bit-identical to the reference; attention differs only through expf.
#include "kernels.cuh"
#include "bulk.cuh"

#include <cuda_fp16.h>

namespace krt {
namespace {

constexpr unsigned kFullMask = 0xffffffffu;

__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float bf16f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

cudaError_t launched() {
    count_launch();
    return cudaGetLastError();
}

// ---- projections --------------------------------------------------------------

constexpr int kBK = 32;   // k per staged chunk (one Q8_0 block)
constexpr int kBN = 64;   // outputs per CTA: 16 threads x 4
constexpr int kPad = 4;   // floats of padding per staged k-row

// A CTA computes a BM x 64 tile of y with 16 x 16 threads, TM rows x 4 outputs
// each.  Per chunk of 32 k it stages x[rows, k] and the decoded W[outputs, k]
// transposed in shared memory; every accumulator then takes the chunk's k in
// order, so each output is the reference's sequential dot.  Two staging
// buffers: chunk k + 1 is loaded from global memory into registers before
// chunk k's products and stored after them, so the loads' latency overlaps
// the arithmetic.  k past in_dim is staged as zeros: 0*0 added to a partial
// sum that starts at +0 and never becomes -0 leaves it unchanged.  Requires
// in_dim % 8 == 0 (% 32 for Q8_0).
template <int SRC, int TM>
__global__ void __launch_bounds__(256) k_project(const void *__restrict__ w, const float *__restrict__ wsc,
                                                 int out_dim, int in_dim, const float *__restrict__ x, int rows,
                                                 float *__restrict__ y) {
    constexpr int BM = 16 * TM;
    constexpr int XV = (BM * (kBK / 4) + 255) / 256;  // x float4 per thread per chunk
    __shared__ __align__(16) float xs[2][kBK][BM + kPad];
    __shared__ __align__(16) float ws[2][kBK][kBN + kPad];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int o0 = blockIdx.x * kBN, r0 = blockIdx.y * BM;
    float acc[TM][4];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    // one chunk's global loads, held in registers until they are staged
    float4 xr[XV];
    uint4 wt = make_uint4(0u, 0u, 0u, 0u);
    float wsc_r = 0.0f;
    float4 wf[2];
    auto load = [&](int k0) {
#pragma unroll
        for (int v = 0; v < XV; ++v) {
            const int idx = tid + 256 * v, r = idx >> 3, c = (idx & 7) << 2;
            xr[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (idx < BM * (kBK / 4) && r0 + r < rows && k0 + c < in_dim)
                xr[v] = __ldg(reinterpret_cast<const float4 *>(x + (size_t)(r0 + r) * in_dim + k0 + c));
        }
        if constexpr (SRC == SRC_BF16) {
            const int o = tid >> 2, c = (tid & 3) << 3;
            wt = make_uint4(0u, 0u, 0u, 0u);
            if (o0 + o < out_dim && k0 + c < in_dim)
                wt = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(w) + (size_t)(o0 + o) * in_dim +
                                                           k0 + c));
        } else if constexpr (SRC == SRC_Q8) {
            const int o = tid >> 1, c = (tid & 1) << 4;
            wt = make_uint4(0u, 0u, 0u, 0u);
            wsc_r = 0.0f;
            if (tid < 128 && o0 + o < out_dim && k0 + c < in_dim) {
                wt = __ldg(reinterpret_cast<const uint4 *>(static_cast<const int8_t *>(w) + (size_t)(o0 + o) * in_dim +
                                                           k0 + c));
                wsc_r = __ldg(wsc + (size_t)(o0 + o) * (in_dim >> 5) + (k0 >> 5));
            }
        } else {
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                const int idx = tid + 256 * v, o = idx >> 3, c = (idx & 7) << 2;
                wf[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (o0 + o < out_dim && k0 + c < in_dim)
                    wf[v] = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(w) +
                                                                   (size_t)(o0 + o) * in_dim + k0 + c));
            }
        }
    };
    // the held chunk into staging buffer b: x k-major, W decoded as
    // Matrix::decode_row does, k-major
    auto stage = [&](int b) {
#pragma unroll
        for (int v = 0; v < XV; ++v) {
            const int idx = tid + 256 * v, r = idx >> 3, c = (idx & 7) << 2;
            if (idx < BM * (kBK / 4)) {
                xs[b][c][r] = xr[v].x;
                xs[b][c + 1][r] = xr[v].y;
                xs[b][c + 2][r] = xr[v].z;
                xs[b][c + 3][r] = xr[v].w;
            }
        }
        if constexpr (SRC == SRC_BF16) {
            const int o = tid >> 2, c = (tid & 3) << 3;
            const uint32_t p[4] = {wt.x, wt.y, wt.z, wt.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ws[b][c + 2 * e][o] = bf16f(p[e] & 0xffffu);
                ws[b][c + 2 * e + 1][o] = bf16f(p[e] >> 16);
            }
        } else if constexpr (SRC == SRC_Q8) {
            if (tid < 128) {
                const int o = tid >> 1, c = (tid & 1) << 4;
                const uint32_t p[4] = {wt.x, wt.y, wt.z, wt.w};
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    ws[b][c + e][o] = mul_rn((float)(int8_t)((p[e >> 2] >> (8 * (e & 3))) & 0xffu), wsc_r);
            }
        } else {
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                const int idx = tid + 256 * v, o = idx >> 3, c = (idx & 7) << 2;
                ws[b][c][o] = wf[v].x;
                ws[b][c + 1][o] = wf[v].y;
                ws[b][c + 2][o] = wf[v].z;
                ws[b][c + 3][o] = wf[v].w;
            }
        }
    };

    load(0);
    stage(0);
    __syncthreads();
    int b = 0;
    for (int k0 = 0; k0 < in_dim; k0 += kBK) {
        const bool more = k0 + kBK < in_dim;
        if (more) load(k0 + kBK);
#pragma unroll 8
        for (int kk = 0; kk < kBK; ++kk) {
            float a[TM];
            if constexpr (TM == 4) {
                const float4 t = *reinterpret_cast<const float4 *>(&xs[b][kk][ty * 4]);
                a[0] = t.x; a[1] = t.y; a[2] = t.z; a[3] = t.w;
            } else {
#pragma unroll
                for (int i = 0; i < TM; ++i) a[i] = xs[b][kk][ty * TM + i];
            }
            const float4 bv = *reinterpret_cast<const float4 *>(&ws[b][kk][tx * 4]);
#pragma unroll
            for (int i = 0; i < TM; ++i) {
                acc[i][0] = add_rn(acc[i][0], mul_rn(bv.x, a[i]));
                acc[i][1] = add_rn(acc[i][1], mul_rn(bv.y, a[i]));
                acc[i][2] = add_rn(acc[i][2], mul_rn(bv.z, a[i]));
                acc[i][3] = add_rn(acc[i][3], mul_rn(bv.w, a[i]));
            }
        }
        // the other buffer was last read before the previous barrier
        if (more) stage(b ^ 1);
        __syncthreads();
        b ^= 1;
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = r0 + ty * TM + i;
        if (r >= rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + tx * 4 + j;
            if (o < out_dim) y[(size_t)r * out_dim + o] = acc[i][j];
        }
    }
}

// Any shape: one thread per output, the dot in order, decoding each weight.
template <int SRC>
__global__ void __launch_bounds__(256) k_project_scalar(const void *__restrict__ w, const float *__restrict__ wsc,
                                                        int out_dim, int in_dim, const float *__restrict__ x,
                                                        int rows, float *__restrict__ y) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)rows * out_dim) return;
    const int r = (int)(i / out_dim), o = (int)(i - (long long)r * out_dim);
    const float *xr = x + (size_t)r * in_dim;
    float sum = 0.0f;
    for (int k = 0; k < in_dim; ++k) {
        float wv;
        if constexpr (SRC == SRC_BF16) wv = bf16f(static_cast<const uint16_t *>(w)[(size_t)o * in_dim + k]);
        else if constexpr (SRC == SRC_Q8)
            wv = mul_rn((float)static_cast<const int8_t *>(w)[(size_t)o * in_dim + k],
                        wsc[(size_t)o * (in_dim >> 5) + (k >> 5)]);
        else wv = static_cast<const float *>(w)[(size_t)o * in_dim + k];
        sum = add_rn(sum, mul_rn(wv, xr[k]));
    }
    y[i] = sum;
}

// Decode projections (R <= 4 rows): one consumer warp per 32 outputs, lane o
// running output o's dots for the R rows, and one producer warp that streams
// the 32 weight rows and the R x rows through kGemvStages shared-memory stages
// of CK columns, one bulk copy per row per stage (producer lane o copies row
// o).  The copy engine takes the 32 requests of a stage one after another
// (about a microsecond per stage); with its own warp issuing them that time
// overlaps the consumer's sequential accumulations instead of adding to them.
// full[s] counts a stage's bytes in, empty[s] hands it back to the producer.
// Row slots are padded to an odd number of 16-byte units: the lanes' 16-byte
// reads of one column land in distinct banks.  Requires in_dim % 8 (% 128
// for Q8_0, whose block scales then move in 16-byte units too).
// Chunks of CK = 512 columns, or 1024 when the matrix has fewer warps of
// outputs than the GPU has SMs: each SM then runs one CTA, whose copy engine
// takes a stage's 32 requests one after another, and wider requests move more
// bytes per request.
constexpr int kGemvCK = 512;
constexpr int kGemvCKWide = 1024;
constexpr int kGemvStages = 2;

template <int SRC, int CK>
struct GemvGeom {
    static constexpr int esz = SRC == SRC_BF16 ? 2 : (SRC == SRC_Q8 ? 1 : 4);
    static constexpr int wrow = CK * esz + (SRC == SRC_Q8 ? CK / 8 : 0);  // codes (+ scales)
    static constexpr int wstride = ((wrow + 31) & ~31) + 16;              // odd x 16 B
    __host__ __device__ static constexpr size_t stage_bytes(int rows) { return 32 * (size_t)wstride + (size_t)rows * CK * 4; }
};

// Up to three matrices sharing x and in_dim in one launch (the trait's
// project_qkv / project_gate_up, mod.rs:320-337): their CTAs run side by side
// instead of one projection after another.
struct GemvSet {
    const void *w[3];
    const float *wsc[3];
    float *y[3];
    int out_dim[3];
    int cta_end[3];  // exclusive prefix sums of each matrix's CTAs
    int n;
};

// a[m] for a kernel-parameter array with constant indices only (a runtime
// index would copy the whole parameter struct to local memory)
template <class T>
__device__ __forceinline__ T pick3(const T (&a)[3], int m) {
    return m == 0 ? a[0] : (m == 1 ? a[1] : a[2]);
}

// Lane o's sums over one stage's columns [0, tc) for the R rows, in column
// order.  wr is the lane's weight row slot (codes, then Q8_0 block scales at
// +CK), xs the stage's R rows of x.  One warp issues all of a column's work
// (shared-memory loads, decoding, the multiply and the dependent add), so the
// issue rate, not the add latency, sets the pace: 16 columns a step with the
// next step's raw words loaded ahead and the loop unrolled 4 times issues a
// column in about 5.3 cycles, against 6.9 for 8 columns a step with decoded
// values carried over (one warp on one B200 sub-partition).  tc % 16 == 0.
template <int SRC, int R, int CK>
struct GemvWords16 {
    uint4 w[SRC == SRC_F32 ? 4 : (SRC == SRC_BF16 ? 2 : 1)];
    float sc;
    float4 x[R][4];
};

__device__ __forceinline__ uint32_t u4_at(const uint4 &u, int i) { return i == 0 ? u.x : (i == 1 ? u.y : (i == 2 ? u.z : u.w)); }
__device__ __forceinline__ float f4_at(const float4 &u, int i) { return i == 0 ? u.x : (i == 1 ? u.y : (i == 2 ? u.z : u.w)); }

template <int SRC, int R, int CK>
__device__ __forceinline__ void gemv_chain16(const unsigned char *wr, const float *xs, int tc, float (&acc)[R]) {
    using Words = GemvWords16<SRC, R, CK>;
    auto load = [&](int k, Words &t) {
        if constexpr (SRC == SRC_BF16) {
            t.w[0] = *reinterpret_cast<const uint4 *>(wr + 2 * k);
            t.w[1] = *reinterpret_cast<const uint4 *>(wr + 2 * k + 16);
        } else if constexpr (SRC == SRC_Q8) {
            t.w[0] = *reinterpret_cast<const uint4 *>(wr + k);
            t.sc = reinterpret_cast<const float *>(wr + CK)[k >> 5];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) t.w[i] = *reinterpret_cast<const uint4 *>(wr + 4 * k + 16 * i);
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) t.x[r][i] = *reinterpret_cast<const float4 *>(xs + r * CK + k + 4 * i);
    };
    auto step = [&](const Words &t) {
        float wv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            if constexpr (SRC == SRC_BF16) {
                const uint32_t p = u4_at(t.w[e >> 3], (e >> 1) & 3);
                wv[e] = __uint_as_float((e & 1) ? (p & 0xffff0000u) : (p << 16));
            } else if constexpr (SRC == SRC_Q8) {
                const uint32_t p = u4_at(t.w[0], e >> 2);
                wv[e] = mul_rn((float)(int8_t)((p >> (8 * (e & 3))) & 0xffu), t.sc);
            } else {
                wv[e] = __uint_as_float(u4_at(t.w[e >> 2], e & 3));
            }
        }
#pragma unroll
        for (int e = 0; e < 16; ++e)
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = add_rn(acc[r], mul_rn(wv[e], f4_at(t.x[r][e >> 2], e & 3)));
    };
    Words cur, nxt;
    load(0, cur);
#pragma unroll 4
    for (int k = 0; k < tc; k += 16) {
        load(k + 16 < tc ? k + 16 : k, nxt);
        step(cur);
        cur = nxt;
    }
}

// The same, 8 columns a step (tc % 8 == 0): the next step's words loaded and
// decoded ahead of the current step's products and adds.
template <int SRC, int R, int CK>
__device__ __forceinline__ void gemv_chain8(const unsigned char *wr, const float *xs, int tc, float (&acc)[R]) {
    // step k's eight weights (decoded) and x values; the next
    // step is loaded and decoded ahead of the current step's adds,
    // so shared-memory latency and decoding stay off the chain
    auto ldw = [&](int k, float *wv) {
        if constexpr (SRC == SRC_BF16) {
            const uint4 t = *reinterpret_cast<const uint4 *>(wr + 2 * k);
            const uint32_t p[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                wv[2 * e] = __uint_as_float(p[e] << 16);
                wv[2 * e + 1] = __uint_as_float(p[e] & 0xffff0000u);
            }
        } else if constexpr (SRC == SRC_Q8) {
            const uint2 t = *reinterpret_cast<const uint2 *>(wr + k);
            const float sc = reinterpret_cast<const float *>(wr + CK)[k >> 5];
            const uint32_t p[2] = {t.x, t.y};
#pragma unroll
            for (int e = 0; e < 8; ++e)
                wv[e] = mul_rn((float)(int8_t)((p[e >> 2] >> (8 * (e & 3))) & 0xffu), sc);
        } else {
            const float4 a = *reinterpret_cast<const float4 *>(wr + 4 * k);
            const float4 b2 = *reinterpret_cast<const float4 *>(wr + 4 * k + 16);
            wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
            wv[4] = b2.x; wv[5] = b2.y; wv[6] = b2.z; wv[7] = b2.w;
        }
    };
    auto ldx = [&](int k, float (*xv)[8]) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float4 x0 = *reinterpret_cast<const float4 *>(xs + r * CK + k);
            const float4 x1 = *reinterpret_cast<const float4 *>(xs + r * CK + k + 4);
            xv[r][0] = x0.x; xv[r][1] = x0.y; xv[r][2] = x0.z; xv[r][3] = x0.w;
            xv[r][4] = x1.x; xv[r][5] = x1.y; xv[r][6] = x1.z; xv[r][7] = x1.w;
        }
    };
    float wv[8], xv[R][8], nwv[8], nxv[R][8];
    ldw(0, wv);
    ldx(0, xv);
#pragma unroll 2
    for (int k = 0; k < tc; k += 8) {
        const int kn = k + 8 < tc ? k + 8 : k;
        ldw(kn, nwv);
        ldx(kn, nxv);
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r] = add_rn(acc[r], mul_rn(wv[e], xv[r][e]));
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            wv[e] = nwv[e];
#pragma unroll
            for (int r = 0; r < R; ++r) xv[r][e] = nxv[r][e];
        }
    }
}

template <int SRC, int R, int CK>
__global__ void __launch_bounds__(64) k_gemv(GemvSet set, int in_dim, const float *__restrict__ x, int *err) {
    using Geo = GemvGeom<SRC, CK>;
    constexpr int NS = kGemvStages;
    constexpr int SB = (int)Geo::stage_bytes(R);
    extern __shared__ __align__(16) unsigned char gsm[];
    __shared__ __align__(8) uint64_t full[NS], empty[NS];
    __shared__ int issued_sh;
    int m = 0;
    if (set.n > 1 && (int)blockIdx.x >= set.cta_end[0]) m = (set.n > 2 && (int)blockIdx.x >= set.cta_end[1]) ? 2 : 1;
    const int blk = (int)blockIdx.x - (m == 0 ? 0 : (m == 1 ? set.cta_end[0] : set.cta_end[1]));
    const int out_dim = pick3(set.out_dim, m);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, o = blk * 32 + lane;
    const bool live = o < out_dim;
    const int nlive = min(32, out_dim - blk * 32);
    const int nchunks = (in_dim + CK - 1) / CK;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    bool ok = true;
    int consumed = 0;
    if (warp == 1) {
        // producer: chunk c into stage c % NS once chunk c - NS has been consumed
        const void *__restrict__ w = pick3(set.w, m);
        const float *__restrict__ wsc = pick3(set.wsc, m);
        int issued = 0;
        for (; issued < nchunks; ++issued) {
            const int c = issued, k0 = c * CK, tc = min(CK, in_dim - k0);
            if (c >= NS && !__all_sync(kFullMask, mbar_wait_bounded(&empty[c % NS], (uint32_t)(c / NS - 1) & 1u)))
                break;  // the consumer stopped: issue nothing more
            const uint32_t wb = (uint32_t)(tc * Geo::esz), sb = SRC == SRC_Q8 ? (uint32_t)(tc / 8) : 0u;
            uint64_t *b = &full[c % NS];
            if (lane == 0) mbar_arrive_expect_tx(b, (uint32_t)nlive * (wb + sb) + (uint32_t)(R * tc * 4));
            __syncwarp();
            unsigned char *st = gsm + (size_t)(c % NS) * SB;
            if (live) {
                bulk_load(st + (size_t)lane * Geo::wstride,
                          static_cast<const unsigned char *>(w) + ((size_t)o * in_dim + k0) * Geo::esz, wb, b);
                if constexpr (SRC == SRC_Q8)
                    bulk_load(st + (size_t)lane * Geo::wstride + CK, wsc + (size_t)o * (in_dim >> 5) + (k0 >> 5),
                              sb, b);
            }
            if (lane < R)
                bulk_load(st + 32 * Geo::wstride + (size_t)lane * CK * 4, x + (size_t)lane * in_dim + k0,
                          (uint32_t)(tc * 4), b);
        }
        if (lane == 0) issued_sh = issued;
    } else {
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            if (!__all_sync(kFullMask, mbar_wait_bounded(&full[c % NS], (uint32_t)(c / NS) & 1u))) {
                if (lane == 0) atomicOr(err, ERR_TIMEOUT);
                ok = false;
                break;
            }
            const unsigned char *st = gsm + (size_t)(c % NS) * SB;
            const unsigned char *wr = st + (size_t)lane * Geo::wstride;
            const float *xs = reinterpret_cast<const float *>(st + 32 * Geo::wstride);
            const int tc = min(CK, in_dim - c * CK);
            if (live) {
                if ((tc & 15) == 0) gemv_chain16<SRC, R, CK>(wr, xs, tc, acc);
                else gemv_chain8<SRC, R, CK>(wr, xs, tc, acc);
            }
            // every lane's reads of this stage are done before it goes back
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[c % NS]);
            consumed = c + 1;
        }
        if (ok && live)
#pragma unroll
            for (int r = 0; r < R; ++r) pick3(set.y, m)[(size_t)r * out_dim + o] = acc[r];
    }
    __syncthreads();
    if (!ok && threadIdx.x == 0)
        // copies still in flight: wait for them (bounded) before the memory goes
        for (int c = consumed; c < issued_sh; ++c) mbar_wait_bounded(&full[c % NS], (uint32_t)(c / NS) & 1u);
}

// the stages plus a little static shared memory within the 227 KB opt-in limit
template <int SRC, int CK>
bool gemv_smem_fits(int rows) {
    return (size_t)kGemvStages * GemvGeom<SRC, CK>::stage_bytes(rows) + 256 <= 232448;
}

template <int SRC, int R, int CK>
cudaError_t launch_gemv_ck(const GemvSet &set, int in_dim, const float *x, int *err, cudaStream_t s) {
    const size_t smem = (size_t)kGemvStages * GemvGeom<SRC, CK>::stage_bytes(R);
    cudaError_t e = cudaFuncSetAttribute(k_gemv<SRC, R, CK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_gemv<SRC, R, CK><<<(unsigned)set.cta_end[set.n - 1], 64, smem, s>>>(set, in_dim, x, err);
    return launched();
}

template <int SRC, int R>
cudaError_t launch_gemv(const GemvSet &set, int in_dim, const float *x, int *err, cudaStream_t s) {
    const bool wide = set.cta_end[set.n - 1] < device_sms() && in_dim > kGemvCK && gemv_smem_fits<SRC, kGemvCKWide>(R);
    return wide ? launch_gemv_ck<SRC, R, kGemvCKWide>(set, in_dim, x, err, s)
                : launch_gemv_ck<SRC, R, kGemvCK>(set, in_dim, x, err, s);
}

template <int SRC>
cudaError_t gemv_rows(const GemvSet &set, int in_dim, const float *x, int rows, int *err, cudaStream_t s) {
    switch (rows) {
    case 1: return launch_gemv<SRC, 1>(set, in_dim, x, err, s);
    case 2: return launch_gemv<SRC, 2>(set, in_dim, x, err, s);
    case 3: return launch_gemv<SRC, 3>(set, in_dim, x, err, s);
    default: return launch_gemv<SRC, 4>(set, in_dim, x, err, s);
    }
}

template <int SRC>
bool gemv_fits(const void *w, const float *wsc, int in_dim, const float *x, int rows) {
    return rows <= 4 && gemv_smem_fits<SRC, kGemvCK>(rows) && in_dim % (SRC == SRC_Q8 ? 128 : 8) == 0 &&
           ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 && (SRC != SRC_Q8 || ((uintptr_t)wsc & 15) == 0);
}

template <int SRC>
cudaError_t project_src(const void *w, const float *wsc, int out_dim, int in_dim, const float *x, int rows, float *y,
                        int *err, cudaStream_t s) {
    if (gemv_fits<SRC>(w, wsc, in_dim, x, rows)) {
        GemvSet set{};
        set.w[0] = w;
        set.wsc[0] = wsc;
        set.y[0] = y;
        set.out_dim[0] = out_dim;
        set.cta_end[0] = (out_dim + 31) / 32;
        set.n = 1;
        return gemv_rows<SRC>(set, in_dim, x, rows, err, s);
    }
    const bool tiled = in_dim % (SRC == SRC_Q8 ? 32 : 8) == 0 && ((uintptr_t)x & 15) == 0 &&
                       ((uintptr_t)w & 15) == 0;
    if (!tiled) {
        const long long n = (long long)rows * out_dim;
        k_project_scalar<SRC><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w, wsc, out_dim, in_dim, x, rows, y);
        return launched();
    }
    const unsigned gx = (unsigned)((out_dim + kBN - 1) / kBN);
    if (rows >= 64) {
        k_project<SRC, 4><<<dim3(gx, (unsigned)((rows + 63) / 64)), 256, 0, s>>>(w, wsc, out_dim, in_dim, x, rows, y);
    } else {
        k_project<SRC, 1><<<dim3(gx, (unsigned)((rows + 15) / 16)), 256, 0, s>>>(w, wsc, out_dim, in_dim, x, rows, y);
    }
    return launched();
}

// ---- key/value cache ------------------------------------------------------------

// reference.rs:151-159: row i of k and v into cache row dst_rows[i]
// (layer * seq_len + slot).
__global__ void __launch_bounds__(256) k_kv_write(float *__restrict__ kc, float *__restrict__ vc, int kv_dim,
                                                  const int32_t *__restrict__ dst_rows, const float *__restrict__ k,
                                                  const float *__restrict__ v, int rows) {
    const long long n = (long long)rows * kv_dim;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / kv_dim), e = (int)(i - (long long)r * kv_dim);
        const size_t d = (size_t)dst_rows[r] * kv_dim + e;
        kc[d] = k[i];
        vc[d] = v[i];
    }
}

// The same with 16-byte items (kv_dim % 4, 16-byte aligned buffers): q4
// float4 per row, n4 items in all.
__global__ void __launch_bounds__(256) k_kv_write4(float *__restrict__ kc, float *__restrict__ vc, int q4,
                                                   const int32_t *__restrict__ dst_rows, const float *__restrict__ k,
                                                   const float *__restrict__ v, int n4) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const int r = i / q4, e = i - r * q4;
        const size_t d = ((size_t)dst_rows[r] * q4 + e) * 4;
        *reinterpret_cast<float4 *>(kc + d) = *reinterpret_cast<const float4 *>(k + (size_t)i * 4);
        *reinterpret_cast<float4 *>(vc + d) = *reinterpret_cast<const float4 *>(v + (size_t)i * 4);
    }
}

// ---- attention ------------------------------------------------------------------

// sum_{i < n} v[i] from shared memory in index order, one thread: sixteen
// values loaded ahead of their adds, so the loads stay off the add chain.
__device__ __forceinline__ float seq_sum_smem(const float *v, int n) {
    float sum = 0.0f;
    int i = 0;
    if (((uintptr_t)v & 15) == 0)
        for (; i + 16 <= n; i += 16) {
            float4 t[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) t[j] = *reinterpret_cast<const float4 *>(v + i + 4 * j);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sum = add_rn(sum, t[j].x);
                sum = add_rn(sum, t[j].y);
                sum = add_rn(sum, t[j].z);
                sum = add_rn(sum, t[j].w);
            }
        }
    for (; i < n; ++i) sum = add_rn(sum, v[i]);
    return sum;
}

// reference.rs:418-482 for one (query row, head): a CTA of 128 threads.
//   scores: thread per position, each a sequential dot over head_size, times
//           1/sqrt(head_size);
//   softmax: the maximum (order-free), exp(s - max), the sum by one thread in
//            position order, then s / sum (written to att);
//   output: thread per element, accumulated over positions in order.
// Window: positions shared_start..shared_end, then att_start..=slot.
__global__ void __launch_bounds__(128) k_attention(const float *__restrict__ q, float *__restrict__ out,
                                                   float *__restrict__ att, const float *__restrict__ kc,
                                                   const float *__restrict__ vc, const int32_t *__restrict__ win,
                                                   int n_heads, int kv_mul, int head_size, int kv_dim, int seq_len,
                                                   size_t loff) {
    extern __shared__ __align__(16) float asm_[];
    const int row = blockIdx.x / n_heads, h = blockIdx.x - row * n_heads;
    const int tid = threadIdx.x;
    const int att_start = win[4 * row], slot = win[4 * row + 1], ss = win[4 * row + 2], se = win[4 * row + 3];
    const int n_shared = se - ss, count = n_shared + slot - att_start + 1;
    float *qh = asm_;                       // [head_size]
    float *sc = asm_ + ((head_size + 3) & ~3);  // [count]
    __shared__ float red[4];
    __shared__ float total;
    const int width = n_heads * head_size;
    const float *qg = q + (size_t)row * width + (size_t)h * head_size;
    for (int e = tid; e < head_size; e += 128) qh[e] = qg[e];
    __syncthreads();
    const size_t kv = (size_t)(h / kv_mul) * head_size;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)head_size));
    auto pos_of = [&](int i) { return i < n_shared ? ss + i : att_start + (i - n_shared); };
    for (int i = tid; i < count; i += 128) {
        const float *kr = kc + loff + (size_t)pos_of(i) * kv_dim + kv;
        float d = 0.0f;
        for (int e = 0; e < head_size; ++e) d = add_rn(d, mul_rn(qh[e], kr[e]));
        sc[i] = mul_rn(d, scale);
    }
    __syncthreads();
    // the maximum over positions, NaN scores skipped as the reference's `>` does
    float m = -INFINITY;
    for (int i = tid; i < count; i += 128) m = fmaxf(m, sc[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    for (int i = tid; i < count; i += 128) sc[i] = expf(__fsub_rn(sc[i], m));
    __syncthreads();
    if (tid == 0) total = seq_sum_smem(sc, count);
    __syncthreads();
    const float sum = total;
    float *ag = att + ((size_t)row * n_heads + h) * seq_len;
    for (int i = tid; i < count; i += 128) {
        const float a = __fdiv_rn(sc[i], sum);
        sc[i] = a;
        ag[i] = a;
    }
    __syncthreads();
    float *og = out + (size_t)row * width + (size_t)h * head_size;
    for (int e = tid; e < head_size; e += 128) {
        float o = 0.0f;
        for (int i = 0; i < count; ++i) o = add_rn(o, mul_rn(sc[i], vc[loff + (size_t)pos_of(i) * kv_dim + kv + e]));
        og[e] = o;
    }
}

// ---- attention in two kernels ---------------------------------------------------

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Window position i of a row: the shared range first, then the row's own.
__device__ __forceinline__ int win_pos(const int32_t *w, int i) {
    const int n_shared = w[3] - w[2];
    return i < n_shared ? w[2] + i : w[0] + (i - n_shared);
}

// Scores (reference.rs:439-446): raw[row][h][i] = dot(q_h, k_pos) * scale,
// thread per position, each dot over head_size in order, into scratch rows of
// `stride` floats.  Grid (row x head, position blocks of 128).
__global__ void __launch_bounds__(128) k_att_scores(const float *__restrict__ q, float *__restrict__ raw,
                                                    const float *__restrict__ kc, const int32_t *__restrict__ win,
                                                    int n_heads, int kv_mul, int head_size, int kv_dim, int stride,
                                                    size_t loff) {
    extern __shared__ __align__(16) float qsh[];
    const int row = blockIdx.x / n_heads, h = blockIdx.x - row * n_heads;
    const int32_t *w = win + 4 * row;
    const int count = (w[3] - w[2]) + w[1] - w[0] + 1;
    const int i = blockIdx.y * 128 + threadIdx.x;
    if ((int)blockIdx.y * 128 >= count) return;
    const float *qg = q + ((size_t)row * n_heads + h) * head_size;
    for (int e = threadIdx.x; e < head_size; e += 128) qsh[e] = qg[e];
    __syncthreads();
    if (i >= count) return;
    const float *kr = kc + loff + (size_t)win_pos(w, i) * kv_dim + (size_t)(h / kv_mul) * head_size;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)head_size));
    float d = 0.0f;
    if ((head_size & 3) == 0 && ((uintptr_t)kr & 15) == 0) {
        // eight float4 of the key in flight, then their products in order
        for (int e0 = 0; e0 < head_size; e0 += 32) {
            float4 kv4[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (e0 + 4 * j < head_size) kv4[j] = __ldg(reinterpret_cast<const float4 *>(kr + e0 + 4 * j));
            float4 q4[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (e0 + 4 * j < head_size) q4[j] = *reinterpret_cast<const float4 *>(qsh + e0 + 4 * j);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (e0 + 4 * j >= head_size) break;
                d = add_rn(d, mul_rn(q4[j].x, kv4[j].x));
                d = add_rn(d, mul_rn(q4[j].y, kv4[j].y));
                d = add_rn(d, mul_rn(q4[j].z, kv4[j].z));
                d = add_rn(d, mul_rn(q4[j].w, kv4[j].w));
            }
        }
    } else {
        for (int e = 0; e < head_size; ++e) d = add_rn(d, mul_rn(qsh[e], kr[e]));
    }
    raw[((size_t)row * n_heads + h) * stride + i] = mul_rn(d, scale);
}

// Scores for windows that map window positions to the same cache slots (the
// rows of one sequence: the same shared range and start, their own last
// slot): a CTA takes 16 rows x 64 positions of one head.  The 64 key rows are
// staged once in shared memory and serve all 16 rows, and each thread runs
// eight dots (eight rows, one position), each over head_size in order
// (reference.rs:439-446), so the eight chains overlap.  Grid (row blocks,
// position blocks, heads); blocks past every row's window exit at once.
constexpr int kScRows = 16, kScPos = 64;

__global__ void __launch_bounds__(128) k_att_scores_rows(const float *__restrict__ q, float *__restrict__ raw,
                                                         const float *__restrict__ kc,
                                                         const int32_t *__restrict__ win, int n_rows, int n_heads,
                                                         int kv_mul, int head_size, int kv_dim, int stride,
                                                         size_t loff) {
    extern __shared__ __align__(16) float scs[];
    const int hs = head_size + 4;                 // row stride: 16-byte reads of one column in distinct banks
    float *ks = scs;                              // [kScPos][hs]
    float *qs = scs + kScPos * hs;                // [kScRows][hs]
    __shared__ int cnt[kScRows];
    const int r0 = blockIdx.x * kScRows, p0 = blockIdx.y * kScPos, h = blockIdx.z;
    const int tid = threadIdx.x;
    const int nr = min(kScRows, n_rows - r0);
    if (tid < kScRows) {
        int c = 0;
        if (tid < nr) {
            const int32_t *w = win + 4 * (r0 + tid);
            c = (w[3] - w[2]) + w[1] - w[0] + 1;
        }
        cnt[tid] = c;
    }
    __syncthreads();
    int maxc = 0;
    for (int r = 0; r < nr; ++r) maxc = max(maxc, cnt[r]);
    if (p0 >= maxc) return;
    const int np = min(kScPos, maxc - p0);
    const int32_t *w0 = win + 4 * r0;  // every row of the launch maps positions alike
    const int h4 = head_size >> 2;
    for (int idx = tid; idx < np * h4; idx += 128) {
        const int p = idx / h4, e = (idx - p * h4) << 2;
        *reinterpret_cast<float4 *>(ks + p * hs + e) = __ldg(reinterpret_cast<const float4 *>(
            kc + loff + (size_t)win_pos(w0, p0 + p) * kv_dim + (size_t)(h / kv_mul) * head_size + e));
    }
    for (int idx = tid; idx < nr * h4; idx += 128) {
        const int r = idx / h4, e = (idx - r * h4) << 2;
        *reinterpret_cast<float4 *>(qs + r * hs + e) =
            __ldg(reinterpret_cast<const float4 *>(q + ((size_t)(r0 + r) * n_heads + h) * head_size + e));
    }
    __syncthreads();
    const int p = tid & (kScPos - 1), rg = tid >> 6;  // rows rg, rg + 2, ..., rg + 14
    if (p >= np) return;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)head_size));
    float d[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = 0.0f;
    const float *kp = ks + p * hs;
#pragma unroll 2
    for (int e = 0; e < head_size; e += 4) {
        const float4 k4 = *reinterpret_cast<const float4 *>(kp + e);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 q4 = *reinterpret_cast<const float4 *>(qs + (rg + 2 * j) * hs + e);  // broadcast
            d[j] = add_rn(d[j], mul_rn(q4.x, k4.x));
            d[j] = add_rn(d[j], mul_rn(q4.y, k4.y));
            d[j] = add_rn(d[j], mul_rn(q4.z, k4.z));
            d[j] = add_rn(d[j], mul_rn(q4.w, k4.w));
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int r = rg + 2 * j;
        if (r < nr && p0 + p < cnt[r]) raw[((size_t)(r0 + r) * n_heads + h) * stride + p0 + p] = mul_rn(d[j], scale);
    }
}

// Softmax and output (reference.rs:448-480) for one (row, head) and a slice
// of `sw` output elements: the raw scores, their maximum (order-free),
// exp(s - max), the sum by one thread in position order, s / sum (slice 0
// writes these to att); then thread e of the slice runs out[e] = sum_i a_i *
// v_pos(i)[e] in position order.  Slices of one head repeat the softmax,
// which is cheap next to the value rows they stream.  The slice's value
// columns move through shared memory in tiles of 2048 / sw positions,
// kAttStages - 1 tiles ahead, every thread issuing 16-byte cp.async copies.
constexpr int kAttTileFloats = 2048;  // positions x slice width per stage (8 KB)

template <int kAttStages>
__global__ void __launch_bounds__(128) k_att_out(float *__restrict__ out, float *__restrict__ att,
                                                 const float *__restrict__ raw, const float *__restrict__ vc,
                                                 const int32_t *__restrict__ win, int n_heads, int kv_mul,
                                                 int head_size, int kv_dim, int seq_len, size_t loff, int stride,
                                                 int sw) {
    extern __shared__ __align__(16) float osm[];
    const int nsl = (head_size + sw - 1) / sw, tp = kAttTileFloats / sw;
    const int rh = blockIdx.x / nsl, sl = blockIdx.x - rh * nsl;
    const int row = rh / n_heads, h = rh - row * n_heads;
    const int tid = threadIdx.x;
    const int32_t *w = win + 4 * row;
    const int count = (w[3] - w[2]) + w[1] - w[0] + 1;
    const int e0 = sl * sw, ne = min(sw, head_size - e0);
    float *sc = osm;                             // [stride]
    float *tiles = osm + ((stride + 3) & ~3);    // [kAttStages][tp][sw]
    __shared__ float red[4];
    __shared__ float total;
    const float *rg = raw + (size_t)rh * stride;
    for (int i = tid; i < count; i += 128) sc[i] = rg[i];
    __syncthreads();
    float m = -INFINITY;  // NaN scores skipped, as the reference's `>` does
    for (int i = tid; i < count; i += 128) m = fmaxf(m, sc[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    for (int i = tid; i < count; i += 128) sc[i] = expf(__fsub_rn(sc[i], m));
    __syncthreads();
    if (tid == 0) total = seq_sum_smem(sc, count);
    __syncthreads();
    const float sum = total;
    float *ag = att + (size_t)rh * seq_len;
    for (int i = tid; i < count; i += 128) {
        const float a = __fdiv_rn(sc[i], sum);
        sc[i] = a;
        if (sl == 0) ag[i] = a;
    }
    const size_t vo = loff + (size_t)(h / kv_mul) * head_size + e0;
    const int chunks = ne >> 2;  // 16-byte pieces of a position's slice
    const int ntiles = (count + tp - 1) / tp;
    auto load_tile = [&](int t) {
        float *dst = tiles + (size_t)(t % kAttStages) * kAttTileFloats;
        const int p0 = t * tp, np = min(tp, count - p0);
        for (int c = tid; c < np * chunks; c += 128) {
            const int p = c / chunks, j = c - p * chunks;
            cp_async16(dst + p * sw + 4 * j, vc + vo + (size_t)win_pos(w, p0 + p) * kv_dim + 4 * j);
        }
    };
    for (int t = 0; t < kAttStages - 1; ++t) {
        if (t < ntiles) load_tile(t);
        cp_async_commit();
    }
    float o = 0.0f;
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<kAttStages - 2>();  // tile t has landed (for this thread's copies)
        __syncthreads();                  // ... and every thread's
        // the stage tile t - 1 used is free: tile t + S - 1 goes there
        if (t + kAttStages - 1 < ntiles) load_tile(t + kAttStages - 1);
        cp_async_commit();
        if (tid < ne) {
            const float *tile = tiles + (size_t)(t % kAttStages) * kAttTileFloats;
            const int p0 = t * tp, np = min(tp, count - p0);
            int p = 0;
            // eight weights and values loaded ahead of their products in order
            for (; p + 8 <= np; p += 8) {
                float a[8], v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    a[j] = sc[p0 + p + j];
                    v[j] = tile[(p + j) * sw + tid];
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) o = add_rn(o, mul_rn(a[j], v[j]));
            }
            for (; p < np; ++p) o = add_rn(o, mul_rn(sc[p0 + p], tile[p * sw + tid]));
        }
    }
    cp_async_wait<0>();
    if (tid < ne) out[(size_t)rh * head_size + e0 + tid] = o;
}

// Decode form of k_att_out (few (row, head) pairs, 32-element slices): the
// same operations in the same order, with the roles split so the value rows
// stream while the chains run.  All 128 threads load the raw scores, take the
// maximum and exp(s - max); then
//   warps 1-3 stream the slice's value rows through a ring of kDecStages tiles
//            of kDecTile positions (16-byte cp.async pieces; each thread's
//            pieces arrive on full[s] when they land, mbarrier.arrive.noinc),
//            starting while warp 0 still sums;
//   warp 0   lane 0 runs the sum in position order; then per tile the warp
//            divides the tile's exps by the sum (writing att for slice 0),
//            runs out[e] = sum_i a_i v_pos(i)[e] over the tile in position
//            order, 16 positions a step with the next step's words loaded
//            ahead, and hands the tile back (empty[s]).
// One warp issuing the copies of every tile between its chain steps, with a
// block barrier per tile, ran the chain at ~25 cycles a position; alone it
// runs at ~6.
constexpr int kDecTile = 128, kDecStages = 6, kDecSw = 32;
constexpr int kDecLoaders = 96;

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__global__ void __launch_bounds__(128) k_att_out_dec(float *__restrict__ out, float *__restrict__ att,
                                                     const float *__restrict__ raw, const float *__restrict__ vc,
                                                     const int32_t *__restrict__ win, int n_heads, int kv_mul,
                                                     int head_size, int kv_dim, int seq_len, size_t loff, int stride,
                                                     int *err) {
    extern __shared__ __align__(16) float osm[];
    __shared__ __align__(8) uint64_t full[kDecStages], empty[kDecStages];
    __shared__ float red[4];
    const int nsl = (head_size + kDecSw - 1) / kDecSw;
    const int rh = blockIdx.x / nsl, sl = blockIdx.x - rh * nsl;
    const int row = rh / n_heads, h = rh - row * n_heads;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int32_t *w = win + 4 * row;
    const int count = (w[3] - w[2]) + w[1] - w[0] + 1;
    const int e0 = sl * kDecSw, ne = min(kDecSw, head_size - e0), chunks = ne >> 2;
    float *sc = osm;                           // [stride]
    float *ring = osm + ((stride + 3) & ~3);   // [kDecStages][kDecTile][kDecSw]
    if (tid == 0) {
        for (int i = 0; i < kDecStages; ++i) {
            mbar_init(&full[i], kDecLoaders);
            mbar_init(&empty[i], 1);
        }
        mbar_fence_init();
    }
    const float *rg = raw + (size_t)rh * stride;
    for (int i = tid; i < count; i += 128) sc[i] = rg[i];
    __syncthreads();
    float m = -INFINITY;  // NaN scores skipped, as the reference's `>` does
    for (int i = tid; i < count; i += 128) m = fmaxf(m, sc[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    for (int i = tid; i < count; i += 128) sc[i] = expf(__fsub_rn(sc[i], m));
    __syncthreads();
    const int ntiles = (count + kDecTile - 1) / kDecTile;
    if (warp > 0) {
        const int lt = tid - 32;
        const size_t vo = loff + (size_t)(h / kv_mul) * head_size + e0;
        for (int t = 0; t < ntiles; ++t) {
            const int st = t % kDecStages;
            if (t >= kDecStages && !mbar_wait_bounded(&empty[st], (uint32_t)(t / kDecStages - 1) & 1u)) {
                atomicOr(err, ERR_TIMEOUT);
                break;  // the summing warp stopped
            }
            float *dst = ring + (size_t)st * kDecTile * kDecSw;
            const int p0 = t * kDecTile, np = min(kDecTile, count - p0);
            for (int c = lt; c < np * chunks; c += kDecLoaders) {
                const int p = c / chunks, j = c - p * chunks;
                cp_async16(dst + p * kDecSw + 4 * j, vc + vo + (size_t)win_pos(w, p0 + p) * kv_dim + 4 * j);
            }
            cp_async_arrive_noinc(&full[st]);
        }
        cp_async_wait<0>();  // nothing in flight when the CTA ends
        return;
    }
    // warp 0
    float sum = 0.0f;
    if (lane == 0) sum = seq_sum_smem(sc, count);
    sum = __shfl_sync(kFullMask, sum, 0);
    float *ag = att + (size_t)rh * seq_len;
    float o = 0.0f;
    for (int t = 0; t < ntiles; ++t) {
        const int st = t % kDecStages;
        if (!__all_sync(kFullMask, mbar_wait_bounded(&full[st], (uint32_t)(t / kDecStages) & 1u))) {
            if (lane == 0) atomicOr(err, ERR_TIMEOUT);
            return;
        }
        const int p0 = t * kDecTile, np = min(kDecTile, count - p0);
        if (np == kDecTile) {
            // the tile's kDecTile / 32 quotients of a lane are independent:
            // loaded, divided and stored side by side
            float a[kDecTile / 32];
#pragma unroll
            for (int j = 0; j < kDecTile / 32; ++j) a[j] = sc[p0 + lane + 32 * j];
#pragma unroll
            for (int j = 0; j < kDecTile / 32; ++j) a[j] = __fdiv_rn(a[j], sum);
#pragma unroll
            for (int j = 0; j < kDecTile / 32; ++j) {
                sc[p0 + lane + 32 * j] = a[j];
                if (sl == 0) ag[p0 + lane + 32 * j] = a[j];
            }
        } else {
            for (int i = lane; i < np; i += 32) {
                const float a = __fdiv_rn(sc[p0 + i], sum);
                sc[p0 + i] = a;
                if (sl == 0) ag[p0 + i] = a;
            }
        }
        __syncwarp();
        const float *tl = ring + (size_t)st * kDecTile * kDecSw;
        const float *as = sc + p0;
        if (lane < ne) {
            int p = 0;
            if (np >= 16 && ((uintptr_t)as & 15) == 0) {
                float4 a4[4];
                float v[16];
#pragma unroll
                for (int j = 0; j < 4; ++j) a4[j] = *reinterpret_cast<const float4 *>(as + 4 * j);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = tl[j * kDecSw + lane];
                for (; p + 16 <= np; p += 16) {
                    const int pn = p + 32 <= np ? p + 16 : p;  // the next full step, or this one again
                    float4 na[4];
                    float nv[16];
#pragma unroll
                    for (int j = 0; j < 4; ++j) na[j] = *reinterpret_cast<const float4 *>(as + pn + 4 * j);
#pragma unroll
                    for (int j = 0; j < 16; ++j) nv[j] = tl[(pn + j) * kDecSw + lane];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        o = add_rn(o, mul_rn(a4[j].x, v[4 * j]));
                        o = add_rn(o, mul_rn(a4[j].y, v[4 * j + 1]));
                        o = add_rn(o, mul_rn(a4[j].z, v[4 * j + 2]));
                        o = add_rn(o, mul_rn(a4[j].w, v[4 * j + 3]));
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) a4[j] = na[j];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = nv[j];
                }
            }
            for (; p < np; ++p) o = add_rn(o, mul_rn(as[p], tl[p * kDecSw + lane]));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (lane < ne) out[(size_t)rh * head_size + e0 + lane] = o;
}

// ---- attention in tolerance mode ------------------------------------------------
// The reference's softmax sum and output elements are chains over the window
// (reference.rs:448-480); in tolerance mode (kernrt_cuda_set_exact(ctx, 0))
// the window is cut into chunks of kTolChunk positions summed in parallel
// (64: a decode row at position 511 spreads over 8 chunks per head).
// Pass 1, per (row, head, chunk): the scores (fused multiply-adds), the
// chunk's maximum m, its sum l of exp(s - m) by a block reduction, and its
// partial output o[e] = sum of exp(s_i - m) v_i[e]; the raw scores go to att.
// Pass 2, per (row, head): M = max m, L = sum of l exp(m - M), out = sum of o
// exp(m - M) / L, att[i] = exp(s_i - M) / L.
constexpr int kTolChunk = 64;

__device__ __forceinline__ float block_reduce128(float v, bool is_max, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(kFullMask, v, o);
        v = is_max ? fmaxf(v, t) : v + t;
    }
    __syncthreads();  // red is free
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    return is_max ? fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])) : (red[0] + red[1]) + (red[2] + red[3]);
}

__global__ void __launch_bounds__(128) k_att_tol_part(const float *__restrict__ q, float *__restrict__ att,
                                                      float *__restrict__ part, const float *__restrict__ kc,
                                                      const float *__restrict__ vc, const int32_t *__restrict__ win,
                                                      int n_heads, int kv_mul, int head_size, int kv_dim,
                                                      int seq_len, size_t loff, int nch) {
    extern __shared__ __align__(16) float tsm[];
    const int rh = blockIdx.x, row = rh / n_heads, h = rh - row * n_heads, c = blockIdx.y, tid = threadIdx.x;
    const int32_t *w = win + 4 * row;
    const int count = (w[3] - w[2]) + w[1] - w[0] + 1, i0 = c * kTolChunk;
    if (i0 >= count) return;
    const int np = min(kTolChunk, count - i0), hs4 = (head_size + 3) & ~3;
    float *qh = tsm, *p = tsm + hs4, *acc = p + kTolChunk;  // acc: [128]
    __shared__ float red[4];
    const float *qg = q + (size_t)rh * head_size;
    for (int e = tid; e < head_size; e += 128) qh[e] = qg[e];
    __syncthreads();
    const size_t kv = loff + (size_t)(h / kv_mul) * head_size;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)head_size));
    float m = -INFINITY;
    for (int i = tid; i < np; i += 128) {
        const float *kr = kc + kv + (size_t)win_pos(w, i0 + i) * kv_dim;
        float d = 0.0f;
        if ((head_size & 3) == 0 && ((uintptr_t)kr & 15) == 0) {
            // eight float4 of the key in flight, then their products
            for (int e0 = 0; e0 < head_size; e0 += 32) {
                float4 k4[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (e0 + 4 * j < head_size) k4[j] = __ldg(reinterpret_cast<const float4 *>(kr + e0) + j);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (e0 + 4 * j >= head_size) break;
                    const float4 q4 = *reinterpret_cast<const float4 *>(qh + e0 + 4 * j);
                    d = __fmaf_rn(q4.x, k4[j].x, d);
                    d = __fmaf_rn(q4.y, k4[j].y, d);
                    d = __fmaf_rn(q4.z, k4[j].z, d);
                    d = __fmaf_rn(q4.w, k4[j].w, d);
                }
            }
        } else {
            for (int e = 0; e < head_size; ++e) d = __fmaf_rn(qh[e], __ldg(kr + e), d);
        }
        const float sc = d * scale;
        p[i] = sc;
        att[(size_t)rh * seq_len + i0 + i] = sc;
        m = fmaxf(m, sc);  // NaN scores skipped, as the reference's `>` does
    }
    m = block_reduce128(m, true, red);
    float l = 0.0f;
    for (int i = tid; i < np; i += 128) {
        const float e = expf(p[i] - m);
        p[i] = e;
        l += e;
    }
    l = block_reduce128(l, false, red);  // its barriers also publish p
    // partial output: thread t takes element t % hs of positions t / hs, t / hs
    // + G, ... (G = 128 / hs groups when hs <= 128), the groups then added
    float *pg = part + ((size_t)rh * nch + c) * (2 + head_size);
    if (head_size <= 128) {
        const int G = 128 / head_size, e = tid % head_size, gi = tid / head_size;
        float o = 0.0f;
        if (gi < G) {
            int i = gi;
            for (; i + 7 * G < np; i += 8 * G) {  // eight value rows in flight
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldg(vc + kv + (size_t)win_pos(w, i0 + i + j * G) * kv_dim + e);
#pragma unroll
                for (int j = 0; j < 8; ++j) o = __fmaf_rn(p[i + j * G], v[j], o);
            }
            for (; i < np; i += G) o = __fmaf_rn(p[i], __ldg(vc + kv + (size_t)win_pos(w, i0 + i) * kv_dim + e), o);
        }
        acc[tid] = o;
        __syncthreads();
        if (tid < head_size) {
            float t = 0.0f;
            for (int g2 = 0; g2 < G; ++g2) t += acc[g2 * head_size + tid];
            pg[2 + tid] = t;
        }
    } else {
        for (int e = tid; e < head_size; e += 128) {
            float o = 0.0f;
            int i = 0;
            for (; i + 8 <= np; i += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldg(vc + kv + (size_t)win_pos(w, i0 + i + j) * kv_dim + e);
#pragma unroll
                for (int j = 0; j < 8; ++j) o = __fmaf_rn(p[i + j], v[j], o);
            }
            for (; i < np; ++i) o = __fmaf_rn(p[i], __ldg(vc + kv + (size_t)win_pos(w, i0 + i) * kv_dim + e), o);
            pg[2 + e] = o;
        }
    }
    if (tid == 0) {
        pg[0] = m;
        pg[1] = l;
    }
}

__global__ void __launch_bounds__(128) k_att_tol_combine(float *__restrict__ out, float *__restrict__ att,
                                                         const float *__restrict__ part,
                                                         const int32_t *__restrict__ win, int n_heads, int head_size,
                                                         int seq_len, int nch) {
    extern __shared__ __align__(16) float csm[];  // [nch] maxima, then [nch] scales
    const int rh = blockIdx.x, row = rh / n_heads, tid = threadIdx.x;
    const int32_t *w = win + 4 * row;
    const int count = (w[3] - w[2]) + w[1] - w[0] + 1;
    const int nc = (count + kTolChunk - 1) / kTolChunk, stride = 2 + head_size;
    const float *pr = part + (size_t)rh * nch * stride;
    float *cm = csm, *cf = csm + nch;
    __shared__ float red[4];
    // the chunks' maxima and sums, loaded side by side
    float m = -INFINITY;
    for (int c = tid; c < nc; c += 128) {
        cm[c] = pr[(size_t)c * stride];
        m = fmaxf(m, cm[c]);
    }
    const float M = block_reduce128(m, true, red);
    float l = 0.0f;
    for (int c = tid; c < nc; c += 128) {
        const float f = expf(cm[c] - M);
        cf[c] = f;
        l += pr[(size_t)c * stride + 1] * f;
    }
    const float inv = 1.0f / block_reduce128(l, false, red);  // its barriers also publish cf
    for (int e = tid; e < head_size; e += 128) {
        float o = 0.0f;
        int c = 0;
        for (; c + 8 <= nc; c += 8) {  // eight chunks' partials in flight
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = pr[(size_t)(c + j) * stride + 2 + e];
#pragma unroll
            for (int j = 0; j < 8; ++j) o = __fmaf_rn(v[j], cf[c + j], o);
        }
        for (; c < nc; ++c) o = __fmaf_rn(pr[(size_t)c * stride + 2 + e], cf[c], o);
        out[(size_t)rh * head_size + e] = o * inv;
    }
    float *ar = att + (size_t)rh * seq_len;
    for (int i = tid; i < count; i += 128) ar[i] = expf(ar[i] - M) * inv;
}

}  // namespace

cudaError_t launch_project(int src, const void *w, const float *wsc, int out_dim, int in_dim, const float *x,
                           int rows, float *y, int *err, cudaStream_t s) {
    if (rows <= 0 || out_dim <= 0) return cudaSuccess;
    switch (src) {
    case SRC_BF16: return project_src<SRC_BF16>(w, wsc, out_dim, in_dim, x, rows, y, err, s);
    case SRC_Q8: return project_src<SRC_Q8>(w, wsc, out_dim, in_dim, x, rows, y, err, s);
    default: return project_src<SRC_F32>(w, wsc, out_dim, in_dim, x, rows, y, err, s);
    }
}

cudaError_t launch_project_set(int src, int n, const void *const *w, const float *const *wsc, const int *out_dim,
                               int in_dim, const float *x, int rows, float *const *y, int *err, cudaStream_t s) {
    if (rows <= 0 || n <= 0) return cudaSuccess;
    bool one = n <= 3 && rows <= 4;
    for (int i = 0; one && i < n; ++i) {
        switch (src) {
        case SRC_BF16: one = gemv_fits<SRC_BF16>(w[i], wsc[i], in_dim, x, rows); break;
        case SRC_Q8: one = gemv_fits<SRC_Q8>(w[i], wsc[i], in_dim, x, rows); break;
        default: one = gemv_fits<SRC_F32>(w[i], wsc[i], in_dim, x, rows); break;
        }
    }
    if (!one) {  // one projection after another
        for (int i = 0; i < n; ++i) {
            const cudaError_t e = launch_project(src, w[i], wsc[i], out_dim[i], in_dim, x, rows, y[i], err, s);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    GemvSet set{};
    int ctas = 0;
    for (int i = 0; i < n; ++i) {
        set.w[i] = w[i];
        set.wsc[i] = wsc[i];
        set.y[i] = y[i];
        set.out_dim[i] = out_dim[i];
        ctas += (out_dim[i] + 31) / 32;
        set.cta_end[i] = ctas;
    }
    set.n = n;
    switch (src) {
    case SRC_BF16: return gemv_rows<SRC_BF16>(set, in_dim, x, rows, err, s);
    case SRC_Q8: return gemv_rows<SRC_Q8>(set, in_dim, x, rows, err, s);
    default: return gemv_rows<SRC_F32>(set, in_dim, x, rows, err, s);
    }
}

cudaError_t launch_kv_write(float *kc, float *vc, int kv_dim, const int32_t *dst_rows, const float *k, const float *v,
                            int rows, cudaStream_t s) {
    if (rows <= 0 || kv_dim <= 0) return cudaSuccess;
    const long long n = (long long)rows * kv_dim;
    if ((kv_dim & 3) == 0 && ((((uintptr_t)kc) | ((uintptr_t)vc) | ((uintptr_t)k) | ((uintptr_t)v)) & 15) == 0 &&
        n / 4 < (1ll << 31)) {
        const int n4 = (int)(n / 4);
        const int grid = (n4 + 255) / 256 < 148 * 16 ? (n4 + 255) / 256 : 148 * 16;
        k_kv_write4<<<(unsigned)grid, 256, 0, s>>>(kc, vc, kv_dim >> 2, dst_rows, k, v, n4);
        return launched();
    }
    long long grid = (n + 255) / 256;
    if (grid > 148 * 16) grid = 148 * 16;
    k_kv_write<<<(unsigned)grid, 256, 0, s>>>(kc, vc, kv_dim, dst_rows, k, v, rows);
    return launched();
}

size_t attention_smem_bytes(int head_size, int max_count) {
    return (size_t)(((head_size + 3) & ~3) + max_count) * sizeof(float);
}

size_t attention_scratch_floats(int n_rows, int n_heads, int max_count) {
    return (size_t)n_rows * n_heads * (size_t)((max_count + 3) & ~3);
}

cudaError_t launch_attention(const float *q, float *out, float *att, const float *kc, const float *vc,
                             const int32_t *win, int n_rows, int n_heads, int kv_mul, int head_size, int kv_dim,
                             int seq_len, size_t loff, int max_count, float *raw, bool shared_map, int *err,
                             cudaStream_t s) {
    if (n_rows <= 0 || n_heads <= 0) return cudaSuccess;
    // Two kernels where the value slices move in 16-byte pieces and a scratch
    // for the raw scores is given: parallel scores, then per (row, head,
    // slice) the softmax and the output chains with the value rows streamed.
    const int stride = (max_count + 3) & ~3;
    // Few (row, head) pairs (decode): slices of 32 elements and twelve stages
    // spread a long window's value rows over more SMs and keep ~90 KB of them
    // in flight per CTA.  Many pairs (prefill) fill the GPU by themselves: one
    // slice per head, three stages, several CTAs per SM.
    const bool few = n_rows * n_heads < 2 * 148;
    const int stages = few ? 12 : 3;
    const size_t out_smem = (size_t)(stride + stages * kAttTileFloats) * sizeof(float);
    const bool split = raw && (head_size & 3) == 0 && (kv_dim & 3) == 0 && out_smem <= 200 * 1024;
    if (split) {
        // rows that map positions alike share their key tiles (16 rows x 64 positions per CTA)
        const size_t rows_smem = (size_t)(kScPos + kScRows) * (head_size + 4) * sizeof(float);
        if (shared_map && n_rows >= 2 && rows_smem <= 48 * 1024 && (((uintptr_t)q | (uintptr_t)kc) & 15) == 0) {
            k_att_scores_rows<<<dim3((unsigned)((n_rows + kScRows - 1) / kScRows),
                                     (unsigned)((max_count + kScPos - 1) / kScPos), (unsigned)n_heads),
                                128, rows_smem, s>>>(q, raw, kc, win, n_rows, n_heads, kv_mul, head_size, kv_dim,
                                                     stride, loff);
        } else {
            k_att_scores<<<dim3((unsigned)(n_rows * n_heads), (unsigned)((max_count + 127) / 128)), 128,
                           (size_t)head_size * sizeof(float), s>>>(q, raw, kc, win, n_heads, kv_mul, head_size,
                                                                   kv_dim, stride, loff);
        }
        cudaError_t e = launched();
        if (e != cudaSuccess) return e;
        const size_t dec_smem = (size_t)(stride + kDecStages * kDecTile * kDecSw) * sizeof(float);
        if (few && err && dec_smem <= 200 * 1024) {
            e = cudaFuncSetAttribute(k_att_out_dec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec_smem);
            if (e != cudaSuccess) return e;
            const int nsl = (head_size + kDecSw - 1) / kDecSw;
            k_att_out_dec<<<(unsigned)(n_rows * n_heads * nsl), 128, dec_smem, s>>>(
                out, att, raw, vc, win, n_heads, kv_mul, head_size, kv_dim, seq_len, loff, stride, err);
            return launched();
        }
        const int sw = few ? 32 : (head_size > 128 ? 128 : head_size);
        const int nsl = (head_size + sw - 1) / sw;
        auto kern = few ? k_att_out<12> : k_att_out<3>;
        if (out_smem > 48 * 1024) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)out_smem);
            if (e != cudaSuccess) return e;
        }
        kern<<<(unsigned)(n_rows * n_heads * nsl), 128, out_smem, s>>>(out, att, raw, vc, win, n_heads, kv_mul,
                                                                       head_size, kv_dim, seq_len, loff, stride, sw);
        return launched();
    }
    const size_t smem = attention_smem_bytes(head_size, max_count);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    k_attention<<<(unsigned)(n_rows * n_heads), 128, smem, s>>>(q, out, att, kc, vc, win, n_heads, kv_mul, head_size,
                                                                kv_dim, seq_len, loff);
    return launched();
}

size_t attention_tol_scratch_floats(int n_rows, int n_heads, int head_size, int max_count) {
    const int nch = (max_count + kTolChunk - 1) / kTolChunk;
    return (size_t)n_rows * n_heads * nch * (2 + head_size);
}

cudaError_t launch_attention_tol(const float *q, float *out, float *att, const float *kc, const float *vc,
                                 const int32_t *win, int n_rows, int n_heads, int kv_mul, int head_size, int kv_dim,
                                 int seq_len, size_t loff, int max_count, float *part, cudaStream_t s) {
    if (n_rows <= 0 || n_heads <= 0) return cudaSuccess;
    const int nch = (max_count + kTolChunk - 1) / kTolChunk;
    const size_t smem = (size_t)(((head_size + 3) & ~3) + kTolChunk + 128) * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(k_att_tol_part, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    k_att_tol_part<<<dim3((unsigned)(n_rows * n_heads), (unsigned)nch), 128, smem, s>>>(
        q, att, part, kc, vc, win, n_heads, kv_mul, head_size, kv_dim, seq_len, loff, nch);
    cudaError_t e = launched();
    if (e != cudaSuccess) return e;
    k_att_tol_combine<<<(unsigned)(n_rows * n_heads), 128, (size_t)2 * nch * sizeof(float), s>>>(
        out, att, part, win, n_heads, head_size, seq_len, nch);
    return launched();
}

}  // namespace krt
