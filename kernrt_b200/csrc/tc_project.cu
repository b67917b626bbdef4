// Tensor-core projections for the tolerance mode: y[r, o] = sum_k W[o, k] x[r, k]
// with W bf16 [out_dim, in_dim] (Backend::project, mod.rs:318) on the sm_100a
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
// The reference's dot (reference.rs:73-79) is one f32 accumulator left to
// right; tensor cores cannot reproduce that order, so this path is opt-in and
// held to a tolerance instead of bit parity.  Activations are f32; both
// operands of one kind::f16 MMA must be the same 16-bit type, so x is split as
// x = hi + lo with hi = bf16(x) and lo = bf16(x - hi) (x - hi is exact in f32:
// hi is within a factor 2 of x).  Both halves are multiplied by the bf16
// weights (each product exact in f32) into one f32 accumulator, keeping ~16
// bits of each activation's mantissa: a relative error near 2^-17 per term
// plus the accumulation's rounding, against the 2^-9 of rounding x to bf16.
//
// x is split once per call by k_split_bf16 (x f32 -> hi, lo bf16 [rows,
// in_dim], also shared by the matrices of a project_qkv / project_gate_up).
// One CTA computes a tile of 128 outputs x 128 rows over the whole K in
// stages of 64 (one 128-byte swizzled row of bf16 per matrix row), four 48 KB
// stages in flight.  The stage's hi and lo tiles sit back to back with the
// same 1 KB group stride, so they are one 256-row B operand: one MMA per K-step
// (M = 128, N = 256) gives W.hi in accumulator columns 0-127 and W.lo in
// 128-255, reading the W slice once.  The kernel is bound by the operand bytes
// it pulls through L2: 128 rows a tile carry 48 KB of operands per 64-wide
// K-step for twice the MMA work of 64 rows (32 KB), and measured 1.5-1.7x
// faster where the grid still fills the SMs (4096 x 8192 x 2048: 419 -> 249
// us; 512 x 8192 x 2048: 65 -> 41 us), the same where it does not (512 x 2048
// x 2048: 64 tiles, 22.4 -> 22.7 us):
//   warp 0   one thread issues the TMA copies of stage kb: the W tile (128 x 64)
//            and the hi and lo tiles (128 x 64), all 128-byte swizzled,
//            counted on full[s];
//   warp 1   allocates the 256 TMEM columns, and one thread issues the MMAs:
//            per stage 4 K-steps of 16, then tcgen05.commit frees the stage
//            (empty[s]); a last commit signals `done`;
//   warps 2-5 read the accumulator (tcgen05.ld, warp w owns TMEM lanes
//            32 (w % 4) ..), add the hi and lo columns of each row, and store
//            y: for each row a warp writes 32 consecutive outputs.
// Also measured on B200 (64-row tiles, 512 x 2048 x 2048, split included): two
// N = 64 MMAs per K-step, each reading the W slice, 24.8 us; four stages
// instead of six 25.5 us; the split done in the kernel, by four or eight
// converting warps writing the swizzled hi / lo tiles in place of a TMA-loaded
// f32 tile, 32.9 / 30.9 us; the stage's copies issued by three lanes, 24.9 us.
// The TMA tensor maps cover this GPU's memory only, with no cluster multicast.
// Every mbarrier wait is bounded: a wait that runs out sets ERR_TIMEOUT in the
// error word, the roles stop, the producer waits (bounded) for the copies it
// still has in flight, and warp 1 waits for its MMAs before freeing TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "bulk.cuh"
#include "kernels.cuh"

namespace krt {

namespace {

constexpr int kTcM = 128;  // outputs per tile (MMA M)
constexpr int kTcN = 128;  // rows per tile (MMA N = 2 kTcN: their hi and lo halves)
constexpr int kTcK = 64;   // K per stage: 64 bf16 = one 128-byte swizzled row
constexpr int kTcStages = 4;
constexpr int kTcThreads = 192;
constexpr uint32_t kTileA = kTcM * kTcK * 2;      // 16 KB of W
constexpr uint32_t kTileB = kTcN * kTcK * 2;      // 16 KB: one of hi, lo
constexpr uint32_t kStage = kTileA + 2 * kTileB;  // 48 KB
constexpr size_t kTcSmem = (size_t)kTcStages * kStage + 1024;  // + slack to align the tiles to 1 KB
constexpr uint32_t kTmemCols = 2 * kTcN;  // f32 accumulator columns: W.hi, then W.lo (a power of 2, >= 32)

// Shared-memory matrix descriptor of a K-major tile stored as TMA's 128-byte
// swizzle writes it: rows of 128 bytes, 8-row groups 1 KB apart (the stride
// byte offset), tile 1 KB aligned (base offset 0), version 1 (bits 46-47),
// layout SWIZZLE_128B (bits 61-63 = 2).  The leading byte offset is unused for
// swizzled K-major tiles.  A K step of 16 bf16 inside the 128-byte row is the
// start address + 32 bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D f32 (bits 4-5 = 1), A and B bf16
// (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N / 8 at bits 17-22
// (N = 2 kTcN: the hi and lo rows), M / 16 at bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)((2 * kTcN) >> 3) << 17) |
                            ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every MMA this thread issued before it has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 consecutive accumulator columns of this warp's 32 TMEM lanes, one lane
// per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat16 a, __nv_bfloat16 b) {
    return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}

__device__ __forceinline__ void set_err_tc(int *err, int code) {
    if (err) atomicOr(err, code);
}

__global__ void __launch_bounds__(kTcThreads, 1)
    k_project_tc(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap thi,
                 const __grid_constant__ CUtensorMap tlo, int out_dim, int in_dim, int rows, float *__restrict__ y,
                 int *err) {
    extern __shared__ unsigned char tc_smem[];
    __shared__ uint64_t full[kTcStages], empty[kTcStages], done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort, s_issued, s_consumed;
    const uint32_t raw = smem_addr(tc_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1 KB aligned tiles (128-byte swizzle atoms)
    unsigned char *tiles = tc_smem + (base - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTcM, n0 = blockIdx.y * kTcN;
    const int nk = (in_dim + kTcK - 1) / kTcK;
    volatile int *abort_flag = &s_abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        s_abort = 0;
        s_issued = 0;
        s_consumed = 0;
        mbar_fence_init();
    }
    if (warp == 1) {  // the whole warp allocates
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kTcStages;
                if (kb >= kTcStages && !mbar_wait_bounded(&empty[s], (uint32_t)((kb / kTcStages) - 1) & 1u)) {
                    set_err_tc(err, ERR_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                unsigned char *st = tiles + (size_t)s * kStage;
                mbar_arrive_expect_tx(&full[s], kStage);
                tma_load_2d(st, &tw, kb * kTcK, m0, &full[s]);
                tma_load_2d(st + kTileA, &thi, kb * kTcK, n0, &full[s]);
                tma_load_2d(st + kTileA + kTileB, &tlo, kb * kTcK, n0, &full[s]);
                issued = kb + 1;
            }
            s_issued = issued;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kTcStages;
                if (*abort_flag || !mbar_wait_bounded(&full[s], (uint32_t)(kb / kTcStages) & 1u)) {
                    if (!*abort_flag) set_err_tc(err, ERR_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                s_consumed = kb + 1;
                tc_fence_after();
                const uint32_t a = base + (uint32_t)s * kStage, b = a + kTileA;  // b: hi rows, then lo rows
#pragma unroll
                for (int k = 0; k < kTcK / 16; ++k)
                    mma_bf16(tmem, sw128_desc(a + 32u * k), sw128_desc(b + 32u * k), (kb | k) != 0);
                mma_commit(&empty[s]);  // the stage's tiles are free once these MMAs are done
            }
            mma_commit(&done);  // every MMA issued, finished loop or not
        }
    } else {
        // warps 2-5: warp w reads TMEM lanes 32 (w % 4) .. + 31
        {
            const int q = warp & 3;
            const bool ok = mbar_wait_bounded(&done, 0);
            if (!ok) {
                if (lane == 0) set_err_tc(err, ERR_TIMEOUT);
                *abort_flag = 1;
            }
            tc_fence_after();
            // tcgen05.ld is warp-collective: the warp reads or skips as one
            if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
                const int o = m0 + 32 * q + lane;
#pragma unroll
                for (int c0 = 0; c0 < kTcN; c0 += 32) {
                    uint32_t vh[32], vl[32];
                    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
                    tmem_ld32(lane_base + (uint32_t)c0, vh);         // W.hi of rows n0 + c0 ..
                    tmem_ld32(lane_base + (uint32_t)(kTcN + c0), vl);  // W.lo of the same rows
                    if (o < out_dim) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int r = n0 + c0 + j;
                            if (r < rows)
                                y[(size_t)r * out_dim + o] = __fadd_rn(__uint_as_float(vh[j]), __uint_as_float(vl[j]));
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    // Teardown.  Copies issued but never waited for (only after a wait ran
    // out) must land before the shared memory goes; the MMAs must be done
    // before their TMEM is freed.
    if (warp == 0 && lane == 0)
        for (int kb = s_consumed; kb < s_issued; ++kb)
            mbar_wait_bounded(&full[kb % kTcStages], (uint32_t)(kb / kTcStages) & 1u);
    if (warp == 1) {
        mbar_wait_bounded(&done, 0);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// x f32 -> hi = bf16(x) and lo = bf16(x - hi), both round to nearest even;
// four elements per thread and step.
__global__ void __launch_bounds__(256) k_split_bf16(const float4 *__restrict__ x, uint2 *__restrict__ hi,
                                                    uint2 *__restrict__ lo, size_t n4) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = __ldcs(x + i);
        const __nv_bfloat16 h0 = __float2bfloat16_rn(v.x), h1 = __float2bfloat16_rn(v.y),
                            h2 = __float2bfloat16_rn(v.z), h3 = __float2bfloat16_rn(v.w);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(__fsub_rn(v.x, __bfloat162float(h0))),
                            l1 = __float2bfloat16_rn(__fsub_rn(v.y, __bfloat162float(h1))),
                            l2 = __float2bfloat16_rn(__fsub_rn(v.z, __bfloat162float(h2))),
                            l3 = __float2bfloat16_rn(__fsub_rn(v.w, __bfloat162float(h3)));
        hi[i] = make_uint2(bf16x2_bits(h0, h1), bf16x2_bits(h2, h3));
        lo[i] = make_uint2(bf16x2_bits(l0, l1), bf16x2_bits(l2, l3));
    }
}

// cuTensorMapEncodeTiled from the driver, found once through the runtime (the
// library links no libcuda).
using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;
EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// A 2-D bf16 tensor [outer, inner] (row stride inner * 2 bytes) in boxes of
// box_outer x 64, 128-byte swizzled; out-of-range elements read as zero.
bool bf16_map(CUtensorMap *m, const void *ptr, int inner, int outer, int box_outer) {
    EncodeTiled enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcK, (cuuint32_t)box_outer};
    const cuuint32_t elem[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tolerance mode, decode-sized calls (at most 4 rows, bf16 weights): the
// reference's dot (reference.rs:73-79) is one left-to-right chain per output,
// 2048 to 8192 dependent adds, which caps the exact kernels far below HBM.
// Here each output is one warp's: lane l takes 16-byte chunks l, l + 32, ...
// of the weight row (four in flight; eight, or two outputs per warp, measured
// slower), keeps a partial sum per row with fused
// multiply-adds, and the warp adds the 32 partials by shuffles, so the weights
// stream at HBM speed.  A set of up to three matrices over one x (q/k/v,
// gate/up) is one launch over their outputs end to end.
constexpr int kTolWarps = 8;
template <int R>
__global__ void __launch_bounds__(32 * kTolWarps) k_gemv_tol(TolGemvSet set, int in_dim, const float *__restrict__ x) {
    // x staged once per CTA when it fits (the warps' reads of it then come
    // from shared memory; measured 1.5 % faster over a decode token)
    extern __shared__ __align__(16) float xsm[];
    const bool sx = R * in_dim * 4 <= 48 * 1024;
    if (sx) {
        for (int i = threadIdx.x; i < R * in_dim / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(xsm)[i] = __ldg(reinterpret_cast<const float4 *>(x) + i);
        __syncthreads();
    }
    const float *xs = sx ? xsm : x;
    const int lane = threadIdx.x & 31;
    const int g = blockIdx.x * kTolWarps + (threadIdx.x >> 5);
    const int e0 = set.end[0], e1 = set.end[1], e2 = set.end[2];
    if (g >= (set.n == 1 ? e0 : set.n == 2 ? e1 : e2)) return;
    const int m = g < e0 ? 0 : (g < e1 ? 1 : 2);
    const int o = g - (m == 0 ? 0 : (m == 1 ? e0 : e1));
    const uint16_t *w = m == 0 ? set.w[0] : (m == 1 ? set.w[1] : set.w[2]);
    float *y = m == 0 ? set.y[0] : (m == 1 ? set.y[1] : set.y[2]);
    const int out_dim = m == 0 ? set.out_dim[0] : (m == 1 ? set.out_dim[1] : set.out_dim[2]);
    const uint4 *wr = reinterpret_cast<const uint4 *>(w + (size_t)o * in_dim);
    const int n8 = in_dim >> 3;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    auto step = [&](int c, uint4 u) {
        const float wv[8] = {__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                             __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u),
                             __uint_as_float(u.z << 16), __uint_as_float(u.z & 0xffff0000u),
                             __uint_as_float(u.w << 16), __uint_as_float(u.w & 0xffff0000u)};
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float4 a = reinterpret_cast<const float4 *>(xs + (size_t)r * in_dim)[2 * c];
            const float4 b = reinterpret_cast<const float4 *>(xs + (size_t)r * in_dim)[2 * c + 1];
            float t = acc[r];
            t = __fmaf_rn(wv[0], a.x, t); t = __fmaf_rn(wv[1], a.y, t);
            t = __fmaf_rn(wv[2], a.z, t); t = __fmaf_rn(wv[3], a.w, t);
            t = __fmaf_rn(wv[4], b.x, t); t = __fmaf_rn(wv[5], b.y, t);
            t = __fmaf_rn(wv[6], b.z, t); t = __fmaf_rn(wv[7], b.w, t);
            acc[r] = t;
        }
    };
    int c = lane;
    for (; c + 96 < n8; c += 128) {  // four chunks in flight
        const uint4 u0 = __ldcs(wr + c), u1 = __ldcs(wr + c + 32), u2 = __ldcs(wr + c + 64), u3 = __ldcs(wr + c + 96);
        step(c, u0);
        step(c + 32, u1);
        step(c + 64, u2);
        step(c + 96, u3);
    }
    for (; c < n8; c += 32) step(c, __ldcs(wr + c));
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], d);
    if (lane == 0)
#pragma unroll
        for (int r = 0; r < R; ++r) y[(size_t)r * out_dim + o] = acc[r];
}

}  // namespace

bool project_tc_supported(int out_dim, int in_dim, const void *w, const float *x, const float *y) {
    return out_dim > 0 && in_dim > 0 && in_dim % 8 == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0 &&
           ((uintptr_t)y & 3) == 0 && encode_fn() != nullptr;
}

cudaError_t launch_split_bf16(const float *x, uint16_t *hi, uint16_t *lo, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const size_t n4 = n / 4;  // n % 8 == 0 here (in_dim % 8 == 0)
    const size_t cap = (size_t)device_sms() * 8;
    const unsigned grid = (unsigned)((n4 + 255) / 256 < cap ? (n4 + 255) / 256 : cap);
    k_split_bf16<<<grid, 256, 0, s>>>(reinterpret_cast<const float4 *>(x), reinterpret_cast<uint2 *>(hi),
                                      reinterpret_cast<uint2 *>(lo), n4);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_project_tc(const uint16_t *w, int out_dim, int in_dim, const uint16_t *hi, const uint16_t *lo,
                              int rows, float *y, int *err, cudaStream_t s) {
    if (rows <= 0 || out_dim <= 0) return cudaSuccess;
    CUtensorMap tw, thi, tlo;
    if (!bf16_map(&tw, w, in_dim, out_dim, kTcM) || !bf16_map(&thi, hi, in_dim, rows, kTcN) ||
        !bf16_map(&tlo, lo, in_dim, rows, kTcN))
        return cudaErrorInvalidValue;
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_done[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(k_project_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
        if (e != cudaSuccess) return e;
        attr_done[dev] = true;
    }
    const dim3 grid((unsigned)((out_dim + kTcM - 1) / kTcM), (unsigned)((rows + kTcN - 1) / kTcN));
    k_project_tc<<<grid, kTcThreads, kTcSmem, s>>>(tw, thi, tlo, out_dim, in_dim, rows, y, err);
    count_launch();
    return cudaGetLastError();
}

bool gemv_tol_supported(const void *w, const float *x, int in_dim, int rows) {
    return rows >= 1 && rows <= 4 && in_dim > 0 && in_dim % 8 == 0 && ((uintptr_t)w & 15) == 0 &&
           ((uintptr_t)x & 15) == 0;
}

cudaError_t launch_gemv_tol(int n, const uint16_t *const *w, const int *out_dim, int in_dim, const float *x, int rows,
                            float *const *y, cudaStream_t s) {
    if (n < 1 || n > 3 || rows < 1 || rows > 4) return cudaErrorInvalidValue;
    TolGemvSet set{};
    int total = 0;
    for (int i = 0; i < 3; ++i) {
        if (i < n) {
            set.w[i] = w[i];
            set.y[i] = y[i];
            set.out_dim[i] = out_dim[i];
            total += out_dim[i];
        }
        set.end[i] = total;
    }
    set.n = n;
    if (total == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((total + kTolWarps - 1) / kTolWarps);
    const size_t xsb = (size_t)rows * in_dim * 4 <= 48 * 1024 ? (size_t)rows * in_dim * 4 : 0;  // x in shared memory
    switch (rows) {
    case 1: k_gemv_tol<1><<<grid, 32 * kTolWarps, xsb, s>>>(set, in_dim, x); break;
    case 2: k_gemv_tol<2><<<grid, 32 * kTolWarps, xsb, s>>>(set, in_dim, x); break;
    case 3: k_gemv_tol<3><<<grid, 32 * kTolWarps, xsb, s>>>(set, in_dim, x); break;
    default: k_gemv_tol<4><<<grid, 32 * kTolWarps, xsb, s>>>(set, in_dim, x); break;
    }
    count_launch();
    return cudaGetLastError();
}

}  // namespace krt
