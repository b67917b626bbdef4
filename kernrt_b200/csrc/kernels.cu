// sm_100a kernels for KernRT's per-row layer ops.
//
// Parity rules (the reference is KernRT's scalar backend,
// src/backends/reference.rs, whose arithmetic this file reproduces):
//   * every f32 operation that the reference performs is issued as one
//     separately rounded IEEE operation (__fmul_rn / __fadd_rn / __fsub_rn /
//     __fdiv_rn / __fsqrt_rn), so nvcc cannot contract it into an FMA;
//   * every reduction whose order is observable (the RMS sum of squares) runs
//     left to right in one thread, exactly as the reference loop;
//   * order-free reductions (the Q8 block amax: max is exact) use warp shuffles;
//   * RoPE reads cos/sin from a table the host built with the same libm calls
//     as the reference (powf, sinf, cosf), so only the rotation runs here;
//   * SwiGLU calls CUDA's expf: the one op held to a tolerance, not bit parity.
// No kernel asserts or traps: bad token ids / positions set a bit in a device
// error word that the host checks at its next barrier.
#include "kernels.cuh"
#include "bulk.cuh"
#include "q8_math.cuh"

#include <cuda_fp16.h>

#include <atomic>
#include <cstdlib>

namespace krt {

// Kernels this library has launched in this process (all devices).
static std::atomic<unsigned long long> g_kernel_launches{0};
void count_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }
unsigned long long kernel_launches() { return g_kernel_launches.load(std::memory_order_relaxed); }
// The launch status of the kernel just launched, counting it.
static cudaError_t launched() {
    count_launch();
    return cudaGetLastError();
}

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kThreads = 256;
// The norm pipeline runs one 16-warp CTA per SM: one summing warp, so the
// serial sums own an SM sub-partition's issue slots, and all of the SM's
// shared memory for its row slots.
constexpr int kPipeThreads = 512;

__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }

// dot.rs:222-224: a bf16 pattern is the top half of an f32.
__device__ __forceinline__ float bf16f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// reference.rs:171-173: ss /= n; ss += eps; scale = 1 / sqrt(ss).
__device__ __forceinline__ float rms_scale(float ss, float n, float eps) {
    ss = div_rn(ss, n);
    ss = add_rn(ss, eps);
    return div_rn(1.0f, __fsqrt_rn(ss));
}

// The exact-order sum of squares (reference.rs:167-170): ss + q(0) + q(1) + ...
// in that order, where sq16(b, q) computes the 16 squares of block b (elements
// 16b .. 16b + 15).  The squares of block b + 1 are computed before the adds
// of block b, so the dependent adds run back to back instead of each waiting
// on its own load and multiply.  Measured on B200, one lane per row out of
// shared memory: 7.26 cycles per element for a plain unrolled loop, 4.95 this
// way, 4.59 for the bare dependent add.
template <class Sq16>
__device__ __forceinline__ float chain_add16(float ss, int n16, Sq16 sq16) {
    if (n16 <= 0) return ss;
    float cur[16], nxt[16];
    sq16(0, cur);
    for (int b = 1; b < n16; ++b) {
        sq16(b, nxt);
#pragma unroll
        for (int e = 0; e < 16; ++e) ss = add_rn(ss, cur[e]);
#pragma unroll
        for (int e = 0; e < 16; ++e) cur[e] = nxt[e];
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) ss = add_rn(ss, cur[e]);
    return ss;
}

// The 16 squares of f32 values at p[0..16) (16-byte aligned).
__device__ __forceinline__ void squares16_f32(const float *p, float (&q)[16]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 v = reinterpret_cast<const float4 *>(p)[i];
        q[4 * i] = mul_rn(v.x, v.x);
        q[4 * i + 1] = mul_rn(v.y, v.y);
        q[4 * i + 2] = mul_rn(v.z, v.z);
        q[4 * i + 3] = mul_rn(v.w, v.w);
    }
}

// The 16 squares of bf16 patterns at p[0..16) (16-byte aligned).
__device__ __forceinline__ void squares16_bf16(const uint16_t *p, float (&q)[16]) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint4 u = reinterpret_cast<const uint4 *>(p)[i];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float lo = bf16f(w4[j] & 0xffffu), hi = bf16f(w4[j] >> 16);
            q[8 * i + 2 * j] = mul_rn(lo, lo);
            q[8 * i + 2 * j + 1] = mul_rn(hi, hi);
        }
    }
}

// quant.rs:722-758 is IEEE binary16 round-to-nearest-even; the block scale it
// converts is never NaN (the amax fold drops NaNs), and for every other input
// CUDA's RN conversion gives the same bits.
__device__ __forceinline__ uint16_t f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// The correctly rounded f32 quotient a / b, computed as a double division
// rounded to f32.  Rounding twice is harmless here: the double quotient carries
// 53 >= 2*24 + 2 bits, so rounding it to f32 gives the correctly rounded f32
// quotient (S. Figueroa, "When is double rounding innocuous?", SIGNUM
// Newsletter 30(3), 1995).  Unlike an f32 division, whose subnormal operands
// take a slow path, f32 values are never subnormal as doubles, so the cost does
// not depend on the data (in-place SwiGLU outputs drift toward subnormals when
// a step is repeated on its own output).
__device__ __forceinline__ float div_rn_exact(float a, float b) {
    return __double2float_rn(__ddiv_rn((double)a, (double)b));
}

// reference.rs:81-83 silu(g) * up.
__device__ __forceinline__ float silu_mul1(float g, float u) {
    return mul_rn(div_rn_exact(g, add_rn(1.0f, expf(-g))), u);
}

__device__ __forceinline__ void set_err(int *err, int code) {
    if (err) atomicOr(err, code);
}

// Streaming loads/stores for data touched once.
__device__ __forceinline__ float4 ld4(const float *p) { return __ldcs(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ void st4(float *p, float4 v) { __stcs(reinterpret_cast<float4 *>(p), v); }

// 256-bit loads and stores (sm_100): eight floats per lane in one
// instruction, a warp's 32 lanes one contiguous kilobyte.  p is 32-byte
// aligned.
__device__ __forceinline__ void ld8_stream(const float *p, float (&v)[8]) {
    asm("ld.global.cs.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
        : "l"(p));
}
__device__ __forceinline__ void ld8_ro(const float *p, float (&v)[8]) {
    asm("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
        : "l"(p));
}
__device__ __forceinline__ void st8_stream(float *p, const float (&v)[8]) {
    asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]),
                 "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                 : "memory");
}

// 16-byte global -> shared copies that need no registers: a warp issues all
// of a row's copies back to back and waits once.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// --------------------------------------------------------------------------
// Row-local building blocks (one warp per row)
// --------------------------------------------------------------------------

// reference.rs:180-207 qk_norm of one row, in place.  Lane h owns head h: its
// sum of squares runs left to right over the head in one thread, then the
// warp rescales the row with coalesced accesses.
__device__ void qk_norm_row_warp(float *v, int width, int head, const float *__restrict__ w,
                                 float eps, int lane) {
    const int nh = width / head;
    const bool vec = ((head | width) & 3) == 0;
    for (int h0 = 0; h0 < nh; h0 += 32) {
        const int h = h0 + lane;
        float scale = 0.0f;
        if (h < nh) {
            const float *p = v + h * head;
            float ss = 0.0f;
            if (vec) {
                for (int j = 0; j < head; j += 4) {
                    const float4 t = *reinterpret_cast<const float4 *>(p + j);
                    ss = add_rn(ss, mul_rn(t.x, t.x));
                    ss = add_rn(ss, mul_rn(t.y, t.y));
                    ss = add_rn(ss, mul_rn(t.z, t.z));
                    ss = add_rn(ss, mul_rn(t.w, t.w));
                }
            } else {
                for (int j = 0; j < head; ++j) ss = add_rn(ss, mul_rn(p[j], p[j]));
            }
            scale = rms_scale(ss, (float)head, eps);
        }
        __syncwarp();
        const int lo = h0 * head, hi = min(nh, h0 + 32) * head;
        if (vec) {
            for (int base = lo; base < hi; base += 128) {
                const int e = base + lane * 4;
                const bool ok = e < hi;
                const int hh = ok ? e / head - h0 : 0;
                const float sc = __shfl_sync(kFull, scale, hh);
                if (ok) {
                    float4 x = *reinterpret_cast<float4 *>(v + e);
                    const int j = e - (e / head) * head;
                    const float4 ww = __ldg(reinterpret_cast<const float4 *>(w + j));
                    x.x = mul_rn(ww.x, mul_rn(sc, x.x));
                    x.y = mul_rn(ww.y, mul_rn(sc, x.y));
                    x.z = mul_rn(ww.z, mul_rn(sc, x.z));
                    x.w = mul_rn(ww.w, mul_rn(sc, x.w));
                    *reinterpret_cast<float4 *>(v + e) = x;
                }
            }
        } else {
            for (int base = lo; base < hi; base += 32) {
                const int e = base + lane;
                const bool ok = e < hi;
                const int hh = ok ? e / head - h0 : 0;
                const float sc = __shfl_sync(kFull, scale, hh);
                if (ok) v[e] = mul_rn(w[e % head], mul_rn(sc, v[e]));
            }
        }
        __syncwarp();
    }
}

// reference.rs:239-254 half-split RoPE of `nh` heads of one row.
// ct/st: the table row of this row's position, `half` entries each.
// `lane` of `nl` cooperating threads (a warp, or several warps on one row).
__device__ void rope_half_row(float *v, int nh, int head, int half, const float *__restrict__ ct,
                              const float *__restrict__ st, bool vec, int lane, int nl = 32, float *dup = nullptr) {
    if (vec) {
        const int per = half >> 2, n = nh * per;
        for (int t = lane; t < n; t += nl) {
            const int h = t / per;
            const int j = (t - h * per) << 2;
            float *b = v + h * head;
            const float4 lo = *reinterpret_cast<const float4 *>(b + j);
            const float4 hi = *reinterpret_cast<const float4 *>(b + half + j);
            const float4 c = __ldg(reinterpret_cast<const float4 *>(ct + j));
            const float4 s = __ldg(reinterpret_cast<const float4 *>(st + j));
            float4 nl, nhv;
            nl.x = sub_rn(mul_rn(lo.x, c.x), mul_rn(hi.x, s.x));
            nl.y = sub_rn(mul_rn(lo.y, c.y), mul_rn(hi.y, s.y));
            nl.z = sub_rn(mul_rn(lo.z, c.z), mul_rn(hi.z, s.z));
            nl.w = sub_rn(mul_rn(lo.w, c.w), mul_rn(hi.w, s.w));
            nhv.x = add_rn(mul_rn(lo.x, s.x), mul_rn(hi.x, c.x));
            nhv.y = add_rn(mul_rn(lo.y, s.y), mul_rn(hi.y, c.y));
            nhv.z = add_rn(mul_rn(lo.z, s.z), mul_rn(hi.z, c.z));
            nhv.w = add_rn(mul_rn(lo.w, s.w), mul_rn(hi.w, c.w));
            *reinterpret_cast<float4 *>(b + j) = nl;
            *reinterpret_cast<float4 *>(b + half + j) = nhv;
            if (dup) {  // the rotated values to a second row as well (a cache row)
                *reinterpret_cast<float4 *>(dup + h * head + j) = nl;
                *reinterpret_cast<float4 *>(dup + h * head + half + j) = nhv;
            }
        }
    } else {
        const int n = nh * half;
        for (int t = lane; t < n; t += nl) {
            const int h = t / half, j = t - h * half;
            float *b = v + h * head;
            const float lo = b[j], hi = b[j + half], c = ct[j], s = st[j];
            const float a0 = sub_rn(mul_rn(lo, c), mul_rn(hi, s)), a1 = add_rn(mul_rn(lo, s), mul_rn(hi, c));
            b[j] = a0;
            b[j + half] = a1;
            if (dup) {
                dup[h * head + j] = a0;
                dup[h * head + j + half] = a1;
            }
        }
    }
}

// reference.rs:220-237 adjacent-pair RoPE over `npairs` pairs of one row;
// pair i uses the frequency of head_dim = (2*i) % head.
__device__ void rope_pair_row(float *v, int npairs, int head, const float *__restrict__ ct,
                              const float *__restrict__ st, bool vec, int lane, int nl = 32) {
    if (vec) {  // two pairs per float4; head % 4 == 0 keeps them in one head
        const int n = npairs >> 1;
        for (int t = lane; t < n; t += nl) {
            const int i = t << 2;
            const int j = (i % head) >> 1;
            float4 x = *reinterpret_cast<float4 *>(v + i);
            const float2 c = __ldg(reinterpret_cast<const float2 *>(ct + j));
            const float2 s = __ldg(reinterpret_cast<const float2 *>(st + j));
            const float x0 = x.x, x1 = x.y, x2 = x.z, x3 = x.w;
            x.x = sub_rn(mul_rn(x0, c.x), mul_rn(x1, s.x));
            x.y = add_rn(mul_rn(x0, s.x), mul_rn(x1, c.x));
            x.z = sub_rn(mul_rn(x2, c.y), mul_rn(x3, s.y));
            x.w = add_rn(mul_rn(x2, s.y), mul_rn(x3, c.y));
            *reinterpret_cast<float4 *>(v + i) = x;
        }
    } else {
        for (int p = lane; p < npairs; p += nl) {
            const int i = 2 * p;
            const int j = (i % head) >> 1;
            const float x0 = v[i], x1 = v[i + 1], c = ct[j], s = st[j];
            v[i] = sub_rn(mul_rn(x0, c), mul_rn(x1, s));
            v[i + 1] = add_rn(mul_rn(x0, s), mul_rn(x1, c));
        }
    }
}

// One row's q or k vector through qk_norm (w != null, reference.rs:180-207)
// and RoPE (mode 1 half-split, 2 adjacent pairs; reference.rs:209-257), staged
// in this warp's shared memory `sm`: the row is loaded once with 16-byte
// coalesced loads into head slots padded by 4 floats, lane h sums head h's
// squares left to right out of shared memory (bank-conflict free), then the
// warp normalises, rotates and stores the row with coalesced 16-byte stores.
// Covers the row's nh = width/head full heads; in pair mode the first
// `npairs` pairs are rotated (all of them when the row is whole heads).
// Requires head % 4 == 0 and width % 4 == 0.  sm holds nh*(head+4) + nh floats.
__device__ void qk_rope_row_smem(float *v, int width, int head, const float *__restrict__ w, float eps,
                                 const float *__restrict__ ct, const float *__restrict__ st, int mode, int npairs,
                                 float *sm, int lane) {
    const int nh = width / head;
    if (nh == 0) return;
    const int hs = head + 4, half = head >> 1;
    float *sc = sm + nh * hs;
    const int n4 = (nh * head) >> 2, per = head >> 2;
    for (int t = lane; t < n4; t += 32) {
        const int h = t / per, j = (t - h * per) << 2;
        cp_async16(sm + h * hs + j, v + 4 * t);
    }
    cp_async_wait_all();
    __syncwarp();
    if (w) {
        for (int h = lane; h < nh; h += 32) {
            const float *p = sm + h * hs;
            float ss = 0.0f;
            // the next four values are loaded ahead of the current four's adds
            float4 t4 = *reinterpret_cast<const float4 *>(p);
#pragma unroll 4
            for (int j = 0; j < head; j += 4) {
                const float4 n4v = *reinterpret_cast<const float4 *>(p + (j + 4 < head ? j + 4 : j));
                ss = add_rn(ss, mul_rn(t4.x, t4.x));
                ss = add_rn(ss, mul_rn(t4.y, t4.y));
                ss = add_rn(ss, mul_rn(t4.z, t4.z));
                ss = add_rn(ss, mul_rn(t4.w, t4.w));
                t4 = n4v;
            }
            sc[h] = rms_scale(ss, (float)head, eps);
        }
        __syncwarp();
    }
    auto norm4 = [&](float4 x, int h, int j) {
        if (!w) return x;
        const float s = sc[h];
        const float4 ww = __ldg(reinterpret_cast<const float4 *>(w + j));
        return make_float4(mul_rn(ww.x, mul_rn(s, x.x)), mul_rn(ww.y, mul_rn(s, x.y)), mul_rn(ww.z, mul_rn(s, x.z)),
                           mul_rn(ww.w, mul_rn(s, x.w)));
    };
    auto scale4 = [&](float4 x, float s, float4 ww) {
        return make_float4(mul_rn(ww.x, mul_rn(s, x.x)), mul_rn(ww.y, mul_rn(s, x.y)), mul_rn(ww.z, mul_rn(s, x.z)),
                           mul_rn(ww.w, mul_rn(s, x.w)));
    };
    auto rot_half = [&](float4 lo, float4 hi, float4 c, float4 s, float *dlo, float *dhi) {
        float4 nl, nhv;
        nl.x = sub_rn(mul_rn(lo.x, c.x), mul_rn(hi.x, s.x));
        nl.y = sub_rn(mul_rn(lo.y, c.y), mul_rn(hi.y, s.y));
        nl.z = sub_rn(mul_rn(lo.z, c.z), mul_rn(hi.z, s.z));
        nl.w = sub_rn(mul_rn(lo.w, c.w), mul_rn(hi.w, s.w));
        nhv.x = add_rn(mul_rn(lo.x, s.x), mul_rn(hi.x, c.x));
        nhv.y = add_rn(mul_rn(lo.y, s.y), mul_rn(hi.y, c.y));
        nhv.z = add_rn(mul_rn(lo.z, s.z), mul_rn(hi.z, c.z));
        nhv.w = add_rn(mul_rn(lo.w, s.w), mul_rn(hi.w, c.w));
        *reinterpret_cast<float4 *>(dlo) = nl;
        *reinterpret_cast<float4 *>(dhi) = nhv;
    };
    if (mode == 1) {
        const int ph = half >> 2;  // float4 items per head (lo half)
        if (32 % ph == 0) {
            // every item of a lane has the same column j: its weights and its
            // cos/sin are loaded once per row, not once per item
            const int j = (lane % ph) << 2, hstep = 32 / ph;
            const float4 c = __ldg(reinterpret_cast<const float4 *>(ct + j));
            const float4 sn = __ldg(reinterpret_cast<const float4 *>(st + j));
            float4 wl = make_float4(0.0f, 0.0f, 0.0f, 0.0f), wh = wl;
            if (w) {
                wl = __ldg(reinterpret_cast<const float4 *>(w + j));
                wh = __ldg(reinterpret_cast<const float4 *>(w + half + j));
            }
#pragma unroll 4
            for (int h = lane / ph; h < nh; h += hstep) {
                float4 lo = *reinterpret_cast<const float4 *>(sm + h * hs + j);
                float4 hi = *reinterpret_cast<const float4 *>(sm + h * hs + half + j);
                if (w) {
                    const float s1 = sc[h];
                    lo = scale4(lo, s1, wl);
                    hi = scale4(hi, s1, wh);
                }
                rot_half(lo, hi, c, sn, v + h * head + j, v + h * head + half + j);
            }
        } else {
            for (int t = lane; t < nh * ph; t += 32) {
                const int h = t / ph, j = (t - h * ph) << 2;
                const float4 lo = norm4(*reinterpret_cast<const float4 *>(sm + h * hs + j), h, j);
                const float4 hi = norm4(*reinterpret_cast<const float4 *>(sm + h * hs + half + j), h, half + j);
                const float4 c = __ldg(reinterpret_cast<const float4 *>(ct + j));
                const float4 sn = __ldg(reinterpret_cast<const float4 *>(st + j));
                rot_half(lo, hi, c, sn, v + h * head + j, v + h * head + half + j);
            }
        }
    } else {
        auto pair_rot = [&](float4 x, int t, float2 c, float2 sn) {
            if (mode == 2 && 2 * t < npairs) {
                const float x0 = x.x, x1 = x.y, x2 = x.z, x3 = x.w;
                x.x = sub_rn(mul_rn(x0, c.x), mul_rn(x1, sn.x));
                x.y = add_rn(mul_rn(x0, sn.x), mul_rn(x1, c.x));
                if (2 * t + 1 < npairs) {
                    x.z = sub_rn(mul_rn(x2, c.y), mul_rn(x3, sn.y));
                    x.w = add_rn(mul_rn(x2, sn.y), mul_rn(x3, c.y));
                }
            }
            return x;
        };
        if (32 % per == 0) {
            // a lane's items share the column j (see above)
            const int j = (lane % per) << 2, hstep = 32 / per;
            float2 c = make_float2(0.0f, 0.0f), sn = c;
            if (mode == 2) {
                c = __ldg(reinterpret_cast<const float2 *>(ct + (j >> 1)));
                sn = __ldg(reinterpret_cast<const float2 *>(st + (j >> 1)));
            }
            float4 ww = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (w) ww = __ldg(reinterpret_cast<const float4 *>(w + j));
#pragma unroll 4
            for (int h = lane / per; h < nh; h += hstep) {
                const int t = h * per + (lane % per);
                float4 x = *reinterpret_cast<const float4 *>(sm + h * hs + j);
                if (w) x = scale4(x, sc[h], ww);
                *reinterpret_cast<float4 *>(v + 4 * t) = pair_rot(x, t, c, sn);
            }
        } else {
            for (int t = lane; t < n4; t += 32) {
                const int h = t / per, j = (t - h * per) << 2;
                const float4 x = norm4(*reinterpret_cast<const float4 *>(sm + h * hs + j), h, j);
                float2 c = make_float2(0.0f, 0.0f), sn = c;
                if (mode == 2 && 2 * t < npairs) {
                    c = __ldg(reinterpret_cast<const float2 *>(ct + (j >> 1)));
                    sn = __ldg(reinterpret_cast<const float2 *>(st + (j >> 1)));
                }
                *reinterpret_cast<float4 *>(v + 4 * t) = pair_rot(x, t, c, sn);
            }
        }
    }
    __syncwarp();
}

// Floats of shared memory qk_rope_row_smem needs for a row of `width`.
__host__ __device__ __forceinline__ int qk_smem_floats(int width, int head) {
    const int nh = width / head;
    return ((nh * (head + 4) + nh) + 3) & ~3;
}

// Pairs of K rotated by the reference's interleaved loop: i < kv_width while
// i + 1 < q_width (reference.rs:221-236).
__device__ __forceinline__ int k_pairs_interleaved(int q_width, int kv_width) {
    return min(kv_width / 2, q_width / 2);
}

// reference.rs:395-400 silu_mul over [lo, hi) by threads t of nt.  Each
// thread keeps U independent float4 pairs in flight before using any of them:
// the loop is bound by HBM latency x bytes in flight, not by arithmetic.
template <int U>
__device__ void silu_range(float *__restrict__ g, const float *__restrict__ u, size_t lo, size_t hi,
                           int t, int nt) {
    if (((lo | hi) & 7) == 0 && !(((uintptr_t)g | (uintptr_t)u) & 31)) {
        // 256-bit accesses, the same bytes in flight as U float4 pairs:
        // measured on B200, silu_mul 1.053 -> 1.003 ms at 65 536 x 8192 and
        // the 65 536-row chain 1.739 -> 1.657 ms (twice the bytes in flight
        // was slower: 1.146 / 1.691 ms)
        constexpr int V = U >= 2 ? U / 2 : 1;
        const size_t step = 8 * (size_t)nt;
        size_t i = lo + 8 * (size_t)t;
        for (; i + (V - 1) * step < hi; i += V * step) {
            float gv[V][8], uv[V][8];
#pragma unroll
            for (int k = 0; k < V; ++k) {
                ld8_stream(g + i + k * step, gv[k]);
                ld8_stream(u + i + k * step, uv[k]);
            }
#pragma unroll
            for (int k = 0; k < V; ++k) {
#pragma unroll
                for (int e = 0; e < 8; ++e) gv[k][e] = silu_mul1(gv[k][e], uv[k][e]);
                st8_stream(g + i + k * step, gv[k]);
            }
        }
        for (; i < hi; i += step) {
            float gv[8], uv[8];
            ld8_stream(g + i, gv);
            ld8_stream(u + i, uv);
#pragma unroll
            for (int e = 0; e < 8; ++e) gv[e] = silu_mul1(gv[e], uv[e]);
            st8_stream(g + i, gv);
        }
        return;
    }
    if (((lo | hi) & 3) == 0) {
        const size_t step = 4 * (size_t)nt;
        size_t i = lo + 4 * (size_t)t;
        for (; i + (U - 1) * step < hi; i += U * step) {
            float4 gv[U], uv[U];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                gv[k] = ld4(g + i + k * step);
                uv[k] = ld4(u + i + k * step);
            }
#pragma unroll
            for (int k = 0; k < U; ++k) {
                gv[k].x = silu_mul1(gv[k].x, uv[k].x);
                gv[k].y = silu_mul1(gv[k].y, uv[k].y);
                gv[k].z = silu_mul1(gv[k].z, uv[k].z);
                gv[k].w = silu_mul1(gv[k].w, uv[k].w);
                st4(g + i + k * step, gv[k]);
            }
        }
        for (; i < hi; i += step) {
            float4 gv = ld4(g + i);
            const float4 uv = ld4(u + i);
            gv.x = silu_mul1(gv.x, uv.x);
            gv.y = silu_mul1(gv.y, uv.y);
            gv.z = silu_mul1(gv.z, uv.z);
            gv.w = silu_mul1(gv.w, uv.w);
            st4(g + i, gv);
        }
    } else {
        for (size_t i = lo + t; i < hi; i += nt) g[i] = silu_mul1(g[i], u[i]);
    }
}

// Half-split RoPE (reference.rs:239-254) over rows [r0, r0 + g) of a
// [rows, width] buffer as one flat range of float4 (lo, hi) pairs, U pairs in
// flight per thread.  Requires half % 4 == 0 and width % 4 == 0.
template <int U>
__device__ void rope_half_rows(float *v, int width, int head, int half, int r0, int g,
                               const int32_t *__restrict__ pos, const float *__restrict__ cos_t,
                               const float *__restrict__ sin_t, int max_pos, int *err, int t, int nt) {
    const int per = half >> 2;
    const int nh = width / head;
    const int per_row = nh * per;
    const int n = g * per_row;
    int i = t;
    for (; i < n; i += U * nt) {
        float4 lo[U], hi[U];
        float *b[U];
        int j[U], p[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int it = i + k * nt;
            b[k] = nullptr;
            if (it < n) {
                const int r = it / per_row;
                const int rem = it - r * per_row;
                const int h = rem / per;
                j[k] = (rem - h * per) << 2;
                p[k] = pos[r0 + r];
                b[k] = v + (size_t)(r0 + r) * width + h * head;
                lo[k] = *reinterpret_cast<const float4 *>(b[k] + j[k]);
                hi[k] = *reinterpret_cast<const float4 *>(b[k] + half + j[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            if (!b[k]) continue;
            if ((unsigned)p[k] >= (unsigned)max_pos) {
                set_err(err, ERR_POSITION);
                continue;
            }
            const float4 c = __ldg(reinterpret_cast<const float4 *>(cos_t + (size_t)p[k] * half + j[k]));
            const float4 s = __ldg(reinterpret_cast<const float4 *>(sin_t + (size_t)p[k] * half + j[k]));
            float4 nl, nhv;
            nl.x = sub_rn(mul_rn(lo[k].x, c.x), mul_rn(hi[k].x, s.x));
            nl.y = sub_rn(mul_rn(lo[k].y, c.y), mul_rn(hi[k].y, s.y));
            nl.z = sub_rn(mul_rn(lo[k].z, c.z), mul_rn(hi[k].z, s.z));
            nl.w = sub_rn(mul_rn(lo[k].w, c.w), mul_rn(hi[k].w, s.w));
            nhv.x = add_rn(mul_rn(lo[k].x, s.x), mul_rn(hi[k].x, c.x));
            nhv.y = add_rn(mul_rn(lo[k].y, s.y), mul_rn(hi[k].y, c.y));
            nhv.z = add_rn(mul_rn(lo[k].z, s.z), mul_rn(hi[k].z, c.z));
            nhv.w = add_rn(mul_rn(lo[k].w, s.w), mul_rn(hi[k].w, c.w));
            *reinterpret_cast<float4 *>(b[k] + j[k]) = nl;
            *reinterpret_cast<float4 *>(b[k] + half + j[k]) = nhv;
        }
    }
}

// --------------------------------------------------------------------------
// Embedding gather (reference.rs:133-140 -> quant.rs:659-693), one warp/row
// --------------------------------------------------------------------------

template <int KIND, bool VEC>
__global__ void __launch_bounds__(kThreads) k_embed_gather(GatherArgs a) {
    const int lane = threadIdx.x & 31;
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= a.n) return;
    const int tok = a.tokens[row];
    const int dim = a.dim;
    float *dst = a.dst + (a.dst_off ? a.dst_off[row] : (int64_t)row * dim);
    if ((unsigned)tok >= (unsigned)a.vocab) {
        if (lane == 0) set_err(a.err, ERR_TOKEN);
        for (int i = lane; i < dim; i += 32) dst[i] = 0.0f;
        return;
    }
    const size_t base = (size_t)tok * dim;
    if constexpr (KIND == SRC_BF16) {
        const uint16_t *src = static_cast<const uint16_t *>(a.table) + base;
        if constexpr (VEC) {
            for (int c = lane * 8; c < dim; c += 256) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src + c));
                const float4 lo = make_float4(bf16f(v.x & 0xffffu), bf16f(v.x >> 16),
                                              bf16f(v.y & 0xffffu), bf16f(v.y >> 16));
                const float4 hi = make_float4(bf16f(v.z & 0xffffu), bf16f(v.z >> 16),
                                              bf16f(v.w & 0xffffu), bf16f(v.w >> 16));
                *reinterpret_cast<float4 *>(dst + c) = lo;
                *reinterpret_cast<float4 *>(dst + c + 4) = hi;
            }
        } else {
            for (int i = lane; i < dim; i += 32) dst[i] = bf16f(src[i]);
        }
    } else if constexpr (KIND == SRC_Q8) {
        const int8_t *src = static_cast<const int8_t *>(a.table) + base;
        const float *sc = a.tscales + (size_t)tok * (dim / 32);
        if constexpr (VEC) {
            for (int c = lane * 16; c < dim; c += 512) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src + c));
                const float s = __ldg(sc + (c >> 5));
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t b = w4[q];
                    float4 o;
                    o.x = mul_rn((float)(int8_t)(b & 0xffu), s);
                    o.y = mul_rn((float)(int8_t)((b >> 8) & 0xffu), s);
                    o.z = mul_rn((float)(int8_t)((b >> 16) & 0xffu), s);
                    o.w = mul_rn((float)(int8_t)(b >> 24), s);
                    *reinterpret_cast<float4 *>(dst + c + 4 * q) = o;
                }
            }
        } else {
            for (int i = lane; i < dim; i += 32) dst[i] = mul_rn((float)src[i], sc[i >> 5]);
        }
    } else {
        const float *src = static_cast<const float *>(a.table) + base;
        if constexpr (VEC) {
            for (int c = lane * 4; c < dim; c += 128)
                *reinterpret_cast<float4 *>(dst + c) = __ldg(reinterpret_cast<const float4 *>(src + c));
        } else {
            for (int i = lane; i < dim; i += 32) dst[i] = src[i];
        }
    }
}

// --------------------------------------------------------------------------
// The fused row-group kernel
// --------------------------------------------------------------------------
//
// One CTA owns G consecutive token rows.  Stage 0 stages the rows being
// normalised (raw table bytes of the gathered embedding rows, or the f32 x
// rows) in shared memory with 16-byte loads.  Stage 1 splits the CTA: in warp
// 0, lane r runs row r's sum of squares left to right out of shared memory
// (the reference's exact order; row slots are padded by 16 bytes so the lanes'
// 16-byte reads are bank-conflict free) while warps 1.. stream the same rows'
// independent ops — qk_norm, RoPE, SwiGLU — from HBM.  Stage 2 writes the
// normalised rows and the residual sum from the staged copy, so every
// activation row crosses HBM once.

template <int SRC>
__device__ __forceinline__ int src_row_bytes(int dim) {
    return SRC == SRC_BF16 ? dim * 2 : (SRC == SRC_Q8 ? dim : dim * 4);
}

__host__ __device__ __forceinline__ int align16(int v) { return (v + 15) & ~15; }

// Decode n consecutive values of a staged row starting at column c.
template <int SRC, int N>
__device__ __forceinline__ void decode_staged(const unsigned char *row, int dim, int c, float *v) {
    if constexpr (SRC == SRC_BF16) {
        if constexpr (N == 8) {
            const uint4 t = *reinterpret_cast<const uint4 *>(row + 2 * c);
            v[0] = bf16f(t.x & 0xffffu); v[1] = bf16f(t.x >> 16);
            v[2] = bf16f(t.y & 0xffffu); v[3] = bf16f(t.y >> 16);
            v[4] = bf16f(t.z & 0xffffu); v[5] = bf16f(t.z >> 16);
            v[6] = bf16f(t.w & 0xffffu); v[7] = bf16f(t.w >> 16);
        } else if constexpr (N == 4) {
            const uint2 t = *reinterpret_cast<const uint2 *>(row + 2 * c);
            v[0] = bf16f(t.x & 0xffffu); v[1] = bf16f(t.x >> 16);
            v[2] = bf16f(t.y & 0xffffu); v[3] = bf16f(t.y >> 16);
        } else {
#pragma unroll
            for (int e = 0; e < N; ++e) v[e] = bf16f(reinterpret_cast<const uint16_t *>(row)[c + e]);
        }
    } else if constexpr (SRC == SRC_Q8) {
        // codes at row[0..dim), block scales at row + align16(dim); one
        // f32 multiply per value (quant.rs:686-688)
        const float *sc = reinterpret_cast<const float *>(row + align16(dim));
        if constexpr (N == 8 || N == 4) {
            const float s = sc[c >> 5];  // c % N == 0, so all N share a block
            if constexpr (N == 8) {
                const uint2 t = *reinterpret_cast<const uint2 *>(row + c);
                const uint32_t w2[2] = {t.x, t.y};
#pragma unroll
                for (int q = 0; q < 2; ++q)
#pragma unroll
                    for (int b = 0; b < 4; ++b)
                        v[4 * q + b] = mul_rn((float)(int8_t)((w2[q] >> (8 * b)) & 0xffu), s);
            } else {
                const uint32_t t = *reinterpret_cast<const uint32_t *>(row + c);
#pragma unroll
                for (int b = 0; b < 4; ++b) v[b] = mul_rn((float)(int8_t)((t >> (8 * b)) & 0xffu), s);
            }
        } else {
#pragma unroll
            for (int e = 0; e < N; ++e)
                v[e] = mul_rn((float)reinterpret_cast<const int8_t *>(row)[c + e], sc[(c + e) >> 5]);
        }
    } else {
        const float *f = reinterpret_cast<const float *>(row);
        if constexpr (N == 8) {
            const float4 t0 = *reinterpret_cast<const float4 *>(f + c);
            const float4 t1 = *reinterpret_cast<const float4 *>(f + c + 4);
            v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
            v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
        } else if constexpr (N == 4) {
            const float4 t0 = *reinterpret_cast<const float4 *>(f + c);
            v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
        } else {
#pragma unroll
            for (int e = 0; e < N; ++e) v[e] = f[c + e];
        }
    }
}

struct ChainLayout {
    int G;        // rows per CTA
    int xstride;  // bytes per staged source row slot
    int rstride;  // bytes per staged residual row slot (FQ with resid), else 0
    size_t smem;
};


template <int SRC, bool FQ, bool VEC>
__global__ void __launch_bounds__(kThreads, 3) k_chain(ChainArgs a, ChainLayout L) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int dim = a.dim;
    const int r0 = blockIdx.x * L.G;
    const int g = min(L.G, a.rows - r0);
    const bool fq_resid = FQ && a.resid != nullptr;
    unsigned char *xs = smem;
    unsigned char *rs = smem + (size_t)L.G * L.xstride;
    float *sc1 = reinterpret_cast<float *>(rs + (size_t)L.G * L.rstride);
    float *sc2 = sc1 + 32;

    auto src_row = [&](int r) -> const unsigned char * {
        if constexpr (SRC == SRC_X) {
            return reinterpret_cast<const unsigned char *>(a.x_in + (size_t)(r0 + r) * dim);
        } else {
            const int tok = a.tokens[r0 + r];
            if ((unsigned)tok >= (unsigned)a.vocab) return nullptr;
            return static_cast<const unsigned char *>(a.table) +
                   (size_t)tok * (size_t)src_row_bytes<SRC>(dim);
        }
    };

    if (warp == 0) {
        // ---- stage 0 (warp 0 alone): stage the rows being normalised, and for
        // the final norm the residual rows, into shared memory.  cp.async keeps
        // every copy in flight at once without a register round trip.
        const int rb = src_row_bytes<SRC>(dim);
        for (int r = 0; r < g; ++r) {
            const unsigned char *sp = src_row(r);
            unsigned char *dst = xs + (size_t)r * L.xstride;
            if (!sp && lane == 0) set_err(a.err, ERR_TOKEN);
            if constexpr (VEC) {
                for (int c = lane; c < (rb >> 4); c += 32) {
                    if (sp) cp_async16(dst + 16 * c, sp + 16 * c);
                    else *reinterpret_cast<uint4 *>(dst + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
                }
            } else {
                for (int c = lane; c < rb; c += 32) dst[c] = sp ? sp[c] : (unsigned char)0;
            }
            if constexpr (SRC == SRC_Q8) {
                const int nb = dim >> 5;
                const int tok = a.tokens[r0 + r];
                float *sdst = reinterpret_cast<float *>(dst + align16(dim));
                for (int b = lane; b < nb; b += 32) sdst[b] = sp ? __ldg(a.tscales + (size_t)tok * nb + b) : 0.0f;
            }
            if (fq_resid) {
                const float *rsrc = a.resid + (size_t)(r0 + r) * dim;
                float *rdst = reinterpret_cast<float *>(rs + (size_t)r * L.rstride);
                if constexpr (VEC) {
                    for (int c = lane; c < (dim >> 2); c += 32) cp_async16(rdst + 4 * c, rsrc + 4 * c);
                } else {
                    for (int c = lane; c < dim; c += 32) rdst[c] = rsrc[c];
                }
            }
        }
        if constexpr (VEC) cp_async_wait_all();
        __syncwarp();

        // ---- stage 1, warp 0: lane r sums row r's squares left to right
        // (reference.rs:167-170), out of shared memory.
        if (lane < g) {
            const unsigned char *row = xs + (size_t)lane * L.xstride;
            const float *rrow = reinterpret_cast<const float *>(rs + (size_t)lane * L.rstride);
            float ss = 0.0f, ss2 = 0.0f;
            if constexpr (VEC) {
                for (int c = 0; c < dim; c += 8) {
                    float v[8];
                    decode_staged<SRC, 8>(row, dim, c, v);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        ss = add_rn(ss, mul_rn(v[e], v[e]));
                        if constexpr (FQ) {
                            const float xo = fq_resid ? add_rn(v[e], rrow[c + e]) : v[e];
                            ss2 = add_rn(ss2, mul_rn(xo, xo));
                        }
                    }
                }
            } else {
                for (int c = 0; c < dim; ++c) {
                    float v[1];
                    decode_staged<SRC, 1>(row, dim, c, v);
                    ss = add_rn(ss, mul_rn(v[0], v[0]));
                    if constexpr (FQ) {
                        const float xo = fq_resid ? add_rn(v[0], rrow[c]) : v[0];
                        ss2 = add_rn(ss2, mul_rn(xo, xo));
                    }
                }
            }
            sc1[lane] = rms_scale(ss, (float)dim, a.eps);
            if constexpr (FQ) sc2[lane] = rms_scale(ss2, (float)dim, a.final_eps);
        }
    } else {
        // ---- stage 1, warps 1..: the rows' independent streams, from HBM.
        const int st = tid - 32, nst = blockDim.x - 32;
        const int sw = warp - 1, nsw = nwarps - 1;
        const bool half_vec = ((a.half | a.q_dim | a.kv_dim) & 3) == 0;
        if (a.rope_mode == 1 && half_vec && a.w_q == nullptr && a.w_k == nullptr) {
            if (a.q) rope_half_rows<2>(a.q, a.q_dim, a.head, a.half, r0, g, a.pos, a.cos_t, a.sin_t, a.max_pos,
                                       a.err, st, nst);
            if (a.k) rope_half_rows<2>(a.k, a.kv_dim, a.head, a.half, r0, g, a.pos, a.cos_t, a.sin_t, a.max_pos,
                                       a.err, st, nst);
        } else if (a.rope_mode != 0 || a.w_q != nullptr || a.w_k != nullptr) {
            const bool pair_vec = ((a.head | a.q_dim | a.kv_dim) & 3) == 0;
            for (int r = sw; r < g; r += nsw) {
                const int row = r0 + r;
                float *qr = a.q ? a.q + (size_t)row * a.q_dim : nullptr;
                float *kr = a.k ? a.k + (size_t)row * a.kv_dim : nullptr;
                if (a.w_q && qr) qk_norm_row_warp(qr, a.q_dim, a.head, a.w_q, a.eps, lane);
                if (a.w_k && kr) qk_norm_row_warp(kr, a.kv_dim, a.head, a.w_k, a.eps, lane);
                if (a.rope_mode == 0) continue;
                const int p = a.pos[row];
                if ((unsigned)p >= (unsigned)a.max_pos) {
                    if (lane == 0) set_err(a.err, ERR_POSITION);
                    continue;
                }
                const float *ct = a.cos_t + (size_t)p * a.half;
                const float *stt = a.sin_t + (size_t)p * a.half;
                if (a.rope_mode == 1) {
                    if (qr) rope_half_row(qr, a.q_dim / a.head, a.head, a.half, ct, stt, half_vec, lane);
                    if (kr) rope_half_row(kr, a.kv_dim / a.head, a.head, a.half, ct, stt, half_vec, lane);
                } else {
                    const int kp = k_pairs_interleaved(a.q_dim, a.kv_dim);
                    if (qr) rope_pair_row(qr, a.q_dim / 2, a.head, ct, stt, pair_vec, lane);
                    if (kr) rope_pair_row(kr, kp, a.head, ct, stt, pair_vec && kp % 2 == 0, lane);
                }
            }
        }
        if (a.gate) silu_range<4>(a.gate, a.up, (size_t)r0 * a.hidden, (size_t)(r0 + g) * a.hidden, st, nst);
    }
    __syncthreads();

    // ---- stage 2: normalised rows and the residual sum from the staged copy
    if constexpr (!FQ) {
        if (a.xb == nullptr && a.x_out == nullptr) return;
        if constexpr (VEC) {
            constexpr int U = 4;
            const int n4 = dim >> 2;
            const int total = g * n4;
            for (int i0 = tid; i0 < total; i0 += U * blockDim.x) {
                float4 rr[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int idx = i0 + k * blockDim.x;
                    if (idx < total && a.resid && a.x_out) {
                        const int r = idx / n4, c = (idx - r * n4) << 2;
                        rr[k] = ld4(a.resid + (size_t)(r0 + r) * dim + c);
                    }
                }
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int idx = i0 + k * blockDim.x;
                    if (idx >= total) continue;
                    const int r = idx / n4, c = (idx - r * n4) << 2;
                    const size_t o = (size_t)(r0 + r) * dim + c;
                    float v[4];
                    decode_staged<SRC, 4>(xs + (size_t)r * L.xstride, dim, c, v);
                    if (a.xb) {
                        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + c));
                        const float s = sc1[r];
                        st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s, v[0])), mul_rn(w.y, mul_rn(s, v[1])),
                                                  mul_rn(w.z, mul_rn(s, v[2])), mul_rn(w.w, mul_rn(s, v[3]))));
                    }
                    if (a.x_out) {
                        float4 xo = make_float4(v[0], v[1], v[2], v[3]);
                        if (a.resid)
                            xo = make_float4(add_rn(v[0], rr[k].x), add_rn(v[1], rr[k].y), add_rn(v[2], rr[k].z),
                                             add_rn(v[3], rr[k].w));
                        st4(a.x_out + o, xo);
                    }
                }
            }
        } else {
            for (int idx = tid; idx < g * dim; idx += blockDim.x) {
                const int r = idx / dim, c = idx - r * dim;
                const size_t o = (size_t)(r0 + r) * dim + c;
                float v[1];
                decode_staged<SRC, 1>(xs + (size_t)r * L.xstride, dim, c, v);
                if (a.xb) a.xb[o] = mul_rn(a.w_att[c], mul_rn(sc1[r], v[0]));
                if (a.x_out) a.x_out[o] = a.resid ? add_rn(v[0], a.resid[o]) : v[0];
            }
        }
    } else {
        // Final RMSNorm fused with Q8_0 quantisation (quant.rs:856-874): one
        // warp per row, lane l holds element 32*b + l of block b.
        const int nb = (dim + 31) >> 5;
        for (int r = warp; r < g; r += nwarps) {
            const int row = r0 + r;
            const float s1 = sc1[r], s2 = sc2[r];
            const unsigned char *xrow = xs + (size_t)r * L.xstride;
            const float *rrow = reinterpret_cast<const float *>(rs + (size_t)r * L.rstride);
            for (int b = 0; b < nb; ++b) {
                const int i = b * 32 + lane;
                const bool ok = i < dim;
                float v[1] = {0.0f};
                if (ok) decode_staged<SRC, 1>(xrow, dim, i, v);
                const size_t o = (size_t)row * dim + i;
                if (ok && a.xb) a.xb[o] = mul_rn(a.w_att[i], mul_rn(s1, v[0]));
                const float xo = (ok && fq_resid) ? add_rn(v[0], rrow[i]) : v[0];
                if (ok && a.x_out) a.x_out[o] = xo;
                const float y = ok ? mul_rn(a.w_final[i], mul_rn(s2, xo)) : 0.0f;
                float am = fmaxf(0.0f, fabsf(y));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(kFull, am, off));
                const float d = q8_scale(am);
                const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
                a.codes[(size_t)row * nb * 32 + i] = ok ? q8_code(mul_rn(y, inv)) : (int8_t)0;
                if (lane == 0) {
                    a.scales[(size_t)row * nb + b] = d;
                    if (a.scales16) a.scales16[(size_t)row * nb + b] = f16_bits(d);
                }
            }
        }
    }
}

// Four consecutive values of row `row`'s source straight from global memory
// (the f32 x row, or the gathered embedding row in its stored format), as
// decode_staged reads them from a staged slot; nullptr-row for a bad token.
template <int SRC>
__device__ __forceinline__ void decode_global4(const ChainArgs &a, const float *xsrc, int row, int c, float *v) {
    if constexpr (SRC == SRC_X) {
        const float4 t = ld4(xsrc + (size_t)row * a.dim + c);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
        const int tok = a.tokens[row];
        if ((unsigned)tok >= (unsigned)a.vocab) {
            v[0] = v[1] = v[2] = v[3] = 0.0f;
            return;
        }
        if constexpr (SRC == SRC_BF16) {
            const uint2 t = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(a.table) +
                                                                  (size_t)tok * a.dim + c));
            v[0] = bf16f(t.x & 0xffffu); v[1] = bf16f(t.x >> 16);
            v[2] = bf16f(t.y & 0xffffu); v[3] = bf16f(t.y >> 16);
        } else if constexpr (SRC == SRC_Q8) {
            const uint32_t t = __ldg(reinterpret_cast<const uint32_t *>(static_cast<const int8_t *>(a.table) +
                                                                        (size_t)tok * a.dim + c));
            const float s = __ldg(a.tscales + (size_t)tok * (a.dim >> 5) + (c >> 5));
#pragma unroll
            for (int b = 0; b < 4; ++b) v[b] = mul_rn((float)(int8_t)((t >> (8 * b)) & 0xffu), s);
        } else {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.table) +
                                                                    (size_t)tok * a.dim + c));
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        }
    }
}

// The norm stage alone (embed/x -> RMSNorm -> xb, residual add), as a
// persistent, warp-specialised pipeline over groups of G rows held in NS
// shared-memory slots.  In iteration i of a CTA:
//   warps 1..NL stage group i+1 into slot (i+1)%NS (cp.async, or through
//               registers for PRE_ADD),
//   warp 0      sums group i out of slot i%NS: lane r runs row r's squares
//               left to right, the reference's order (reference.rs:167-170),
//   warps NL+1.. write group i-1: xb = w*(scale*x), x + resid.
// One __syncthreads per iteration hands each slot to its next role.
//
// The writers take group i-1's values either from its slot (RR false: three
// slots, so staging, summing and writing use distinct ones) or again from
// global memory (RR true: two slots), where the rows are still L2-resident
// from the staging one iteration earlier.  RR frees a slot, so a slot holds
// 1.5x the rows and more exact chains run per SM; it pays where the re-read
// is one contiguous f32 row (rms_norm of x), not where it is a token gather.
//
// PRE_ADD (f32 x) is the driver's add_in_place -> rms_norm pair (llama.rs:
// 762-765, 769-740): the loaders add the residual while staging, write
// x = x + resid back, and the norm is taken of the sum; writers store xb.
// FQ is the final RMSNorm fused with Q8_0 quantisation (quant.rs:856-874): the
// summing lanes also run the sum of the row that gets quantised (x, or
// x + resid with the residual rows staged beside x), and the writers emit the
// int8 codes and block scales, eight lanes per 32-element block.
template <int SRC, bool VEC, bool PRE_ADD, bool FQ, bool RR>
__global__ void __launch_bounds__(kPipeThreads, 1) k_norm_pipe(ChainArgs a, ChainLayout L) {
    static_assert(!PRE_ADD || (SRC == SRC_X && VEC), "the pre-add form stages f32 rows with vector loads");
    static_assert(!FQ || (VEC && !PRE_ADD), "the quantising form needs whole 32-element blocks");
    constexpr int NL = PRE_ADD ? 3 : 1;  // loader warps 1..NL; writers NL+1..7
    constexpr int NS = RR ? 2 : 3;       // slots
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dim = a.dim;
    const int G = L.G;
    const int ngroups = (a.rows + G - 1) / G;
    const int nmine = (int)blockIdx.x < ngroups ? (ngroups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const size_t slot_bytes = (size_t)G * (L.xstride + L.rstride);
    float *scales = reinterpret_cast<float *>(smem + NS * slot_bytes);  // [NS][64]: s1[32] s2[32]
    const bool fq_resid = FQ && a.resid != nullptr;
    const int rb = src_row_bytes<SRC>(dim);
    // The rows the writers re-read: the loaders' x + resid for PRE_ADD.
    const float *xsrc = PRE_ADD ? a.x_out : a.x_in;

    auto first_row = [&](int i) { return (int)(blockIdx.x + (unsigned)i * gridDim.x) * G; };
    auto slot = [&](int i) { return smem + (size_t)(i % NS) * slot_bytes; };

    auto load = [&](int i) {  // warps 1..NL
        const int r0 = first_row(i), g = min(G, a.rows - r0);
        unsigned char *base = slot(i);
        if constexpr (PRE_ADD) {
            constexpr int U = 4;
            const int lt = tid - 32, nlt = NL * 32;
            const int n4 = dim >> 2, total = g * n4;
            for (int i0 = lt; i0 < total; i0 += U * nlt) {
                float4 xv[U], rv[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int idx = i0 + k * nlt;
                    if (idx < total) {
                        const int r = idx / n4, c = (idx - r * n4) << 2;
                        xv[k] = ld4(a.x_in + (size_t)(r0 + r) * dim + c);
                        rv[k] = ld4(a.resid + (size_t)(r0 + r) * dim + c);
                    }
                }
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int idx = i0 + k * nlt;
                    if (idx >= total) continue;
                    const int r = idx / n4, c = (idx - r * n4) << 2;
                    const float4 xo = make_float4(add_rn(xv[k].x, rv[k].x), add_rn(xv[k].y, rv[k].y),
                                                  add_rn(xv[k].z, rv[k].z), add_rn(xv[k].w, rv[k].w));
                    *reinterpret_cast<float4 *>(base + (size_t)r * L.xstride + 4 * c) = xo;
                    // a normal store: the writers re-read it from L2 next iteration
                    *reinterpret_cast<float4 *>(a.x_out + (size_t)(r0 + r) * dim + c) = xo;
                }
            }
            return;
        }
        for (int r = 0; r < g; ++r) {
            const unsigned char *sp;
            int tok = 0;
            if constexpr (SRC == SRC_X) {
                sp = reinterpret_cast<const unsigned char *>(a.x_in + (size_t)(r0 + r) * dim);
            } else {
                tok = a.tokens[r0 + r];
                sp = (unsigned)tok < (unsigned)a.vocab
                         ? static_cast<const unsigned char *>(a.table) + (size_t)tok * (size_t)rb
                         : nullptr;
                if (!sp && lane == 0) set_err(a.err, ERR_TOKEN);
            }
            unsigned char *dst = base + (size_t)r * L.xstride;
            if constexpr (VEC) {
                for (int c = lane; c < (rb >> 4); c += 32) {
                    if (sp) cp_async16(dst + 16 * c, sp + 16 * c);
                    else *reinterpret_cast<uint4 *>(dst + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
                }
            } else {
                for (int c = lane; c < rb; c += 32) dst[c] = sp ? sp[c] : (unsigned char)0;
            }
            if constexpr (SRC == SRC_Q8) {
                const int nb = dim >> 5;
                float *sdst = reinterpret_cast<float *>(dst + align16(dim));
                for (int b = lane; b < nb; b += 32) sdst[b] = sp ? __ldg(a.tscales + (size_t)tok * nb + b) : 0.0f;
            }
            if (fq_resid) {
                const float *rsrc = a.resid + (size_t)(r0 + r) * dim;
                unsigned char *rdst = base + (size_t)G * L.xstride + (size_t)r * L.rstride;
                for (int c = lane; c < (dim >> 2); c += 32) cp_async16(rdst + 16 * c, rsrc + 4 * c);
            }
        }
        if constexpr (VEC) cp_async_wait_all();
    };

    auto sum = [&](int i) {  // warp 0
        const int r0 = first_row(i), g = min(G, a.rows - r0);
        if (lane >= g) return;
        const unsigned char *row = slot(i) + (size_t)lane * L.xstride;
        float *sc = scales + (i % NS) * 64;
        float ss = 0.0f;
        if constexpr (FQ) {
            if (fq_resid) {
                // x + resid is what gets quantised: a second chain over it
                const float *rrow =
                    reinterpret_cast<const float *>(slot(i) + (size_t)G * L.xstride + (size_t)lane * L.rstride);
                float ss2 = 0.0f;
#pragma unroll 4
                for (int c = 0; c < dim; c += 8) {
                    float v[8];
                    decode_staged<SRC, 8>(row, dim, c, v);
                    const float4 r0v = *reinterpret_cast<const float4 *>(rrow + c);
                    const float4 r1v = *reinterpret_cast<const float4 *>(rrow + c + 4);
                    const float rv[8] = {r0v.x, r0v.y, r0v.z, r0v.w, r1v.x, r1v.y, r1v.z, r1v.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        ss = add_rn(ss, mul_rn(v[e], v[e]));
                        const float xo = add_rn(v[e], rv[e]);
                        ss2 = add_rn(ss2, mul_rn(xo, xo));
                    }
                }
                sc[lane] = rms_scale(ss, (float)dim, a.eps);
                sc[32 + lane] = rms_scale(ss2, (float)dim, a.final_eps);
            } else {
                // the quantised row is x itself: both norms share one sum
#pragma unroll 4
                for (int c = 0; c < dim; c += 8) {
                    float v[8];
                    decode_staged<SRC, 8>(row, dim, c, v);
#pragma unroll
                    for (int e = 0; e < 8; ++e) ss = add_rn(ss, mul_rn(v[e], v[e]));
                }
                sc[lane] = rms_scale(ss, (float)dim, a.eps);
                sc[32 + lane] = rms_scale(ss, (float)dim, a.final_eps);
            }
            return;
        } else if constexpr (VEC) {
#pragma unroll 4
            for (int c = 0; c < dim; c += 8) {
                float v[8];
                decode_staged<SRC, 8>(row, dim, c, v);
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = add_rn(ss, mul_rn(v[e], v[e]));
            }
        } else {
            for (int c = 0; c < dim; ++c) {
                float v[1];
                decode_staged<SRC, 1>(row, dim, c, v);
                ss = add_rn(ss, mul_rn(v[0], v[0]));
            }
        }
        sc[lane] = rms_scale(ss, (float)dim, a.eps);
    };

    // Four values of x (staged or re-read) at (group row r, column c).
    auto fetch4 = [&](const unsigned char *base, int r0, int r, int c, float *v) {
        if constexpr (RR) decode_global4<SRC>(a, xsrc, r0 + r, c, v);
        else decode_staged<SRC, 4>(base + (size_t)r * L.xstride, dim, c, v);
    };

    auto write = [&](int i) {  // warps NL+1..7
        const int r0 = first_row(i), g = min(G, a.rows - r0);
        const unsigned char *base = slot(i);
        const float *sc = scales + (i % NS) * 64;
        const int wt = tid - 32 * (NL + 1), nwt = blockDim.x - 32 * (NL + 1);
        if constexpr (FQ) {
            // 8 lanes x float4 per 32-element block; the loop is warp-uniform
            // so every lane reaches the group shuffles.
            const int nb = dim >> 5, total = g * nb * 8;
            const float *sc2 = sc + 32;
            for (int base_i = wt - lane; base_i < total; base_i += nwt) {
                const int idx = base_i + lane;
                const bool ok = idx < total;
                const int blk = ok ? idx >> 3 : 0, sub = idx & 7;
                const int r = blk / nb, b = blk - r * nb, c = b * 32 + sub * 4;
                const int row = r0 + r;
                float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (ok) {
                    float v[4];
                    fetch4(base, r0, r, c, v);
                    const size_t o = (size_t)row * dim + c;
                    if (a.xb) {
                        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + c));
                        const float s1 = sc[r];
                        st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s1, v[0])), mul_rn(w.y, mul_rn(s1, v[1])),
                                                  mul_rn(w.z, mul_rn(s1, v[2])), mul_rn(w.w, mul_rn(s1, v[3]))));
                    }
                    float4 xo = make_float4(v[0], v[1], v[2], v[3]);
                    if (fq_resid) {
                        const float4 rr = RR ? ld4(a.resid + o)
                                             : *reinterpret_cast<const float4 *>(base + (size_t)G * L.xstride +
                                                                                (size_t)r * L.rstride + 4 * c);
                        xo = make_float4(add_rn(v[0], rr.x), add_rn(v[1], rr.y), add_rn(v[2], rr.z), add_rn(v[3], rr.w));
                    }
                    if (a.x_out) st4(a.x_out + o, xo);
                    const float4 wf = __ldg(reinterpret_cast<const float4 *>(a.w_final + c));
                    const float s2 = sc2[r];
                    y = make_float4(mul_rn(wf.x, mul_rn(s2, xo.x)), mul_rn(wf.y, mul_rn(s2, xo.y)),
                                    mul_rn(wf.z, mul_rn(s2, xo.z)), mul_rn(wf.w, mul_rn(s2, xo.w)));
                }
                float am = fmaxf(fmaxf(fmaxf(0.0f, fabsf(y.x)), fmaxf(0.0f, fabsf(y.y))),
                                 fmaxf(fmaxf(0.0f, fabsf(y.z)), fmaxf(0.0f, fabsf(y.w))));
                am = fmaxf(am, __shfl_xor_sync(kFull, am, 1));
                am = fmaxf(am, __shfl_xor_sync(kFull, am, 2));
                am = fmaxf(am, __shfl_xor_sync(kFull, am, 4));
                if (!ok) continue;
                const float d = q8_scale(am);
                const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
                const uint32_t packed = (uint32_t)(uint8_t)q8_code(mul_rn(y.x, inv)) |
                                        ((uint32_t)(uint8_t)q8_code(mul_rn(y.y, inv)) << 8) |
                                        ((uint32_t)(uint8_t)q8_code(mul_rn(y.z, inv)) << 16) |
                                        ((uint32_t)(uint8_t)q8_code(mul_rn(y.w, inv)) << 24);
                *reinterpret_cast<uint32_t *>(a.codes + (size_t)row * nb * 32 + c) = packed;
                if (sub == 0) {
                    a.scales[(size_t)row * nb + b] = d;
                    if (a.scales16) a.scales16[(size_t)row * nb + b] = f16_bits(d);
                }
            }
            return;
        }
        if constexpr (VEC) {
            constexpr int U = 4;
            const int n4 = dim >> 2, total = g * n4;
            for (int i0 = wt; i0 < total; i0 += U * nwt) {
                float v[U][4];
                float4 rr[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int idx = i0 + k * nwt;
                    if (idx < total) {
                        const int r = idx / n4, c = (idx - r * n4) << 2;
                        fetch4(base, r0, r, c, v[k]);
                        if (!PRE_ADD && a.resid && a.x_out) rr[k] = ld4(a.resid + (size_t)(r0 + r) * dim + c);
                    }
                }
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int idx = i0 + k * nwt;
                    if (idx >= total) continue;
                    const int r = idx / n4, c = (idx - r * n4) << 2;
                    const size_t o = (size_t)(r0 + r) * dim + c;
                    if (a.xb) {
                        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + c));
                        const float s = sc[r];
                        st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s, v[k][0])), mul_rn(w.y, mul_rn(s, v[k][1])),
                                                  mul_rn(w.z, mul_rn(s, v[k][2])), mul_rn(w.w, mul_rn(s, v[k][3]))));
                    }
                    if (!PRE_ADD && a.x_out) {
                        float4 xo = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
                        if (a.resid)
                            xo = make_float4(add_rn(v[k][0], rr[k].x), add_rn(v[k][1], rr[k].y),
                                             add_rn(v[k][2], rr[k].z), add_rn(v[k][3], rr[k].w));
                        st4(a.x_out + o, xo);
                    }
                }
            }
        } else {
            for (int idx = wt; idx < g * dim; idx += nwt) {
                const int r = idx / dim, c = idx - r * dim;
                const size_t o = (size_t)(r0 + r) * dim + c;
                float v;
                if constexpr (!RR) {
                    float t[1];
                    decode_staged<SRC, 1>(base + (size_t)r * L.xstride, dim, c, t);
                    v = t[0];
                } else if constexpr (SRC == SRC_X) {
                    v = xsrc[o];
                } else {
                    const int tok = a.tokens[r0 + r];
                    if ((unsigned)tok >= (unsigned)a.vocab) v = 0.0f;
                    else if constexpr (SRC == SRC_BF16) v = bf16f(static_cast<const uint16_t *>(a.table)[(size_t)tok * dim + c]);
                    else if constexpr (SRC == SRC_Q8)
                        v = mul_rn((float)static_cast<const int8_t *>(a.table)[(size_t)tok * dim + c],
                                   a.tscales[(size_t)tok * (dim >> 5) + (c >> 5)]);
                    else v = static_cast<const float *>(a.table)[(size_t)tok * dim + c];
                }
                if (a.xb) a.xb[o] = mul_rn(a.w_att[c], mul_rn(sc[r], v));
                if (a.x_out) a.x_out[o] = a.resid ? add_rn(v, a.resid[o]) : v;
            }
        }
    };

    if (warp >= 1 && warp <= NL && nmine > 0) load(0);
    __syncthreads();
    for (int i = 0; i <= nmine; ++i) {
        if (warp >= 1 && warp <= NL) {
            if (i + 1 < nmine) load(i + 1);
        } else if (warp == 0) {
            if (i < nmine) sum(i);
        } else {
            if (i >= 1) write(i - 1);
        }
        __syncthreads();
    }
}

constexpr int kRowsThreadsPlain = 640;
// k_norm_rows: 16 warps (12 writers) in the quantising form, 20 (15 writers,
// at most 102 registers each) otherwise, where the writers' residual loads
// and stores want more warps in flight (measured: 0.340 -> 0.321 ms for the
// 65 536-row chain's norm stage; 24 warps no better, 32 spill).
template <bool FQ>
struct RowsShape {
    static constexpr int threads = FQ ? 512 : kRowsThreadsPlain;
    static constexpr int writers = threads / 32 * 3 / 4;  // the warps off sub-partition 0
};

// f32 x rows with the three roles decoupled: one CTA per SM (ColsShape), its
// rows in groups of G, a group's rows cut into T column tiles of TC columns
// (a unit = one tile of one group).
//   warp 4    issues unit u's bulk copies (lane r: row r's x tile, and its
//             resid tile where the sums need it) into slot u % S of a ring
//             of S slots once the summing warp has handed that slot back;
//   warp 0    sums unit after unit, lane r row r left to right (the
//             reference's order, reference.rs:167-170) carried across tiles
//             in a register, hands each slot back, and after a group's last
//             tile stores its scales into one of two buffers;
//   writers   (the warps off warp 0's sub-partition; when quantising, all
//             warps but 0 and 4) take group after group once its scales are
//             stored and write xb, x (+ resid) or the Q8_0 codes from x (and
//             resid) loaded from L2, where the ring's copies left them a
//             group earlier: U 16-byte loads in flight per lane, no barrier
//             between tiles.
// mbarriers connect the roles (full/empty per slot, ready/freed per scale
// buffer), so each runs at its own rate: the summing lanes' chains, the copy
// engine and the writers' L2 traffic overlap instead of meeting at a CTA
// barrier per tile.  In the plain forms the other warps of warp 0's
// sub-partition only wait at the end.
// PRE_ADD: the sums are of x + resid (the driver's add_in_place -> rms_norm,
// llama.rs:762-765) and the writers store x = x + resid and xb.  FQ: a second
// sum of x (+ resid) for the final norm, and the writers quantise it to Q8_0
// (quant.rs:856-874).
// Two ring slots: the larger tiles that two slots leave room for (whole
// 1024-column halves at 2048 columns, 2 KB copies at 1024 when quantising)
// measured faster on B200 than a deeper ring of smaller tiles (4 slots:
// rms_norm 0.222 -> 0.216 ms, add + rms_norm 0.402 -> 0.388 ms, rms_norm_q8_0
// 0.095 -> 0.093 ms; 3 slots slower for rms_norm).
constexpr int kColsSlots = 2;
// The quantising form runs 24 warps, all but the summing and the copying warp
// writers (22, at most 85 registers each, four items per batch): its writers
// are bound by their instruction issue (the block arithmetic), so they take
// sub-partition 0's spare issue slots too, which the summing warp's chains
// leave mostly free.  The plain forms' writers are bound by their loads and
// stores and stay off sub-partition 0: 16 warps, 12 writers, eight items per
// batch.
template <bool FQ>
struct ColsShape {
    static constexpr int threads = FQ ? 768 : 512;
    static constexpr int writers = FQ ? threads / 32 - 2 : threads / 32 * 3 / 4;
    static constexpr int U = FQ ? 4 : 8;  // items per writer lane and batch
};
constexpr unsigned kColsSleepNs = 128;  // poll interval of the issuer's and the writers' waits

struct ColsLayout {
    int G;       // rows per group (<= 32: one summing lane per row)
    int TC;      // columns per tile; the last tile may be shorter
    int T;       // tiles per row
    int stride;  // bytes per staged row: x tile (+ resid tile), an odd multiple of 16
    int rofs;    // byte offset of the resid tile in a staged row
    int slot;    // G * stride
    size_t smem;
};

// k_norm_cols' writers for the plain rms_norm_q8_0 (no residual, no xb, no x
// copy), a group's rows r0.. at its scales s2[r].  The group is one contiguous
// range, so its float4 item j sits at x + r0 * dim + 4 j, its four codes at the
// same element offset and its block scale at r0 * nb + j / 8: no per-row
// address arithmetic.  Writer thread wt takes items wt, wt + nwt, ...; (r, c4)
// follow item j's row and float4 column (dr, dc = nwt / q, nwt % q).  The clamp
// of the codes runs only for blocks whose 1/d overflows (q8_needs_clamp).
template <int U>
__device__ __forceinline__ void fq_write_group(const ChainArgs &a, const float *s2, int r0, int total, int q, int wt,
                                               int nwt, int dr, int dc) {
    const int dim = a.dim, nb = dim >> 5, lane = wt & 31;
    const float4 *xg = reinterpret_cast<const float4 *>(a.x_in + (size_t)r0 * dim);
    const float4 *wf = reinterpret_cast<const float4 *>(a.w_final);
    uint32_t *cg = reinterpret_cast<uint32_t *>(a.codes + (size_t)r0 * dim);
    float *sg = a.scales + (size_t)r0 * nb;
    uint16_t *hg = a.scales16 ? a.scales16 + (size_t)r0 * nb : nullptr;
    int r = wt / q, c4 = wt - r * q;
    for (int j = wt; j - lane < total; j += U * nwt) {
        float4 y[U];
        float am[U];
        int cs[U];
        float ss[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const bool ok = j + k * nwt < total;
            y[k] = ok ? __ldcs(xg + j + k * nwt) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            ss[k] = ok ? s2[r] : 0.0f;
            cs[k] = c4;
            c4 += dc;
            r += dr;
            if (c4 >= q) {
                c4 -= q;
                ++r;
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const float4 w = __ldg(wf + cs[k]);
            const float s = ss[k];
            y[k] = make_float4(mul_rn(w.x, mul_rn(s, y[k].x)), mul_rn(w.y, mul_rn(s, y[k].y)),
                               mul_rn(w.z, mul_rn(s, y[k].z)), mul_rn(w.w, mul_rn(s, y[k].w)));
            // the fold of fmaxf from +0 (quant.rs:862): NaNs drop out
            am[k] = fmaxf(0.0f, fmaxf(fmaxf(fabsf(y[k].x), fabsf(y[k].y)), fmaxf(fabsf(y[k].z), fabsf(y[k].w))));
        }
        // eight lanes per 32-element block, all in one warp and one row
#pragma unroll
        for (int m = 1; m < 8; m <<= 1)
#pragma unroll
            for (int k = 0; k < U; ++k) am[k] = fmaxf(am[k], __shfl_xor_sync(kFull, am[k], m));
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int jk = j + k * nwt;
            if (jk >= total) continue;
            const float d = q8_scale(am[k]);
            const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
            int c0 = q8_round(mul_rn(y[k].x, inv)), c1 = q8_round(mul_rn(y[k].y, inv));
            int c2 = q8_round(mul_rn(y[k].z, inv)), c3 = q8_round(mul_rn(y[k].w, inv));
            if (q8_needs_clamp(d)) {
                c0 = max(-127, min(127, c0));
                c1 = max(-127, min(127, c1));
                c2 = max(-127, min(127, c2));
                c3 = max(-127, min(127, c3));
            }
            __stcs(cg + jk, (uint32_t)(c0 & 0xff) | ((uint32_t)(c1 & 0xff) << 8) | ((uint32_t)(c2 & 0xff) << 16) |
                     ((uint32_t)c3 << 24));
            if ((lane & 7) == 0) {
                sg[jk >> 3] = d;
                if (hg) hg[jk >> 3] = f16_bits(d);
            }
        }
    }
}

// fq_write_group with eight elements per lane and item (x, w_final 32-byte
// aligned, codes 8-byte aligned): a 32-element block is four lanes, so the
// block arithmetic, the amax shuffles (two rounds) and the index bookkeeping
// are spent once per eight elements instead of once per four.  Items count
// octets here (q = dim / 8 per row); the inverse is q8_inv_block's branchless
// form.
template <int U>
__device__ __forceinline__ void fq_write_group8(const ChainArgs &a, const float *s2, int r0, int total, int q,
                                                int wt, int nwt, int dr, int dc) {
    const int dim = a.dim, nb = dim >> 5, lane = wt & 31;
    const float *xg = a.x_in + (size_t)r0 * dim;
    uint2 *cg = reinterpret_cast<uint2 *>(a.codes + (size_t)r0 * dim);
    float *sg = a.scales + (size_t)r0 * nb;
    uint16_t *hg = a.scales16 ? a.scales16 + (size_t)r0 * nb : nullptr;
    int r = wt / q, c8 = wt - r * q;
    for (int j = wt; j - lane < total; j += U * nwt) {
        float y[U][8];
        float am[U], ss[U];
        int cs[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const bool ok = j + k * nwt < total;
            if (ok) {
                ld8_stream(xg + (size_t)8 * (j + k * nwt), y[k]);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) y[k][e] = 0.0f;
            }
            ss[k] = ok ? s2[r] : 0.0f;
            cs[k] = c8;
            c8 += dc;
            r += dr;
            if (c8 >= q) {
                c8 -= q;
                ++r;
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            float w[8];
            ld8_ro(a.w_final + 8 * cs[k], w);
            const float s = ss[k];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[k][e] = mul_rn(w[e], mul_rn(s, y[k][e]));
            // the fold of fmaxf from +0 (quant.rs:862): NaNs drop out
            const float m01 = fmaxf(fabsf(y[k][0]), fabsf(y[k][1])), m23 = fmaxf(fabsf(y[k][2]), fabsf(y[k][3]));
            const float m45 = fmaxf(fabsf(y[k][4]), fabsf(y[k][5])), m67 = fmaxf(fabsf(y[k][6]), fabsf(y[k][7]));
            am[k] = fmaxf(0.0f, fmaxf(fmaxf(m01, m23), fmaxf(m45, m67)));
        }
        // four lanes per 32-element block, all in one warp and one row
#pragma unroll
        for (int m = 1; m < 4; m <<= 1)
#pragma unroll
            for (int k = 0; k < U; ++k) am[k] = fmaxf(am[k], __shfl_xor_sync(kFull, am[k], m));
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int jk = j + k * nwt;
            if (jk >= total) continue;
            const float d = q8_scale(am[k]);
            const float inv = q8_inv_block(d);
            int c[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) c[e] = q8_round(mul_rn(y[k][e], inv));
            if (q8_needs_clamp(d)) {
#pragma unroll
                for (int e = 0; e < 8; ++e) c[e] = max(-127, min(127, c[e]));
            }
            const uint32_t lo = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
            const uint32_t hi = __byte_perm(__byte_perm(c[4], c[5], 0x0040), __byte_perm(c[6], c[7], 0x0040), 0x5410);
            __stcs(cg + jk, make_uint2(lo, hi));
            if ((lane & 3) == 0) {
                sg[jk >> 2] = d;
                if (hg) hg[jk >> 2] = f16_bits(d);
            }
        }
    }
}

template <bool PRE_ADD, bool FQ>
__global__ void __launch_bounds__(ColsShape<FQ>::threads, 1) k_norm_cols(ChainArgs a, ColsLayout L) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int NS = kColsSlots;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dim = a.dim, G = L.G, T = L.T, TC = L.TC;
    const int ngroups = (a.rows + G - 1) / G;
    const int nmine = (int)blockIdx.x < ngroups ? (ngroups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int units = nmine * T;
    float *scales = reinterpret_cast<float *>(smem + NS * (size_t)L.slot);  // [2][64]
    uint64_t *full = reinterpret_cast<uint64_t *>(scales + 128);            // [NS] a slot's bytes landed
    uint64_t *empty = full + NS;                                            // [NS] a slot summed
    uint64_t *ready = empty + NS;                                           // [2] a group's scales stored
    uint64_t *freed = ready + 2;                                            // [2] a group written
    __shared__ volatile int s_abort;
    __shared__ int s_issued, s_consumed;
    const bool has_resid = a.resid != nullptr;
    const bool sum_resid = PRE_ADD || (FQ && has_resid);
    const bool write_resid = has_resid && (PRE_ADD || FQ || a.x_out);
    auto first_row = [&](int g) { return (int)(blockIdx.x + (unsigned)g * gridDim.x) * G; };

    if (tid == 0) {
        s_abort = 0;
        s_issued = s_consumed = 0;
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ready[i], 1);
            mbar_init(&freed[i], ColsShape<FQ>::writers);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // A bounded wait that also gives up once another role has given up; the
    // warp agrees on the outcome.  Roles whose waits are not on the critical
    // path (the copy issuer shares warp 0's sub-partition) sleep between
    // polls, leaving the issue slots to the warps that work.
    auto wait = [&](uint64_t *bar, uint32_t parity, unsigned sleep_ns) {
        bool ok = mbar_try_wait(bar, parity);
        if (!ok) {
            const long long t0 = clock64();
            while (!(ok = mbar_try_wait(bar, parity))) {
                if (sleep_ns) __nanosleep(sleep_ns);
                if (s_abort) break;
                if (clock64() - t0 > (1ll << 31)) {
                    set_err(a.err, ERR_TIMEOUT);
                    s_abort = 1;
                    break;
                }
            }
        }
        return __all_sync(kFull, ok);
    };

    if (warp == 4) {
        // the writers read these rows again a group later: keep them in L2
        const uint64_t keep = l2_evict_last();
        int u = 0;
        for (; u < units; ++u) {
            if (u >= NS && !wait(&empty[u % NS], (uint32_t)(u / NS - 1) & 1u, kColsSleepNs)) break;
            const int g = u / T, t = u - g * T;
            const int r0 = first_row(g), gr = min(G, a.rows - r0);
            const int c0 = t * TC, tc = min(TC, dim - c0);
            uint64_t *bar = &full[u % NS];
            if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)gr * (uint32_t)tc * (sum_resid ? 8u : 4u));
            __syncwarp();
            if (lane < gr) {
                unsigned char *dst = smem + (size_t)(u % NS) * L.slot + (size_t)lane * L.stride;
                const size_t o = (size_t)(r0 + lane) * dim + c0;
                bulk_load_hint(dst, a.x_in + o, (uint32_t)tc * 4u, bar, keep);
                if (sum_resid) bulk_load_hint(dst + L.rofs, a.resid + o, (uint32_t)tc * 4u, bar, keep);
            }
        }
        if (lane == 0) s_issued = u;
    } else if (warp == 0) {
        float ss = 0.0f, ss2 = 0.0f;
        int u = 0;
        bool ok = true;
        for (; u < units && ok; ++u) {
            const int g = u / T, t = u - g * T;
            const int r0 = first_row(g), gr = min(G, a.rows - r0);
            const int tc = min(TC, dim - t * TC);
            if (!wait(&full[u % NS], (uint32_t)(u / NS) & 1u, 0)) break;
            if (lane < gr) {
                const unsigned char *row = smem + (size_t)(u % NS) * L.slot + (size_t)lane * L.stride;
                const float *xr = reinterpret_cast<const float *>(row);
                const float *rr = reinterpret_cast<const float *>(row + L.rofs);
                // one step of eight columns loaded ahead of the step being
                // added, so the shared-memory latency stays off the chain
                auto ld8 = [&](const float *p, int c, float *v) {
                    const float4 p0 = *reinterpret_cast<const float4 *>(p + c), p1 = *reinterpret_cast<const float4 *>(p + c + 4);
                    v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
                    v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
                };
                float v[8], rv[8] = {}, nv[8], nrv[8] = {};
                if (!sum_resid && tc % 16 == 0) {
                    // one chain of x alone: the squares of the next 16
                    // columns ahead of the current adds (with x + resid the
                    // loop below measured faster)
                    ss = chain_add16(ss, tc / 16, [&](int b, float(&q)[16]) { squares16_f32(xr + 16 * b, q); });
                } else {
                ld8(xr, 0, v);
                if (sum_resid) ld8(rr, 0, rv);
#pragma unroll 2
                for (int c = 0; c < tc; c += 8) {
                    const int cn = c + 8 < tc ? c + 8 : c;
                    ld8(xr, cn, nv);
                    if (sum_resid) ld8(rr, cn, nrv);
                    if (PRE_ADD) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float xo = add_rn(v[e], rv[e]);
                            ss = add_rn(ss, mul_rn(xo, xo));
                        }
                    } else if (FQ && has_resid) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            ss = add_rn(ss, mul_rn(v[e], v[e]));
                            const float xo = add_rn(v[e], rv[e]);
                            ss2 = add_rn(ss2, mul_rn(xo, xo));
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) ss = add_rn(ss, mul_rn(v[e], v[e]));
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        v[e] = nv[e];
                        rv[e] = nrv[e];
                    }
                }
                }
            }
            // every lane's reads of the slot are done before it goes back
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[u % NS]);
            if (t == T - 1) {
                // group g's scales go to buffer g % 2 once the writers are
                // done with group g - 2
                if (g >= 2 && !wait(&freed[g & 1], (uint32_t)((g - 2) >> 1) & 1u, 0)) ok = false;
                if (ok) {
                    float *sc = scales + (g & 1) * 64;
                    if (lane < gr) {
                        sc[lane] = rms_scale(ss, (float)dim, a.eps);
                        if (FQ) sc[32 + lane] = rms_scale(has_resid ? ss2 : ss, (float)dim, a.final_eps);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ready[g & 1]);
                }
                ss = 0.0f;
                ss2 = 0.0f;
            }
        }
        // units whose copies were waited for
        if (lane == 0) s_consumed = u;
    } else if (FQ ? warp != 4 : (warp & 3) != 0) {
        const int wi = FQ ? warp - 1 - (warp > 4) : warp - 1 - (warp >> 2);
        const int nwt = ColsShape<FQ>::writers * 32, wt = wi * 32 + lane;
        const int q = dim >> 2;                 // float4 items per row
        const int dr = nwt / q, dc = nwt - dr * q;
        const bool lean = FQ && !a.xb && !a.x_out && !has_resid;
        const bool lean8 = lean && !((uintptr_t)a.x_in & 31) && !((uintptr_t)a.w_final & 31) && !((uintptr_t)a.codes & 7);
        const int q8 = dim >> 3, dr8 = nwt / q8, dc8 = nwt - dr8 * q8;  // octets per row; their strides
        for (int g = 0; g < nmine; ++g) {
            if (!wait(&ready[g & 1], (uint32_t)(g >> 1) & 1u, kColsSleepNs)) break;
            const float *sc = scales + (g & 1) * 64;
            const int r0 = first_row(g), gr = min(G, a.rows - r0);
            const int total = gr * q;  // the group's float4 items, row-major
            if (FQ && lean) {
                if (lean8)
                    fq_write_group8<ColsShape<FQ>::U / 2>(a, sc + 32, r0, gr * q8, q8, wt, nwt, dr8, dc8);
                else
                    fq_write_group<ColsShape<FQ>::U>(a, sc + 32, r0, total, q, wt, nwt, dr, dc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&freed[g & 1]);
                continue;
            }
            int r = wt / q, c4 = wt - r * q;
            constexpr int U = ColsShape<FQ>::U;
            for (int i = wt; i - lane < total; i += U * nwt) {
                int rs[U], cs[U];
                float4 xv[U], rv[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    rs[k] = r;
                    cs[k] = 4 * c4;
                    xv[k] = rv[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (i + k * nwt < total) {
                        const size_t o = (size_t)(r0 + r) * dim + cs[k];
                        xv[k] = ld4(a.x_in + o);
                        if (write_resid) rv[k] = ld4(a.resid + o);
                    }
                    c4 += dc;
                    r += dr;
                    if (c4 >= q) {
                        c4 -= q;
                        ++r;
                    }
                }
                // outputs in phases over the U items, so their latencies
                // (shuffles, loads of weights) overlap
                float4 y[U];
                float am[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const bool ok = i + k * nwt < total;
                    const int c = cs[k];
                    const size_t o = (size_t)(r0 + rs[k]) * dim + c;
                    float4 v = xv[k];
                    if (PRE_ADD)
                        v = make_float4(add_rn(v.x, rv[k].x), add_rn(v.y, rv[k].y), add_rn(v.z, rv[k].z),
                                        add_rn(v.w, rv[k].w));
                    if (a.xb && ok) {
                        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + c));
                        const float s1 = sc[rs[k]];
                        st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s1, v.x)), mul_rn(w.y, mul_rn(s1, v.y)),
                                                  mul_rn(w.z, mul_rn(s1, v.z)), mul_rn(w.w, mul_rn(s1, v.w))));
                    }
                    float4 xo = v;
                    if (!PRE_ADD && has_resid && (FQ || a.x_out))
                        xo = make_float4(add_rn(v.x, rv[k].x), add_rn(v.y, rv[k].y), add_rn(v.z, rv[k].z),
                                         add_rn(v.w, rv[k].w));
                    if (a.x_out && ok) st4(a.x_out + o, xo);
                    if constexpr (FQ) {
                        y[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        if (ok) {
                            const float4 wf = __ldg(reinterpret_cast<const float4 *>(a.w_final + c));
                            const float s2 = sc[32 + rs[k]];
                            y[k] = make_float4(mul_rn(wf.x, mul_rn(s2, xo.x)), mul_rn(wf.y, mul_rn(s2, xo.y)),
                                               mul_rn(wf.z, mul_rn(s2, xo.z)), mul_rn(wf.w, mul_rn(s2, xo.w)));
                        }
                        am[k] = fmaxf(fmaxf(fmaxf(0.0f, fabsf(y[k].x)), fmaxf(0.0f, fabsf(y[k].y))),
                                      fmaxf(fmaxf(0.0f, fabsf(y[k].z)), fmaxf(0.0f, fabsf(y[k].w))));
                    }
                }
                if constexpr (FQ) {
                    // eight lanes per 32-element block: q % 8 == 0 and a
                    // warp's 32 items are consecutive, so a block's lanes
                    // share a warp and a row
#pragma unroll
                    for (int m = 1; m < 8; m <<= 1)
#pragma unroll
                        for (int k = 0; k < U; ++k) am[k] = fmaxf(am[k], __shfl_xor_sync(kFull, am[k], m));
                    const int nb = dim >> 5;
#pragma unroll
                    for (int k = 0; k < U; ++k) {
                        if (i + k * nwt >= total) continue;
                        const int c = cs[k];
                        const float d = q8_scale(am[k]);
                        const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
                        const uint32_t packed = (uint32_t)(uint8_t)q8_code(mul_rn(y[k].x, inv)) |
                                                ((uint32_t)(uint8_t)q8_code(mul_rn(y[k].y, inv)) << 8) |
                                                ((uint32_t)(uint8_t)q8_code(mul_rn(y[k].z, inv)) << 16) |
                                                ((uint32_t)(uint8_t)q8_code(mul_rn(y[k].w, inv)) << 24);
                        const size_t ro = (size_t)(r0 + rs[k]);
                        *reinterpret_cast<uint32_t *>(a.codes + ro * dim + c) = packed;
                        if ((c & 31) == 0) {
                            a.scales[ro * nb + (c >> 5)] = d;
                            if (a.scales16) a.scales16[ro * nb + (c >> 5)] = f16_bits(d);
                        }
                    }
                }
            }
            // this warp's reads of the group's scales are done
            __syncwarp();
            if (lane == 0) mbar_arrive(&freed[g & 1]);
        }
    }
    __syncthreads();
    // Every copy issued was waited for unless a role gave up; then wait
    // (again bounded) for the copies still in flight before the memory goes.
    if (tid == 0 && s_abort)
        for (int u = s_consumed; u < s_issued; ++u) mbar_wait_bounded(&full[u % NS], (uint32_t)(u / NS) & 1u);
}

constexpr int kRowsSlots = 4;  // writing, summing, and two staged ahead

struct RowsLayout {
    int G;        // rows per group (<= 32)
    int xstride;  // bytes per staged row (+ Q8 block scales), an odd multiple of 16
    int rstride;  // bytes per staged f32 residual row, or 0
    int slot;     // G * (xstride + rstride)
    size_t smem;
};

// The norm stage over whole staged rows, one CTA per SM (RowsShape), four slots
// of G rows, each filled by one bulk copy per row (a full row is big enough
// that the copy engine's per-request cost stays far below the row's
// traffic).  In iteration i:
//   warp 4    issues group i+2's copies into slot (i+2)%4, lane r those of
//             row r (its x or embedding row, Q8 block scales, and the f32
//             resid row when the quantised norm sums x + resid), counted on
//             the slot's mbarrier;
//   warp 0    waits for group i and sums it, lane r row r left to right (the
//             reference's order, reference.rs:167-170);
//   writers   (the warps off warp 0's sub-partition) write group i-1 from its
//             slot: xb = w*(scale*x), x + resid (resid from global memory,
//             eight float4 loads in flight per lane), or the Q8_0 codes.
// Staging two groups ahead keeps a group's copies in flight for two
// iterations, longer than their HBM latency under load.  The other warps of
// warp 0's sub-partition only keep the barrier count.  FQ is the final
// RMSNorm fused with Q8_0 quantisation (quant.rs:856-874).
template <int SRC, bool FQ>
__global__ void __launch_bounds__(RowsShape<FQ>::threads, 1) k_norm_rows(ChainArgs a, RowsLayout L) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dim = a.dim, G = L.G;
    const int ngroups = (a.rows + G - 1) / G;
    const int nmine = (int)blockIdx.x < ngroups ? (ngroups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    constexpr int NS = kRowsSlots;
    float *scales = reinterpret_cast<float *>(smem + NS * (size_t)L.slot);  // [NS][64]
    uint64_t *bars = reinterpret_cast<uint64_t *>(scales + NS * 64);        // [NS]
    __shared__ int s_abort;
    const bool has_resid = a.resid != nullptr;
    const bool stage_resid = FQ && has_resid;
    const int rb = src_row_bytes<SRC>(dim);

    auto first_row = [&](int g) { return (int)(blockIdx.x + (unsigned)g * gridDim.x) * G; };
    auto slot = [&](int g) { return smem + (size_t)(g % NS) * L.slot; };

    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    __syncthreads();

    auto issue = [&](int g) {  // warp 4
        const int r0 = first_row(g), gr = min(G, a.rows - r0);
        const unsigned char *sp = nullptr;
        int tok = 0;
        uint32_t mine = 0;
        if (lane < gr) {
            if constexpr (SRC == SRC_X) {
                sp = reinterpret_cast<const unsigned char *>(a.x_in + (size_t)(r0 + lane) * dim);
            } else {
                tok = a.tokens[r0 + lane];
                if ((unsigned)tok < (unsigned)a.vocab)
                    sp = static_cast<const unsigned char *>(a.table) + (size_t)tok * (size_t)rb;
                else
                    set_err(a.err, ERR_TOKEN);
            }
            mine = (sp ? (uint32_t)rb + (SRC == SRC_Q8 ? (uint32_t)(dim / 8) : 0u) : 0u) +
                   (stage_resid ? (uint32_t)dim * 4u : 0u);
        }
        uint32_t total = mine;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(kFull, total, o);
        uint64_t *bar = &bars[g % NS];
        if (lane == 0) mbar_arrive_expect_tx(bar, total);
        __syncwarp();
        if (lane < gr) {
            unsigned char *dst = slot(g) + (size_t)lane * L.xstride;
            if (sp) {
                bulk_load(dst, sp, (uint32_t)rb, bar);
                if constexpr (SRC == SRC_Q8)
                    bulk_load(dst + align16(dim), a.tscales + (size_t)tok * (dim >> 5), (uint32_t)(dim / 8), bar);
            }
            if (stage_resid)
                bulk_load(slot(g) + (size_t)G * L.xstride + (size_t)lane * L.rstride, a.resid + (size_t)(r0 + lane) * dim,
                          (uint32_t)dim * 4u, bar);
        }
    };

    auto sum = [&](int g) {  // warp 0
        const int r0 = first_row(g), gr = min(G, a.rows - r0);
        if (s_abort) return;
        if (!mbar_wait_bounded(&bars[g % NS], (uint32_t)(g / NS) & 1u)) {
            if (lane == 0) {
                set_err(a.err, ERR_TIMEOUT);
                s_abort = 1;
            }
            return;
        }
        if (lane >= gr) return;
        bool valid = true;
        if constexpr (SRC != SRC_X) valid = (unsigned)a.tokens[r0 + lane] < (unsigned)a.vocab;
        const unsigned char *xr = slot(g) + (size_t)lane * L.xstride;
        float *sc = scales + (g % NS) * 64;
        float ss = 0.0f;
        if (FQ && stage_resid) {
            const float *rr = reinterpret_cast<const float *>(slot(g) + (size_t)G * L.xstride + (size_t)lane * L.rstride);
            float ss2 = 0.0f;
#pragma unroll 2
            for (int c = 0; c < dim; c += 8) {
                float v[8];
                decode_staged<SRC, 8>(xr, dim, c, v);
                if (!valid)
                    for (int e = 0; e < 8; ++e) v[e] = 0.0f;
                const float4 p = *reinterpret_cast<const float4 *>(rr + c), q = *reinterpret_cast<const float4 *>(rr + c + 4);
                const float rv[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    ss = add_rn(ss, mul_rn(v[e], v[e]));
                    const float xo = add_rn(v[e], rv[e]);
                    ss2 = add_rn(ss2, mul_rn(xo, xo));
                }
            }
            sc[lane] = rms_scale(ss, (float)dim, a.eps);
            sc[32 + lane] = rms_scale(ss2, (float)dim, a.final_eps);
            return;
        }
        if (valid && dim % 16 == 0) {
            ss = chain_add16(ss, dim / 16, [&](int b, float(&q)[16]) {
                decode_staged<SRC, 8>(xr, dim, 16 * b, q);
                decode_staged<SRC, 8>(xr, dim, 16 * b + 8, q + 8);
#pragma unroll
                for (int e = 0; e < 16; ++e) q[e] = mul_rn(q[e], q[e]);
            });
        } else if (valid) {
#pragma unroll 4
            for (int c = 0; c < dim; c += 8) {
                float v[8];
                decode_staged<SRC, 8>(xr, dim, c, v);
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = add_rn(ss, mul_rn(v[e], v[e]));
            }
        }
        sc[lane] = rms_scale(ss, (float)dim, a.eps);
        if (FQ) sc[32 + lane] = rms_scale(ss, (float)dim, a.final_eps);
    };

    const int wi = warp - 1 - (warp >> 2);
    auto write = [&](int g) {  // the writer warps
        if (s_abort) return;
        const int r0 = first_row(g), gr = min(G, a.rows - r0);
        const unsigned char *base = slot(g);
        const float *sc = scales + (g % NS) * 64;
        const int q = dim >> 2, total = gr * q;
        const int nwt = RowsShape<FQ>::writers * 32;
        const int dr = nwt / q, dc = nwt - dr * q;
        const int wt = wi * 32 + lane;
        int r = wt / q, c4 = wt - r * q;
        int vr = -1;
        bool vok = true;
        auto xval = [&](int rr_, int c, float *v) {
            decode_staged<SRC, 4>(base + (size_t)rr_ * L.xstride, dim, c, v);
            if constexpr (SRC != SRC_X) {
                if (rr_ != vr) {
                    vr = rr_;
                    vok = (unsigned)a.tokens[r0 + rr_] < (unsigned)a.vocab;
                }
                if (!vok) v[0] = v[1] = v[2] = v[3] = 0.0f;
            }
        };
        auto step = [&]() {
            c4 += dc;
            r += dr;
            if (c4 >= q) {
                c4 -= q;
                ++r;
            }
        };
        if constexpr (FQ) {
            for (int i = wt; i - lane < total; i += nwt) {
                const bool ok = i < total;
                const int c = 4 * c4, row = r0 + r;
                float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (ok) {
                    float v[4];
                    xval(r, c, v);
                    const size_t o = (size_t)row * dim + c;
                    if (a.xb) {
                        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + c));
                        const float s1 = sc[r];
                        st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s1, v[0])), mul_rn(w.y, mul_rn(s1, v[1])),
                                                  mul_rn(w.z, mul_rn(s1, v[2])), mul_rn(w.w, mul_rn(s1, v[3]))));
                    }
                    float4 xo = make_float4(v[0], v[1], v[2], v[3]);
                    if (has_resid) {
                        const float4 rv = *reinterpret_cast<const float4 *>(base + (size_t)G * L.xstride +
                                                                            (size_t)r * L.rstride + 4 * c);
                        xo = make_float4(add_rn(v[0], rv.x), add_rn(v[1], rv.y), add_rn(v[2], rv.z), add_rn(v[3], rv.w));
                    }
                    if (a.x_out) st4(a.x_out + o, xo);
                    const float4 wf = __ldg(reinterpret_cast<const float4 *>(a.w_final + c));
                    const float s2 = sc[32 + r];
                    y = make_float4(mul_rn(wf.x, mul_rn(s2, xo.x)), mul_rn(wf.y, mul_rn(s2, xo.y)),
                                    mul_rn(wf.z, mul_rn(s2, xo.z)), mul_rn(wf.w, mul_rn(s2, xo.w)));
                }
                float am = fmaxf(fmaxf(fmaxf(0.0f, fabsf(y.x)), fmaxf(0.0f, fabsf(y.y))),
                                 fmaxf(fmaxf(0.0f, fabsf(y.z)), fmaxf(0.0f, fabsf(y.w))));
                am = fmaxf(am, __shfl_xor_sync(kFull, am, 1));
                am = fmaxf(am, __shfl_xor_sync(kFull, am, 2));
                am = fmaxf(am, __shfl_xor_sync(kFull, am, 4));
                if (ok) {
                    const int nb = dim >> 5;
                    const float d = q8_scale(am);
                    const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
                    const uint32_t packed = (uint32_t)(uint8_t)q8_code(mul_rn(y.x, inv)) |
                                            ((uint32_t)(uint8_t)q8_code(mul_rn(y.y, inv)) << 8) |
                                            ((uint32_t)(uint8_t)q8_code(mul_rn(y.z, inv)) << 16) |
                                            ((uint32_t)(uint8_t)q8_code(mul_rn(y.w, inv)) << 24);
                    *reinterpret_cast<uint32_t *>(a.codes + (size_t)row * dim + c) = packed;
                    if ((c4 & 7) == 0) {
                        a.scales[(size_t)row * nb + (c >> 5)] = d;
                        if (a.scales16) a.scales16[(size_t)row * nb + (c >> 5)] = f16_bits(d);
                    }
                }
                step();
            }
            return;
        }
        constexpr int U = 8;
        for (int i = wt; i < total; i += U * nwt) {
            int rs[U], cs[U];
            float4 rv[U];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                rs[k] = r;
                cs[k] = 4 * c4;
                if (has_resid && a.x_out && i + k * nwt < total) rv[k] = ld4(a.resid + (size_t)(r0 + r) * dim + cs[k]);
                step();
            }
#pragma unroll
            for (int k = 0; k < U; ++k) {
                if (i + k * nwt >= total) break;
                const size_t o = (size_t)(r0 + rs[k]) * dim + cs[k];
                float v[4];
                xval(rs[k], cs[k], v);
                if (a.xb) {
                    const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + cs[k]));
                    const float s = sc[rs[k]];
                    st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s, v[0])), mul_rn(w.y, mul_rn(s, v[1])),
                                              mul_rn(w.z, mul_rn(s, v[2])), mul_rn(w.w, mul_rn(s, v[3]))));
                }
                if (a.x_out) {
                    float4 xo = make_float4(v[0], v[1], v[2], v[3]);
                    if (has_resid)
                        xo = make_float4(add_rn(v[0], rv[k].x), add_rn(v[1], rv[k].y), add_rn(v[2], rv[k].z),
                                         add_rn(v[3], rv[k].w));
                    st4(a.x_out + o, xo);
                }
            }
        }
    };

    // The writers' residual rows (read from global memory) are prefetched
    // into L2 one iteration before they are written, so their loads wait on
    // L2 rather than HBM.
    auto prefetch_resid = [&](int g) {  // warp 4
        const int r0 = first_row(g), gr = min(G, a.rows - r0);
        if (lane < gr) bulk_prefetch_l2(a.resid + (size_t)(r0 + lane) * dim, (uint32_t)dim * 4u);
    };
    const bool fetch_resid = has_resid && !stage_resid && a.x_out;

    // warp 4 stages LA = NS - 2 groups ahead of the sums: group i + LA goes
    // into the slot the writers left in iteration i - 1
    constexpr int LA = NS - 2;
    int issued = 0;  // warp 4's count of groups issued
    if (warp == 4)
        while (issued < min(nmine, LA)) issue(issued++);
    for (int i = 0; i <= nmine; ++i) {
        if (warp == 4) {
            if (issued < nmine && issued == i + LA && !__shfl_sync(kFull, s_abort, 0)) issue(issued++);
            if (fetch_resid && i < nmine) prefetch_resid(i);
        } else if (warp == 0) {
            if (i < nmine) sum(i);
        } else if ((warp & 3) != 0) {
            if (i >= 1) write(i - 1);
        }
        __syncthreads();
    }
    if (warp == 4 && lane == 0 && s_abort)
        for (int g = max(0, issued - NS); g < issued; ++g) mbar_wait_bounded(&bars[g % NS], (uint32_t)(g / NS) & 1u);
}

// The norm stage for a few f32 rows (decode): a CTA per row stages the row
// (x + resid with PRE_ADD, written back as x) in shared memory with all its
// loads in flight at once, one thread runs the row's squares left to right
// (reference.rs:167-170) with sixteen values loaded ahead of their adds, and
// the CTA writes xb = w*(scale*x).  Latency: one load round trip, the
// dependent add chain, one store round.  dim % 4 == 0.
template <bool PRE_ADD>
__global__ void __launch_bounds__(256) k_norm_small(ChainArgs a) {
    extern __shared__ __align__(16) float row_s[];
    __shared__ float scale_s;
    const int r = blockIdx.x, dim = a.dim, n4 = dim >> 2;
    const float *xr = a.x_in + (size_t)r * dim;
    float part = 0.0f;  // tolerance mode: this thread's squares
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 v = *reinterpret_cast<const float4 *>(xr + 4 * i);
        if constexpr (PRE_ADD) {
            const float4 rr = *reinterpret_cast<const float4 *>(a.resid + (size_t)r * dim + 4 * i);
            v = make_float4(add_rn(v.x, rr.x), add_rn(v.y, rr.y), add_rn(v.z, rr.z), add_rn(v.w, rr.w));
            *reinterpret_cast<float4 *>(a.x_out + (size_t)r * dim + 4 * i) = v;
        }
        *reinterpret_cast<float4 *>(row_s + 4 * i) = v;
        part = __fmaf_rn(v.x, v.x, __fmaf_rn(v.y, v.y, __fmaf_rn(v.z, v.z, __fmaf_rn(v.w, v.w, part))));
    }
    __syncthreads();
    if (a.tol) {
        // tolerance mode: the squares summed by warps, then the 8 warp sums
        // by thread 0 (dim % 4 == 0: the float4 items cover the row)
        __shared__ float wsum[8];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(kFull, part, o);
        if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x == 0) {
            float ss = 0.0f;
            for (int w8 = 0; w8 < (int)(blockDim.x >> 5); ++w8) ss += wsum[w8];
            scale_s = rms_scale(ss, (float)dim, a.eps);
        }
    } else if (threadIdx.x == 0) {
        float ss = chain_add16(0.0f, dim / 16, [&](int b, float(&q)[16]) { squares16_f32(row_s + 16 * b, q); });
        int i = dim & ~15;
        for (; i < dim; ++i) ss = add_rn(ss, mul_rn(row_s[i], row_s[i]));
        scale_s = rms_scale(ss, (float)dim, a.eps);
    }
    __syncthreads();
    const float sc = scale_s;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = *reinterpret_cast<const float4 *>(row_s + 4 * i);
        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + 4 * i));
        *reinterpret_cast<float4 *>(a.xb + (size_t)r * dim + 4 * i) =
            make_float4(mul_rn(w.x, mul_rn(sc, v.x)), mul_rn(w.y, mul_rn(sc, v.y)), mul_rn(w.z, mul_rn(sc, v.z)),
                        mul_rn(w.w, mul_rn(sc, v.w)));
    }
}

// The embed -> rms_norm pair for a few rows (decode, llama.rs:734-740): a CTA
// per row gathers table row tokens[r], decoded to f32 as Matrix::decode_row
// does (bf16 bits; a Q8_0 code times its block scale, one multiply; f32),
// into shared memory and x, then runs k_norm_small's exact sum and writes xb.
// An out-of-range token reports ERR_TOKEN and reads as zeros, as the
// pipelines do.  dim % 4 == 0 (% 32 for Q8_0).
template <int SRC>
__global__ void __launch_bounds__(256) k_norm_small_emb(ChainArgs a) {
    extern __shared__ __align__(16) float row_s[];
    __shared__ float scale_s;
    const int r = blockIdx.x, dim = a.dim, n4 = dim >> 2;
    const int tok = a.tokens[r];
    const bool valid = (unsigned)tok < (unsigned)a.vocab;
    if (!valid && threadIdx.x == 0) set_err(a.err, ERR_TOKEN);
    float part = 0.0f;  // tolerance mode: this thread's squares
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (valid) {
            if constexpr (SRC == SRC_BF16) {
                const uint2 t = reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(a.table) +
                                                                (size_t)tok * dim)[i];
                v = make_float4(bf16f(t.x & 0xffffu), bf16f(t.x >> 16), bf16f(t.y & 0xffffu), bf16f(t.y >> 16));
            } else if constexpr (SRC == SRC_Q8) {
                const uint32_t t = reinterpret_cast<const uint32_t *>(static_cast<const int8_t *>(a.table) +
                                                                      (size_t)tok * dim)[i];
                const float sc = a.tscales[(size_t)tok * (dim >> 5) + (i >> 3)];
                v = make_float4(mul_rn((float)(int8_t)(t & 0xffu), sc), mul_rn((float)(int8_t)((t >> 8) & 0xffu), sc),
                                mul_rn((float)(int8_t)((t >> 16) & 0xffu), sc), mul_rn((float)(int8_t)(t >> 24), sc));
            } else {
                v = reinterpret_cast<const float4 *>(static_cast<const float *>(a.table) + (size_t)tok * dim)[i];
            }
        }
        if (a.x_out) *reinterpret_cast<float4 *>(a.x_out + (size_t)r * dim + 4 * i) = v;
        *reinterpret_cast<float4 *>(row_s + 4 * i) = v;
        part = __fmaf_rn(v.x, v.x, __fmaf_rn(v.y, v.y, __fmaf_rn(v.z, v.z, __fmaf_rn(v.w, v.w, part))));
    }
    __syncthreads();
    if (a.tol) {
        __shared__ float wsum[8];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(kFull, part, o);
        if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x == 0) {
            float ss = 0.0f;
            for (int w8 = 0; w8 < (int)(blockDim.x >> 5); ++w8) ss += wsum[w8];
            scale_s = rms_scale(ss, (float)dim, a.eps);
        }
    } else if (threadIdx.x == 0) {
        float ss = chain_add16(0.0f, dim / 16, [&](int b, float(&q)[16]) { squares16_f32(row_s + 16 * b, q); });
        int i = dim & ~15;
        for (; i < dim; ++i) ss = add_rn(ss, mul_rn(row_s[i], row_s[i]));
        scale_s = rms_scale(ss, (float)dim, a.eps);
    }
    __syncthreads();
    const float sc = scale_s;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = *reinterpret_cast<const float4 *>(row_s + 4 * i);
        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + 4 * i));
        *reinterpret_cast<float4 *>(a.xb + (size_t)r * dim + 4 * i) =
            make_float4(mul_rn(w.x, mul_rn(sc, v.x)), mul_rn(w.y, mul_rn(sc, v.y)), mul_rn(w.z, mul_rn(sc, v.z)),
                        mul_rn(w.w, mul_rn(sc, v.w)));
    }
}

// The chain's pure streams (RoPE on Q and K, SwiGLU) over all rows: no
// shared memory and few registers, so an SM holds many more warps than the
// norm stage's CTAs allow.  Grid-stride over one flat index space.
template <int U>
__global__ void __launch_bounds__(kThreads) k_stream(ChainArgs a) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x, nt = gridDim.x * blockDim.x;
    if (a.rope_mode == 1) {
        if (a.q) rope_half_rows<U>(a.q, a.q_dim, a.head, a.half, 0, a.rows, a.pos, a.cos_t, a.sin_t, a.max_pos,
                                   a.err, t, nt);
        if (a.k) rope_half_rows<U>(a.k, a.kv_dim, a.head, a.half, 0, a.rows, a.pos, a.cos_t, a.sin_t, a.max_pos,
                                   a.err, t, nt);
    }
    if (a.gate) silu_range<U>(a.gate, a.up, 0, (size_t)a.rows * a.hidden, t, nt);
}

// The norm stage in two passes, for gathered bf16 / f32 embedding rows
// (the Llama chain's embed -> rms_norm, llama.rs:734-740).
//
// Pass 1, k_row_scales: each row's RMSNorm scale (reference.rs:161-173), lane
// r of a one-warp CTA summing row r's squares left to right (the reference's
// order) out of a ring of column tiles that the same warp fills with 16-byte
// cp.async copies, 16 lanes per 256-byte row tile.  Many CTAs per SM keep
// many rows' chains in flight at once.
// Pass 2 is a ticket type of k_stream_dyn that writes xb = w * (scale * v)
// and x = v + resid from the gathered row v (norm_rows_write): balanced with
// the chain's other streams, no pipeline to fill.
constexpr int kScaleSlots = 4;
constexpr int kScaleTile = 256;                // bytes of a row per tile
constexpr int kScaleStride = kScaleTile + 16;  // odd multiple of 16: lane r's reads hit distinct banks
constexpr size_t kScaleSmem = (size_t)kScaleSlots * 32 * kScaleStride;

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// n16 16-byte chunks of a staged row added into ss, left to right.
template <int SRC>
__device__ __forceinline__ void chain_chunk(float &ss, const uint4 u) {
    if constexpr (SRC == SRC_BF16) {
        const float v[8] = {bf16f(u.x & 0xffffu), bf16f(u.x >> 16), bf16f(u.y & 0xffffu), bf16f(u.y >> 16),
                            bf16f(u.z & 0xffffu), bf16f(u.z >> 16), bf16f(u.w & 0xffffu), bf16f(u.w >> 16)};
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = add_rn(ss, mul_rn(v[e], v[e]));
    } else {
        const float v[4] = {__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w)};
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = add_rn(ss, mul_rn(v[e], v[e]));
    }
}

template <int SRC>
__global__ void __launch_bounds__(32) k_row_scales(ChainArgs a, float *row_scale) {
    static_assert(SRC == SRC_BF16 || SRC == SRC_F32, "bf16 or f32 rows");
    constexpr int ESZ = SRC == SRC_BF16 ? 2 : 4;
    constexpr int N16 = kScaleTile / 16;  // chunks of a full tile
    extern __shared__ __align__(16) unsigned char ring_smem[];  // [kScaleSlots][32 * kScaleStride]
    auto ring = [&](int slot) { return ring_smem + (size_t)slot * 32 * kScaleStride; };
    const int lane = threadIdx.x, r0 = blockIdx.x * 32, gr = min(32, a.rows - r0);
    const int rb = a.dim * ESZ;  // a multiple of 16
    const int ntiles = (rb + kScaleTile - 1) / kScaleTile;
    bool valid = false;
    const unsigned char *mine = nullptr;
    if (lane < gr) {
        const int tok = a.tokens[r0 + lane];
        valid = (unsigned)tok < (unsigned)a.vocab;
        if (!valid) set_err(a.err, ERR_TOKEN);
        else mine = static_cast<const unsigned char *>(a.table) + (size_t)tok * rb;
    }
    // Lane l copies chunk (l & 15) of rows 2j + (l >> 4), j < 16: their row
    // addresses stay in registers.
    const unsigned char *src[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
        src[j] = reinterpret_cast<const unsigned char *>(
            __shfl_sync(kFull, reinterpret_cast<unsigned long long>(mine), 2 * j + (lane >> 4)));
    auto issue = [&](int t) {
        const int off = t * kScaleTile + 16 * (lane & 15);
        if (off >= rb) return;
        unsigned char *dst = ring(t % kScaleSlots) + (lane >> 4) * kScaleStride + 16 * (lane & 15);
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (src[j]) cp_async16(dst + 2 * j * kScaleStride, src[j] + off);
    };
#pragma unroll
    for (int t = 0; t < kScaleSlots - 1; ++t) {
        if (t < ntiles) issue(t);
        cp_async_commit();
    }
    float ss = 0.0f;
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait_group<kScaleSlots - 2>();  // this lane's copies of tile t
        __syncwarp();                            // and every lane's
        if (t + kScaleSlots - 1 < ntiles) issue(t + kScaleSlots - 1);  // the slot tile t - 1 used
        cp_async_commit();
        if (valid) {
            const uint4 *row = reinterpret_cast<const uint4 *>(ring(t % kScaleSlots) + lane * kScaleStride);
            const int n16 = min(kScaleTile, rb - t * kScaleTile) >> 4;
            constexpr int EPC = 16 / ESZ;  // elements per 16-byte chunk
            const int elems = n16 * EPC;
            if (elems % 16 == 0) {
                // the squares of the next 16 elements ahead of the current adds
                ss = chain_add16(ss, elems / 16, [&](int b, float(&q)[16]) {
                    if constexpr (SRC == SRC_BF16)
                        squares16_bf16(reinterpret_cast<const uint16_t *>(row) + 16 * b, q);
                    else
                        squares16_f32(reinterpret_cast<const float *>(row) + 16 * b, q);
                });
            } else {
                for (int c = 0; c < n16; ++c) chain_chunk<SRC>(ss, row[c]);
            }
        }
    }
    cp_async_wait_group<0>();
    if (lane < gr) row_scale[r0 + lane] = rms_scale(ss, (float)a.dim, a.eps);
}

// Pass 2's norm rows [r0, r0 + g): v = the gathered row (0 for a token out of
// range, as the norm pipelines use), xb = w * (scale * v), x = v + resid (or
// v), threads t of nt over the rows' float4 items, U items in flight.
template <int SRC, int U>
__device__ void norm_rows_write(const ChainArgs &a, const float *__restrict__ row_scale, int r0, int g, int t,
                                int nt) {
    const int dim = a.dim, q = dim >> 2, n = g * q;
    for (int i = t; i < n; i += U * nt) {
        float4 v[U], rv[U];
        int row[U], c[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int it = i + k * nt;
            row[k] = -1;
            if (it >= n) continue;
            const int r = it / q;
            row[k] = r0 + r;
            c[k] = 4 * (it - r * q);
            const int tok = a.tokens[row[k]];
            v[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if ((unsigned)tok < (unsigned)a.vocab) {
                if constexpr (SRC == SRC_BF16) {
                    const uint2 b = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(a.table) +
                                                                           (size_t)tok * dim + c[k]));
                    v[k] = make_float4(bf16f(b.x & 0xffffu), bf16f(b.x >> 16), bf16f(b.y & 0xffffu), bf16f(b.y >> 16));
                } else {
                    v[k] = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.table) +
                                                                  (size_t)tok * dim + c[k]));
                }
            }
            if (a.resid && a.x_out) rv[k] = ld4(a.resid + (size_t)row[k] * dim + c[k]);
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            if (row[k] < 0) continue;
            const size_t o = (size_t)row[k] * dim + c[k];
            if (a.xb) {
                const float s = row_scale[row[k]];
                const float4 w = __ldg(reinterpret_cast<const float4 *>(a.w_att + c[k]));
                st4(a.xb + o, make_float4(mul_rn(w.x, mul_rn(s, v[k].x)), mul_rn(w.y, mul_rn(s, v[k].y)),
                                          mul_rn(w.z, mul_rn(s, v[k].z)), mul_rn(w.w, mul_rn(s, v[k].w))));
            }
            if (a.x_out) {
                float4 xo = v[k];
                if (a.resid)
                    xo = make_float4(add_rn(xo.x, rv[k].x), add_rn(xo.y, rv[k].y), add_rn(xo.z, rv[k].z),
                                     add_rn(xo.w, rv[k].w));
                st4(a.x_out + o, xo);
            }
        }
    }
}

// The chain's streams with dynamic work.  The work is cut into tickets that
// the CTAs draw in order from a counter, so no CTA is left with a share of the
// work after the others finish (measured on B200 against the grid-stride
// k_stream over the 65 536-row chain: 1.337 -> 1.243 ms).  In ticket order:
//   the norm rows of the two-pass norm stage (NSRC = SRC_BF16 / SRC_F32),
//   kNormRows rows each, last rows first: pass 1 read them last, so they are
//   the likeliest still to be in L2;
//   SwiGLU spans of kSpanElems elements; RoPE spans of kSpanRows rows of q,
//   then of k.
// Every CTA draws exactly one ticket past the end, so the launch draws
// total + gridDim.x tickets; the CTA holding the last one returns the counter
// to zero for the next launch on this stream.
constexpr unsigned kSpanElems = 16384;  // 192 KB of SwiGLU traffic
constexpr int kSpanRows = 4;            // 64 KB of RoPE traffic at width 2048
constexpr int kNormRows = 4;            // 112 KB of norm traffic at hidden 2048

template <int NSRC, int U>
__global__ void __launch_bounds__(kThreads, 5) k_stream_dyn(ChainArgs a, const float *__restrict__ row_scale,
                                                            unsigned n_norm, unsigned n_silu, unsigned n_q,
                                                            unsigned n_k) {
    __shared__ unsigned s_t[2];
    const unsigned total = n_norm + n_silu + n_q + n_k;
    // Ticket `it` of this CTA is in s_t[it & 1]; thread 0 draws ticket it + 1
    // while the CTA works on ticket it.  Tickets rise, so each work type has a
    // loop of its own.
    int it = 0;
    if (threadIdx.x == 0) s_t[0] = atomicAdd(a.ticket, 1u);
    __syncthreads();
    unsigned t = s_t[0];
    auto next = [&]() {
        __syncthreads();
        t = s_t[++it & 1];
    };
    if constexpr (NSRC >= 0) {
        while (t < n_norm) {
            if (threadIdx.x == 0) s_t[(it + 1) & 1] = atomicAdd(a.ticket, 1u);
            const int r0 = (int)(n_norm - 1 - t) * kNormRows;
            norm_rows_write<NSRC, 2>(a, row_scale, r0, min(kNormRows, a.rows - r0), threadIdx.x, blockDim.x);
            next();
        }
    }
    const size_t n = (size_t)a.rows * a.hidden;
    unsigned base = n_norm;
    while (t < base + n_silu) {
        if (threadIdx.x == 0) s_t[(it + 1) & 1] = atomicAdd(a.ticket, 1u);
        const size_t lo = (size_t)(t - base) * kSpanElems;
        silu_range<U>(a.gate, a.up, lo, lo + kSpanElems < n ? lo + kSpanElems : n, threadIdx.x, blockDim.x);
        next();
    }
    base += n_silu;
    while (t < base + n_q) {
        if (threadIdx.x == 0) s_t[(it + 1) & 1] = atomicAdd(a.ticket, 1u);
        const int r0 = (int)(t - base) * kSpanRows;
        rope_half_rows<U>(a.q, a.q_dim, a.head, a.half, r0, min(kSpanRows, a.rows - r0), a.pos, a.cos_t, a.sin_t,
                          a.max_pos, a.err, threadIdx.x, blockDim.x);
        next();
    }
    base += n_q;
    while (t < total) {
        if (threadIdx.x == 0) s_t[(it + 1) & 1] = atomicAdd(a.ticket, 1u);
        const int r0 = (int)(t - base) * kSpanRows;
        rope_half_rows<U>(a.k, a.kv_dim, a.head, a.half, r0, min(kSpanRows, a.rows - r0), a.pos, a.cos_t, a.sin_t,
                          a.max_pos, a.err, threadIdx.x, blockDim.x);
        next();
    }
    if (threadIdx.x == 0 && t == total + gridDim.x - 1) atomicExch(a.ticket, 0u);
}

// --------------------------------------------------------------------------
// Standalone row ops
// --------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads) k_qk_norm(float *v, int rows, int width, int head,
                                                      const float *__restrict__ w, float eps) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    qk_norm_row_warp(v + (size_t)row * width, width, head, w, eps, threadIdx.x & 31);
}

__global__ void __launch_bounds__(kThreads) k_rope(float *q, float *k, int q_width, int kv_width,
                                                   int rows, int head, const int32_t *pos,
                                                   const float *cos_t, const float *sin_t,
                                                   int max_pos, int interleaved, int *err, int wpr) {
    // wpr warps per row: a few rows (decode) still spread over many threads
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int row = gw / wpr;
    const int lane = (gw - row * wpr) * 32 + (threadIdx.x & 31), nl = 32 * wpr;
    if (row >= rows) return;
    const int p = pos[row];
    if ((unsigned)p >= (unsigned)max_pos) {
        if (lane == 0) set_err(err, ERR_POSITION);
        return;
    }
    const int half = head >> 1;
    const float *ct = cos_t + (size_t)p * half, *st = sin_t + (size_t)p * half;
    float *qr = q + (size_t)row * q_width, *kr = k + (size_t)row * kv_width;
    if (!interleaved) {
        const bool vec = ((half | q_width | kv_width) & 3) == 0;
        rope_half_row(qr, q_width / head, head, half, ct, st, vec, lane, nl);
        rope_half_row(kr, kv_width / head, head, half, ct, st, vec, lane, nl);
    } else {
        const bool vec = ((head | q_width | kv_width) & 3) == 0;
        const int kp = k_pairs_interleaved(q_width, kv_width);
        rope_pair_row(qr, q_width / 2, head, ct, st, vec && (q_width / 2) % 2 == 0, lane, nl);
        rope_pair_row(kr, kp, head, ct, st, vec && kp % 2 == 0, lane, nl);
    }
}

// The driver's rope(q, k) then kv_write(layer, slots, k, v) (llama.rs:744-757)
// in one pass: k_rope's half-split rotation, each lane also storing the k
// values it rotated to the row's cache slot, and the v row copied to its slot
// (reference.rs:151-159, 209-257).  kv_width == the cache's kv_dim, a whole
// number of heads.  A row whose position is out of the table reports it and
// still writes its k and v rows unrotated, as the two separate calls would.
__global__ void __launch_bounds__(kThreads) k_rope_kv(float *q, float *k, int q_width, int kv_width, int rows,
                                                      int head, const int32_t *pos, const float *cos_t,
                                                      const float *sin_t, int max_pos, int *err, int wpr,
                                                      const float *v, float *kc, float *vc,
                                                      const int32_t *dst_rows) {
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int row = gw / wpr;
    const int lane = (gw - row * wpr) * 32 + (threadIdx.x & 31), nl = 32 * wpr;
    if (row >= rows) return;
    float *qr = q + (size_t)row * q_width, *kr = k + (size_t)row * kv_width;
    float *kd = kc + (size_t)dst_rows[row] * kv_width, *vd = vc + (size_t)dst_rows[row] * kv_width;
    const float *vr = v + (size_t)row * kv_width;
    const int p = pos[row];
    if ((unsigned)p >= (unsigned)max_pos) {
        if (lane == 0) set_err(err, ERR_POSITION);
        for (int e = lane; e < kv_width; e += nl) kd[e] = kr[e];
    } else {
        const int half = head >> 1;
        const float *ct = cos_t + (size_t)p * half, *st = sin_t + (size_t)p * half;
        const bool vec = ((half | q_width | kv_width) & 3) == 0;
        rope_half_row(qr, q_width / head, head, half, ct, st, vec, lane, nl);
        rope_half_row(kr, kv_width / head, head, half, ct, st, vec, lane, nl, kd);
    }
    if ((kv_width & 3) == 0 && (((uintptr_t)vr | (uintptr_t)vd) & 15) == 0)
        for (int e = lane; e < kv_width / 4; e += nl)
            reinterpret_cast<float4 *>(vd)[e] = reinterpret_cast<const float4 *>(vr)[e];
    else
        for (int e = lane; e < kv_width; e += nl) vd[e] = vr[e];
}

// The driver's qk_norm(q), qk_norm(k), rope(q, k) sequence (llama.rs:744-754)
// in one pass per row: one warp per row normalises each head (reference.rs
// :180-207) and rotates it (reference.rs:209-257).  Either norm weight may
// be null (that vector is only rotated).
__global__ void __launch_bounds__(kThreads) k_qk_rope(float *q, float *k, int q_width, int kv_width, int rows,
                                                      int head, const float *wq, const float *wk, float eps,
                                                      const int32_t *pos, const float *cos_t, const float *sin_t,
                                                      int max_pos, int interleaved, int *err) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float *qr = q + (size_t)row * q_width, *kr = k + (size_t)row * kv_width;
    if (wq) qk_norm_row_warp(qr, q_width, head, wq, eps, lane);
    if (wk) qk_norm_row_warp(kr, kv_width, head, wk, eps, lane);
    const int p = pos[row];
    if ((unsigned)p >= (unsigned)max_pos) {
        if (lane == 0) set_err(err, ERR_POSITION);
        return;
    }
    const int half = head >> 1;
    const float *ct = cos_t + (size_t)p * half, *st = sin_t + (size_t)p * half;
    if (!interleaved) {
        const bool vec = ((half | q_width | kv_width) & 3) == 0;
        rope_half_row(qr, q_width / head, head, half, ct, st, vec, lane);
        rope_half_row(kr, kv_width / head, head, half, ct, st, vec, lane);
    } else {
        const bool vec = ((head | q_width | kv_width) & 3) == 0;
        const int kp = k_pairs_interleaved(q_width, kv_width);
        rope_pair_row(qr, q_width / 2, head, ct, st, vec && (q_width / 2) % 2 == 0, lane);
        rope_pair_row(kr, kp, head, ct, st, vec && kp % 2 == 0, lane);
    }
}

// Row-staged forms of qk_norm, qk_norm+RoPE and the chain's q/k stream: one
// warp per row (grid-stride over rows), each warp with `smf` floats of
// dynamic shared memory (qk_rope_row_smem).
__global__ void __launch_bounds__(kThreads) k_qk_norm_smem(float *v, int rows, int width, int head,
                                                           const float *__restrict__ w, float eps, int smf) {
    extern __shared__ __align__(16) float qsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *sm = qsm + warp * smf;
    const int wpb = blockDim.x >> 5;
    for (int row = blockIdx.x * wpb + warp; row < rows; row += gridDim.x * wpb)
        qk_rope_row_smem(v + (size_t)row * width, width, head, w, eps, nullptr, nullptr, 0, 0, sm, lane);
}

__global__ void __launch_bounds__(kThreads) k_qk_rope_smem(float *q, float *k, int q_width, int kv_width, int rows,
                                                           int head, const float *wq, const float *wk, float eps,
                                                           const int32_t *pos, const float *cos_t,
                                                           const float *sin_t, int max_pos, int interleaved,
                                                           int *err, int smf) {
    extern __shared__ __align__(16) float qsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *sm = qsm + warp * smf;
    const int wpb = blockDim.x >> 5, half = head >> 1;
    const int mode = interleaved ? 2 : 1;
    const int kp = k_pairs_interleaved(q_width, kv_width);
    for (int row = blockIdx.x * wpb + warp; row < rows; row += gridDim.x * wpb) {
        const int p = pos[row];
        const bool ok = (unsigned)p < (unsigned)max_pos;
        if (!ok && lane == 0) set_err(err, ERR_POSITION);
        const float *ct = ok ? cos_t + (size_t)p * half : nullptr;
        const float *st = ok ? sin_t + (size_t)p * half : nullptr;
        // an out-of-table position still gets its norm; the rotation is skipped
        qk_rope_row_smem(q + (size_t)row * q_width, q_width, head, wq, eps, ct, st, ok ? mode : 0, q_width / 2, sm,
                         lane);
        qk_rope_row_smem(k + (size_t)row * kv_width, kv_width, head, wk, eps, ct, st, ok ? mode : 0, kp, sm, lane);
    }
}

// The chain's streams when q/k carry per-head norms (Qwen3, LFM2): the q/k
// rows through qk_rope_row_smem, then SwiGLU over all rows.
__global__ void __launch_bounds__(kThreads) k_stream_qk(ChainArgs a, int smf) {
    extern __shared__ __align__(16) float qsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *sm = qsm + warp * smf;
    const int wpb = blockDim.x >> 5;
    const int kp = k_pairs_interleaved(a.q_dim, a.kv_dim);
    if (a.q || a.k) {
        for (int row = blockIdx.x * wpb + warp; row < a.rows; row += gridDim.x * wpb) {
            const float *ct = nullptr, *st = nullptr;
            int mode = 0;
            if (a.rope_mode) {
                const int p = a.pos[row];
                if ((unsigned)p < (unsigned)a.max_pos) {
                    ct = a.cos_t + (size_t)p * a.half;
                    st = a.sin_t + (size_t)p * a.half;
                    mode = a.rope_mode;
                } else if (lane == 0) {
                    set_err(a.err, ERR_POSITION);
                }
            }
            if (a.q)
                qk_rope_row_smem(a.q + (size_t)row * a.q_dim, a.q_dim, a.head, a.w_q, a.eps, ct, st, mode,
                                 a.q_dim / 2, sm, lane);
            if (a.k)
                qk_rope_row_smem(a.k + (size_t)row * a.kv_dim, a.kv_dim, a.head, a.w_k, a.eps, ct, st, mode, kp, sm,
                                 lane);
        }
    }
    if (a.gate)
        silu_range<2>(a.gate, a.up, 0, (size_t)a.rows * a.hidden, blockIdx.x * blockDim.x + threadIdx.x,
                      gridDim.x * blockDim.x);
}

// A run of `count` mul calls (reference.rs:315-363) with fixed strides between
// consecutive calls' offsets, as the LFM2 driver issues once per row
// (lfm2.rs:586-596, 612-622).  The host only batches runs whose output buffer
// is not an operand, so the calls are independent.
__global__ void __launch_bounds__(kThreads) k_mul_strided(float *out, const float *a, const float *b, long long so,
                                                          long long sa, long long sb, int len, int count) {
    const long long n = (long long)len * count;
    const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long nt = (long long)gridDim.x * blockDim.x;
    const bool vec = (((uintptr_t)out | (uintptr_t)a | (uintptr_t)b) & 15) == 0 && ((so | sa | sb | len) & 3) == 0;
    if (vec) {
        const int l4 = len >> 2;
        const long long n4 = (long long)l4 * count;
        for (long long e = t; e < n4; e += nt) {
            const long long i = e / l4;
            const int j = (int)(e - i * l4) << 2;
            const float4 x = *reinterpret_cast<const float4 *>(a + i * sa + j);
            const float4 y = *reinterpret_cast<const float4 *>(b + i * sb + j);
            *reinterpret_cast<float4 *>(out + i * so + j) =
                make_float4(mul_rn(x.x, y.x), mul_rn(x.y, y.y), mul_rn(x.z, y.z), mul_rn(x.w, y.w));
        }
    } else {
        for (long long e = t; e < n; e += nt) {
            const long long i = e / len;
            const int j = (int)(e - i * len);
            out[i * so + j] = mul_rn(a[i * sa + j], b[i * sb + j]);
        }
    }
}

__global__ void __launch_bounds__(kThreads) k_silu_mul(float *g, const float *u, size_t n) {
    silu_range<4>(g, u, 0, n, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// reference.rs:308-313
__global__ void __launch_bounds__(kThreads) k_add(float *__restrict__ d, const float *__restrict__ s,
                                                  size_t n) {
    const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nt = (size_t)gridDim.x * blockDim.x;
    if ((n & 3) == 0) {
        for (size_t i = 4 * t; i < n; i += 4 * nt) {
            float4 a = ld4(d + i);
            const float4 b = ld4(s + i);
            a.x = add_rn(a.x, b.x); a.y = add_rn(a.y, b.y); a.z = add_rn(a.z, b.z); a.w = add_rn(a.w, b.w);
            st4(d + i, a);
        }
    } else {
        for (size_t i = t; i < n; i += nt) d[i] = add_rn(d[i], s[i]);
    }
}

// reference.rs:315-363.  Parallel when no thread's write can feed another
// thread's read; otherwise the sequential variant keeps the reference order.
__global__ void __launch_bounds__(kThreads) k_mul(float *o, const float *a, const float *b, size_t n) {
    const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nt = (size_t)gridDim.x * blockDim.x;
    const bool vec = (((uintptr_t)o | (uintptr_t)a | (uintptr_t)b) & 15) == 0 && (n & 3) == 0;
    if (vec) {
        for (size_t i = 4 * t; i < n; i += 4 * nt) {
            const float4 x = *reinterpret_cast<const float4 *>(a + i);
            const float4 y = *reinterpret_cast<const float4 *>(b + i);
            *reinterpret_cast<float4 *>(o + i) =
                make_float4(mul_rn(x.x, y.x), mul_rn(x.y, y.y), mul_rn(x.z, y.z), mul_rn(x.w, y.w));
        }
    } else {
        for (size_t i = t; i < n; i += nt) {
            const float x = a[i], y = b[i];
            o[i] = mul_rn(x, y);
        }
    }
}

__global__ void k_mul_sequential(float *o, const float *a, const float *b, size_t n) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    for (size_t i = 0; i < n; ++i) {
        const float x = a[i], y = b[i];
        o[i] = mul_rn(x, y);
    }
}

// reference.rs:490-503 conv_rows, one thread per (row, channel).
__global__ void __launch_bounds__(kThreads) k_conv_prefill(float *__restrict__ out,
                                                           const float *__restrict__ x,
                                                           const float *__restrict__ w, int rows,
                                                           int dim, int k) {
    const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (idx >= (size_t)rows * dim) return;
    const int r = (int)(idx / dim), i = (int)(idx - (size_t)r * dim);
    float acc = 0.0f;
    for (int j = 0; j < k; ++j) {
        const int h = r - (k - 1) + j;
        if (h >= 0) acc = add_rn(acc, mul_rn(__ldg(w + (size_t)i * k + j), __ldg(x + (size_t)h * dim + i)));
    }
    out[idx] = acc;
}

// reference.rs:372-393: one thread per channel; every read precedes every
// write of that channel, so out may alias x.
__global__ void __launch_bounds__(kThreads) k_conv_decode(float *out, const float *x,
                                                          const float *__restrict__ w,
                                                          float *state, int dim, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    const float xi = x[i];
    float acc = 0.0f;
    for (int j = 0; j < k - 1; ++j) acc = add_rn(acc, mul_rn(w[(size_t)i * k + j], state[(size_t)j * dim + i]));
    acc = add_rn(acc, mul_rn(w[(size_t)i * k + (k - 1)], xi));
    out[i] = acc;
    if (k > 1) {
        for (int j = 0; j + 1 < k - 1; ++j) state[(size_t)j * dim + i] = state[(size_t)(j + 1) * dim + i];
        state[(size_t)(k - 2) * dim + i] = xi;
    }
}

// lfm2.rs:584-624 conv block fused: h = B*x recomputed for the k-1 halo rows,
// co = conv(h) in tap order, cy = C*co, ring <- the last k-1 rows of h.
__global__ void __launch_bounds__(kThreads) k_lfm2_conv_block(const float *__restrict__ bcx,
                                                              const float *__restrict__ w,
                                                              float *__restrict__ ring,
                                                              float *__restrict__ cy, int lead, int rows,
                                                              int dim, int k) {
    // output element idx: bcx row lead + idx / dim (the first `lead` rows are
    // a shard's halo, as in k_lfm2_conv_block_tiled)
    const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (idx >= (size_t)(rows - lead) * dim) return;
    const int r = lead + (int)(idx / dim), i = (int)(idx - (size_t)(r - lead) * dim);
    const size_t w3 = (size_t)3 * dim;
    float acc = 0.0f, hr = 0.0f;
    for (int j = 0; j < k; ++j) {
        const int h = r - (k - 1) + j;
        if (h >= 0) {
            const float hv = mul_rn(__ldg(bcx + h * w3 + i), __ldg(bcx + h * w3 + 2 * dim + i));
            acc = add_rn(acc, mul_rn(__ldg(w + (size_t)i * k + j), hv));
            if (h == r) hr = hv;
        }
    }
    cy[idx] = mul_rn(__ldg(bcx + r * w3 + dim + i), acc);
    if (ring && k > 1) {
        const int take = min(rows, k - 1);
        if (r >= rows - take) ring[(size_t)(k - 1 - take + (r - (rows - take))) * dim + i] = hr;
    }
}

// The row-tiled forms of the two convolutions for the kernel sizes the
// models use (K = 2..4).  A thread owns V adjacent channels over RT
// consecutive rows: it loads the K-1 halo rows and its RT rows once, all
// loads issued before any arithmetic, then runs each output's taps in the
// reference's order from registers.  Channels are the fastest-varying thread
// index, so a warp's loads of one row are contiguous, and the halo rows a
// tile re-reads were fetched by its neighbour tile moments earlier (L2).
template <int V>
__device__ __forceinline__ void ldv(const float *p, float *v) {
    if constexpr (V == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
        v[0] = __ldg(p);
    }
}
template <int V>
__device__ __forceinline__ void stv(float *p, const float *v) {
    if constexpr (V == 4) *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    else p[0] = v[0];
}

// reference.rs:490-503 conv_rows.
template <int K, int V, int RT>
__global__ void __launch_bounds__(kThreads) k_conv_prefill_tiled(float *__restrict__ out,
                                                                 const float *__restrict__ x,
                                                                 const float *__restrict__ w, int rows,
                                                                 int dim) {
    const int ncg = dim / V;
    const unsigned t = blockIdx.x * blockDim.x + threadIdx.x;
    const int tile = (int)(t / (unsigned)ncg), c = (int)(t - (unsigned)tile * ncg) * V;
    const int r0 = tile * RT;
    if (r0 >= rows) return;
    float wk[V][K];
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < K; ++j) wk[v][j] = __ldg(w + (size_t)(c + v) * K + j);
    // xs[q] holds row r0 - (K-1) + q.
    float xs[RT + K - 1][V];
#pragma unroll
    for (int q = 0; q < RT + K - 1; ++q) {
        const int h = r0 - (K - 1) + q;
        if (h >= 0 && h < rows) ldv<V>(x + (size_t)h * dim + c, xs[q]);
    }
#pragma unroll
    for (int q = 0; q < RT; ++q) {
        const int r = r0 + q;
        if (r >= rows) break;
        float o[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < K; ++j)
                if (r - (K - 1) + j >= 0) acc = add_rn(acc, mul_rn(wk[v][j], xs[q + j][v]));
            o[v] = acc;
        }
        stv<V>(out + (size_t)r * dim + c, o);
    }
}

// lfm2.rs:584-624, row-tiled: h = B*x for the tile's rows and its halo, the
// taps in order, cy = C*co, and the last k-1 rows of h into the ring.  The
// first `lead` (< K) rows of bcx are a shard's halo: they feed h of the rows
// after them and give no output (cy row r - lead for bcx row r); zero padding
// applies before bcx row 0.
template <int K, int V, int RT>
__global__ void __launch_bounds__(kThreads) k_lfm2_conv_block_tiled(const float *__restrict__ bcx,
                                                                    const float *__restrict__ w,
                                                                    float *__restrict__ ring,
                                                                    float *__restrict__ cy, int lead, int rows,
                                                                    int dim) {
    const int ncg = dim / V;
    const unsigned t = blockIdx.x * blockDim.x + threadIdx.x;
    const int tile = (int)(t / (unsigned)ncg), c = (int)(t - (unsigned)tile * ncg) * V;
    const int r0 = lead + tile * RT;
    if (r0 >= rows) return;
    const size_t w3 = (size_t)3 * dim;
    float wk[V][K];
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < K; ++j) wk[v][j] = __ldg(w + (size_t)(c + v) * K + j);
    float bs[RT + K - 1][V], xs[RT + K - 1][V], cs[RT][V];
#pragma unroll
    for (int q = 0; q < RT + K - 1; ++q) {
        const int h = r0 - (K - 1) + q;
        if (h >= 0 && h < rows) {
            ldv<V>(bcx + (size_t)h * w3 + c, bs[q]);
            ldv<V>(bcx + (size_t)h * w3 + 2 * dim + c, xs[q]);
        }
        if (q >= K - 1 && h < rows) ldv<V>(bcx + (size_t)h * w3 + dim + c, cs[q - (K - 1)]);
    }
    float hs[RT + K - 1][V];
#pragma unroll
    for (int q = 0; q < RT + K - 1; ++q)
#pragma unroll
        for (int v = 0; v < V; ++v) hs[q][v] = mul_rn(bs[q][v], xs[q][v]);
    const int take = min(rows, K - 1);
#pragma unroll
    for (int q = 0; q < RT; ++q) {
        const int r = r0 + q;
        if (r >= rows) break;
        float o[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < K; ++j)
                if (r - (K - 1) + j >= 0) acc = add_rn(acc, mul_rn(wk[v][j], hs[q + j][v]));
            o[v] = mul_rn(cs[q][v], acc);
        }
        stv<V>(cy + (size_t)(r - lead) * dim + c, o);
        if (ring && r >= rows - take) stv<V>(ring + (size_t)(K - 1 - take + (r - (rows - take))) * dim + c, hs[q + K - 1]);
    }
}

// quant.rs:856-874 per row: one warp per row, lane l holds element 32b+l.
__global__ void __launch_bounds__(kThreads) k_quantize_q8(const float *__restrict__ x, int rows, int dim,
                                                          int8_t *codes, float *scales,
                                                          uint16_t *scales16) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int nb = (dim + 31) >> 5;
    for (int b = 0; b < nb; ++b) {
        const int i = b * 32 + lane;
        const bool ok = i < dim;
        const float y = ok ? x[(size_t)row * dim + i] : 0.0f;
        float am = fmaxf(0.0f, fabsf(y));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(kFull, am, off));
        const float d = q8_scale(am);
        const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
        codes[(size_t)row * nb * 32 + i] = ok ? q8_code(mul_rn(y, inv)) : (int8_t)0;
        if (lane == 0) {
            scales[(size_t)row * nb + b] = d;
            if (scales16) scales16[(size_t)row * nb + b] = f16_bits(d);
        }
    }
}

// The same quantisation for rows of whole 32-element blocks.  With dim a
// multiple of 32 the blocks of all rows are contiguous, so float4 item i
// holds elements 4i..4i+3 of block i/8 and its codes go to bytes 4i..4i+3:
// the kernel is one flat stream with no row arithmetic.  Eight lanes per
// block, the block amax over the 8-lane group (the loop is warp-uniform so
// every lane reaches the shuffles); each lane loads U items before any
// arithmetic, so U loads per lane are in flight.
template <int U>
__global__ void __launch_bounds__(kThreads) k_quantize_q8v(const float *__restrict__ x, size_t items,
                                                           int8_t *codes, float *scales, uint16_t *scales16) {
    const unsigned lane = threadIdx.x & 31;
    const size_t warp0 = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
    for (size_t base = warp0 * 32 * U; base < items; base += nwarps * 32 * U) {
        float4 y[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const size_t idx = base + 32 * k + lane;
            y[k] = idx < items ? ld4(x + 4 * idx) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const size_t idx = base + 32 * k + lane;
            float am = fmaxf(fmaxf(fmaxf(0.0f, fabsf(y[k].x)), fmaxf(0.0f, fabsf(y[k].y))),
                             fmaxf(fmaxf(0.0f, fabsf(y[k].z)), fmaxf(0.0f, fabsf(y[k].w))));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 1));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 2));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 4));
            if (idx >= items) continue;
            const float d = q8_scale(am);
            const float inv = d > 0.0f ? q8_inv(d) : 0.0f;
            const uint32_t packed = (uint32_t)(uint8_t)q8_code(mul_rn(y[k].x, inv)) |
                                    ((uint32_t)(uint8_t)q8_code(mul_rn(y[k].y, inv)) << 8) |
                                    ((uint32_t)(uint8_t)q8_code(mul_rn(y[k].z, inv)) << 16) |
                                    ((uint32_t)(uint8_t)q8_code(mul_rn(y[k].w, inv)) << 24);
            reinterpret_cast<uint32_t *>(codes)[idx] = packed;
            if ((idx & 7) == 0) {
                scales[idx >> 3] = d;
                if (scales16) scales16[idx >> 3] = f16_bits(d);
            }
        }
    }
}

// k_quantize_q8v with eight elements per lane (x 32-byte aligned, codes
// 8-byte aligned): one 256-bit load per lane, four lanes per block, two
// shuffle rounds, the block arithmetic once per eight elements, the branchless
// reciprocal and the clamp only for blocks whose 1/d overflows.  `items`
// counts octets.
template <int U>
__global__ void __launch_bounds__(kThreads) k_quantize_q8v8(const float *__restrict__ x, size_t items,
                                                            int8_t *codes, float *scales, uint16_t *scales16) {
    const unsigned lane = threadIdx.x & 31;
    const size_t warp0 = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
    for (size_t base = warp0 * 32 * U; base < items; base += nwarps * 32 * U) {
        float y[U][8];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const size_t idx = base + 32 * k + lane;
            if (idx < items) {
                ld8_stream(x + 8 * idx, y[k]);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) y[k][e] = 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const size_t idx = base + 32 * k + lane;
            const float m01 = fmaxf(fabsf(y[k][0]), fabsf(y[k][1])), m23 = fmaxf(fabsf(y[k][2]), fabsf(y[k][3]));
            const float m45 = fmaxf(fabsf(y[k][4]), fabsf(y[k][5])), m67 = fmaxf(fabsf(y[k][6]), fabsf(y[k][7]));
            float am = fmaxf(0.0f, fmaxf(fmaxf(m01, m23), fmaxf(m45, m67)));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 1));
            am = fmaxf(am, __shfl_xor_sync(kFull, am, 2));
            if (idx >= items) continue;
            const float d = q8_scale(am);
            const float inv = q8_inv_block(d);
            int c[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) c[e] = q8_round(mul_rn(y[k][e], inv));
            if (q8_needs_clamp(d)) {
#pragma unroll
                for (int e = 0; e < 8; ++e) c[e] = max(-127, min(127, c[e]));
            }
            const uint32_t lo = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
            const uint32_t hi = __byte_perm(__byte_perm(c[4], c[5], 0x0040), __byte_perm(c[6], c[7], 0x0040), 0x5410);
            __stcs(reinterpret_cast<uint2 *>(codes) + idx, make_uint2(lo, hi));
            if ((idx & 3) == 0) {
                scales[idx >> 2] = d;
                if (scales16) scales16[idx >> 2] = f16_bits(d);
            }
        }
    }
}

// quant.rs:198-220 Q8_0x4::to_row_major with quant.rs:764-769's widening.
__device__ __forceinline__ float f16_scale_to_f32(uint16_t bits) {
    const uint32_t sign = (uint32_t)(bits >> 15) << 31;
    const uint32_t exp = (bits >> 10) & 0x1fu;
    const uint32_t mant = bits & 0x03ffu;
    return __uint_as_float(sign | ((exp + 112u) << 23) | (mant << 13));
}

// Self-test of the bounded waits the pipelines use: one thread waits on an
// mbarrier phase that nothing completes for at most `limit` SM cycles and
// reports ERR_TIMEOUT through the error word, as a pipeline's wait would;
// with `complete` set it first completes the phase itself and the wait ends
// at once.  No copy is in flight, so giving up leaves nothing behind.
__global__ void k_wait_selftest(int *err, long long limit, int complete) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    mbar_fence_init();
    if (complete) mbar_arrive(&bar);
    if (!mbar_wait_bounded(&bar, 0u, limit)) set_err(err, ERR_TIMEOUT);
}

// src/formats/safetensors.rs:365-385 f16_to_f32_local: IEEE binary16 to
// binary32.  A subnormal m * 2^-24 (m < 1024) is exact in f32, which is what
// the reference's normalising loop produces; NaN keeps its payload bits.
__device__ __forceinline__ float f16_to_f32_exact(uint16_t bits) {
    const uint32_t sign = (uint32_t)(bits >> 15) << 31;
    const uint32_t exp = (bits >> 10) & 0x1fu, mant = bits & 0x3ffu;
    if (exp == 0) return __uint_as_float(sign | __float_as_uint(__uint2float_rn(mant) * 0x1p-24f));
    if (exp == 0x1f) return __uint_as_float(sign | 0x7f800000u | (mant << 13));
    return __uint_as_float(sign | ((exp + 112u) << 23) | (mant << 13));
}

__global__ void __launch_bounds__(kThreads) k_widen_f32(int dtype, const uint16_t *__restrict__ src,
                                                        float *__restrict__ dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = dtype == 1 ? bf16f(src[i]) : f16_to_f32_exact(src[i]);
}

// hf.rs:182-188: (v.to_bits() >> 16) as u16, truncation (not rounding)
__global__ void __launch_bounds__(kThreads) k_narrow_bf16(const float *__restrict__ src, uint16_t *__restrict__ dst,
                                                          size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = (uint16_t)(__float_as_uint(src[i]) >> 16);
}

__global__ void __launch_bounds__(kThreads) k_f16_scales_to_f32(const uint16_t *__restrict__ src,
                                                                float *__restrict__ dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = f16_scale_to_f32(src[i]);
}

__global__ void __launch_bounds__(kThreads) k_q8x4_to_row_major(const uint8_t *__restrict__ blocks,
                                                                int out_dim, int in_dim,
                                                                int8_t *quants, float *scales) {
    const int nb = in_dim >> 5;
    const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;  // (group, block, rig)
    if (idx >= (size_t)out_dim * nb) return;
    const int rig = (int)(idx & 3);
    const size_t gb = idx >> 2;
    const int g = (int)(gb / nb), b = (int)(gb - (size_t)g * nb);
    const uint8_t *blk = blocks + gb * 136;
    const uint16_t sbits = (uint16_t)(blk[2 * rig] | (blk[2 * rig + 1] << 8));
    const int row = g * 4 + rig;
    scales[(size_t)row * nb + b] = f16_scale_to_f32(sbits);
    int8_t *dst = quants + (size_t)row * in_dim + b * 32;
    const int8_t *qs = reinterpret_cast<const int8_t *>(blk + 8);
    for (int seg = 0; seg < 8; ++seg)
        for (int lane = 0; lane < 4; ++lane) dst[seg * 4 + lane] = qs[seg * 16 + rig * 4 + lane];
}

inline unsigned grid_for(size_t work, unsigned per_block) {
    size_t b = (work + per_block - 1) / per_block;
    if (b < 1) b = 1;
    if (b > 0x7fffffffull) b = 0x7fffffffull;
    return (unsigned)b;
}

inline unsigned stream_grid(size_t n_elems) {
    // enough CTAs to cover the SMs several times over, capped by the work
    size_t want = (n_elems + 4 * kThreads - 1) / (4 * kThreads);
    if (want > 148 * 16) want = 148 * 16;
    if (want < 1) want = 1;
    return (unsigned)want;
}

template <int SRC>
ChainLayout chain_layout(const ChainArgs &a, bool fq, int G_override) {
    ChainLayout L{};
    const int rb = SRC == SRC_BF16 ? a.dim * 2 : (SRC == SRC_Q8 ? a.dim : a.dim * 4);
    L.xstride = align16(rb) + (SRC == SRC_Q8 ? align16((a.dim / 32) * 4) : 0) + 16;
    L.rstride = (fq && a.resid) ? align16(a.dim * 4) + 16 : 0;
    const int per_row = L.xstride + L.rstride;
    // At most what lets three CTAs share an SM's shared memory (and 32, the
    // lanes of the summing warp); fewer when the rows would otherwise fill
    // under four waves of CTAs.
    int G = (int)((72 * 1024 - 256) / per_row);
    if (G > 32) G = 32;
    static const int env_g = [] {
        const char *e = std::getenv("KERNRT_CHAIN_ROWS_PER_CTA");
        return e ? std::atoi(e) : 0;
    }();
    if (G_override <= 0 && env_g > 0) G_override = env_g < G ? env_g : G;
    if (G_override > 0) {
        G = G_override;
    } else {
        int sms = 148;
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const long want = ((long)a.rows + (long)sms * 3 * 4 - 1) / ((long)sms * 3 * 4);
        if (want < G) G = (int)want;
    }
    if (G < 1) G = 1;
    L.G = G;
    L.smem = (size_t)G * per_row + 64 * sizeof(float);
    return L;
}

template <int SRC, bool FQ, bool VEC>
cudaError_t launch_chain_t(const ChainArgs &a, cudaStream_t s) {
    const ChainLayout L = chain_layout<SRC>(a, FQ, 0);
    if (L.smem > 227 * 1024) return cudaErrorInvalidValue;
    auto kern = k_chain<SRC, FQ, VEC>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem);
    if (e != cudaSuccess) return e;
    const unsigned grid = grid_for((size_t)a.rows, (unsigned)L.G);
    kern<<<grid, kThreads, L.smem, s>>>(a, L);
    return launched();
}


// Warps per CTA and grid for the row-staged q/k kernels; 0 warps when a row
// does not fit, so the caller keeps the unstaged form.
struct QkLaunch {
    int warps = 0, smf = 0;
    size_t smem = 0;
    unsigned grid = 0;
};

template <class K>
QkLaunch qk_launch_config(K kern, int width, int head, int rows) {
    QkLaunch c;
    if (head <= 0 || (head & 3) || (width & 3)) return c;
    c.smf = qk_smem_floats(width, head);
    const size_t per_warp = (size_t)c.smf * sizeof(float);
    if (per_warp == 0) return c;
    int warps = (int)((200 * 1024) / per_warp);
    if (warps > kThreads / 32) warps = kThreads / 32;
    if (warps < 1) return c;
    c.warps = warps;
    c.smem = per_warp * warps;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem) != cudaSuccess) {
        cudaGetLastError();
        c.warps = 0;
        return c;
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, warps * 32, c.smem);
    long grid = (long)device_sms() * (per_sm > 0 ? per_sm : 1);
    const long need = (rows + warps - 1) / warps;
    c.grid = (unsigned)(grid < need ? grid : need);
    if (c.grid == 0) c.grid = 1;
    return c;
}

// The norm stage as the persistent pipeline, one CTA per SM: rows per group
// from the SM's shared memory, fewer when the rows would give a CTA under
// eight groups.  Contiguous f32 rows are re-read by the writers (two slots);
// gathered or quantising rows are written from their slot (three).
template <int SRC, bool VEC, bool PRE_ADD = false, bool FQ = false>
cudaError_t launch_norm_pipe(const ChainArgs &a, cudaStream_t s) {
    constexpr bool RR = SRC == SRC_X && !FQ;
    constexpr int NS = RR ? 2 : 3;
    ChainLayout L{};
    const int rb = SRC == SRC_BF16 ? a.dim * 2 : (SRC == SRC_Q8 ? a.dim : a.dim * 4);
    L.xstride = align16(rb) + (SRC == SRC_Q8 ? align16((a.dim / 32) * 4) : 0) + 16;
    L.rstride = (FQ && a.resid) ? align16(a.dim * 4) + 16 : 0;
    const size_t budget = 224 * 1024 - NS * 64 * sizeof(float);
    int G = (int)(budget / (NS * (size_t)(L.xstride + L.rstride)));
    if (G > 32) G = 32;
    if (G < 1) G = 1;
    const int sms = device_sms();
    const long want = ((long)a.rows + (long)sms * 8 - 1) / ((long)sms * 8);
    if (want < G) G = (int)(want > 0 ? want : 1);
    L.G = G;
    L.smem = NS * (size_t)G * (L.xstride + L.rstride) + NS * 64 * sizeof(float);
    if (L.smem > 227 * 1024) return cudaErrorInvalidValue;
    auto kern = k_norm_pipe<SRC, VEC, PRE_ADD, FQ, RR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPipeThreads, L.smem);
    if (e != cudaSuccess) return e;
    const long groups = ((long)a.rows + G - 1) / G;
    long grid = (long)sms * (per_sm > 0 ? per_sm : 1);
    if (grid > groups) grid = groups;
    kern<<<(unsigned)grid, kPipeThreads, L.smem, s>>>(a, L);
    return launched();
}

// The column-tiled norm pipeline where its bulk copies apply: every staged
// address and size 16-byte aligned (dim % 8, % 32 when quantising, % 128 for
// Q8_0 sources), so every tile boundary is too.  Rows per group come from
// the L2 the writers' re-reads may hold (48 MB over all CTAs, two groups
// each), the tile width from the shared memory of three slots.  Returns
// false (nothing launched) where it does not apply.
inline bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// A CTA per row for a few contiguous f32 rows (fewer than half the SMs):
// shorter than any pipeline's fill.  rms_norm (xb only) or, with PRE_ADD, the
// add_in_place -> rms_norm pair; 16-byte aligned rows that fit in 48 KB.
template <bool PRE_ADD>
bool try_norm_small(const ChainArgs &a, cudaStream_t s, cudaError_t *err) {
    if (a.rows <= 0 || a.rows * 2 > device_sms() || a.dim <= 0 || a.dim % 4 || a.dim > 12288) return false;
    if (!a.xb || (!PRE_ADD && a.x_out) || (PRE_ADD && (!a.resid || !a.x_out)) || a.w_final) return false;
    if (!al16(a.x_in) || !al16(a.xb) || !al16(a.w_att) || (PRE_ADD && (!al16(a.resid) || !al16(a.x_out))))
        return false;
    k_norm_small<PRE_ADD><<<(unsigned)a.rows, 256, (size_t)a.dim * sizeof(float), s>>>(a);
    *err = launched();
    return true;
}

// A CTA per row for a few embed -> rms_norm rows (fewer than half the SMs).
template <int SRC>
bool try_norm_small_emb(const ChainArgs &a, cudaStream_t s, cudaError_t *err) {
    if (a.rows <= 0 || a.rows * 2 > device_sms() || a.dim <= 0 || a.dim % (SRC == SRC_Q8 ? 32 : 4) ||
        a.dim > 12288)
        return false;
    if (!a.xb || !a.tokens || a.resid || a.w_final || !al16(a.table) || !al16(a.xb) || !al16(a.w_att) ||
        (a.x_out && !al16(a.x_out)) || (SRC == SRC_Q8 && !a.tscales))
        return false;
    k_norm_small_emb<SRC><<<(unsigned)a.rows, 256, (size_t)a.dim * sizeof(float), s>>>(a);
    *err = launched();
    return true;
}

// The decoupled column-tiled pipeline for f32 x rows (dim % 8, % 32 when
// quantising; 16-byte aligned rows).  Returns false (nothing launched) when it
// does not apply.
template <bool PRE_ADD, bool FQ>
bool try_norm_cols(const ChainArgs &a, cudaStream_t s, cudaError_t *err) {
    const int gran = FQ ? 32 : 8;
    if (a.rows <= 0 || a.dim <= 0 || a.dim % gran) return false;
    if (!al16(a.x_in) || (a.resid && !al16(a.resid)) || (a.x_out && !al16(a.x_out)) || (a.xb && !al16(a.xb)) ||
        (a.w_att && !al16(a.w_att)) || (FQ && (!al16(a.w_final) || ((uintptr_t)a.codes & 3u))))
        return false;
    if (PRE_ADD && !a.resid) return false;
    const bool sum_resid = PRE_ADD || (FQ && a.resid);
    const int sms = device_sms();
    // the writers' loads of x (and of a summed resid) come from L2, a group
    // after the ring's copies brought them in: two groups per SM in flight.
    // More rows per group keep more exact-order sums in flight; fewer keep
    // more of the writers' loads in L2.  The sums of x + resid cost more per
    // element, so that form takes more rows (measured optimum on B200: about
    // 40 MB of such rows in flight, 60 MB for x + resid).
    const size_t reread = (size_t)a.dim * 4 * (sum_resid ? 2 : 1);
    const size_t budget = (sum_resid ? 60ull : 40ull) << 20;
    long G = (long)(budget / (2 * reread * (size_t)sms));
    if (G > 32) G = 32;
    if (G < 1) G = 1;
    const long per_cta = ((long)a.rows + sms - 1) / sms;
    if (G > per_cta) G = per_cta;
    // ring slots of G staged rows, each row x (+ resid) tiles of TC columns
    const int per_row = (int)((212u << 10) / (kColsSlots * (size_t)G)) - 32;
    long tcmax = (long)(per_row / (4 * (sum_resid ? 2 : 1))) / gran * gran;
    if (tcmax < gran) return false;
    const int T0 = (int)((a.dim + tcmax - 1) / tcmax);
    ColsLayout L{};
    L.G = (int)G;
    L.TC = (int)(((a.dim + T0 - 1) / T0 + gran - 1) / gran * gran);
    L.T = (a.dim + L.TC - 1) / L.TC;
    L.rofs = L.TC * 4;
    // an odd multiple of 16 bytes: the summing lanes' 16-byte loads of one
    // column fall in distinct banks
    L.stride = ((L.TC * 4 * (sum_resid ? 2 : 1) + 31) & ~31) + 16;
    L.slot = L.G * L.stride;
    L.smem = (size_t)kColsSlots * L.slot + 128 * sizeof(float) + (2 * kColsSlots + 4) * sizeof(uint64_t);
    if (L.smem > 226 * 1024) return false;
    auto kern = k_norm_cols<PRE_ADD, FQ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem);
    if (e != cudaSuccess) {
        *err = e;
        return true;
    }
    const long groups = ((long)a.rows + L.G - 1) / L.G;
    const long grid = groups < sms ? groups : sms;
    kern<<<(unsigned)grid, ColsShape<FQ>::threads, L.smem, s>>>(a, L);
    *err = launched();
    return true;
}

// The whole-row pipeline where its bulk copies apply (16-byte aligned rows:
// dim % 8, % 32 when quantising, % 128 for Q8_0 sources) and four slots of
// at least four rows fit in shared memory.  Returns false (nothing launched)
// otherwise.
template <int SRC, bool FQ>
bool try_norm_rows(const ChainArgs &a, cudaStream_t s, cudaError_t *err) {
    const int gran = SRC == SRC_Q8 ? 128 : (FQ ? 32 : 8);
    if (a.rows <= 0 || a.dim <= 0 || a.dim % gran) return false;
    const void *src = SRC == SRC_X ? (const void *)a.x_in : a.table;
    if (!al16(src) || (SRC == SRC_Q8 && !al16(a.tscales)) || (a.resid && !al16(a.resid)) ||
        (a.x_out && !al16(a.x_out)) || (a.xb && !al16(a.xb)) || (a.w_att && !al16(a.w_att)) ||
        (FQ && (!al16(a.w_final) || ((uintptr_t)a.codes & 3u))))
        return false;
    const int esz = SRC == SRC_BF16 ? 2 : (SRC == SRC_Q8 ? 1 : 4);
    RowsLayout L{};
    const int xb = a.dim * esz + (SRC == SRC_Q8 ? align16(a.dim / 8) : 0);
    L.xstride = ((xb + 31) & ~31) + 16;
    L.rstride = (FQ && a.resid) ? ((a.dim * 4 + 31) & ~31) + 16 : 0;
    long G = (long)((214u << 10) / (kRowsSlots * (size_t)(L.xstride + L.rstride)));
    if (G > 32) G = 32;
    if (G < 4) return false;
    const int sms = device_sms();
    const long per_cta = ((long)a.rows + sms - 1) / sms;
    if (G > per_cta) G = per_cta;
    L.G = (int)G;
    L.slot = L.G * (L.xstride + L.rstride);
    L.smem = kRowsSlots * ((size_t)L.slot + 64 * sizeof(float) + sizeof(uint64_t));
    auto kern = k_norm_rows<SRC, FQ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem);
    if (e != cudaSuccess) {
        *err = e;
        return true;
    }
    const long groups = ((long)a.rows + L.G - 1) / L.G;
    const long grid = groups < sms ? groups : sms;
    kern<<<(unsigned)grid, RowsShape<FQ>::threads, L.smem, s>>>(a, L);
    *err = launched();
    return true;
}

template <int SRC>
cudaError_t launch_chain_src_fused(const ChainArgs &a, cudaStream_t s);

// Llama-family chains (no q/k norm, no final Q8, half-split RoPE or none) run
// as two launches on the caller's stream: the norm stage's pipeline, then the
// independent RoPE/SwiGLU streams at full occupancy.  The stages share no
// data, so splitting them moves no extra bytes; it lets each run at the
// occupancy its resources allow.  Other chains run as the one fused kernel.
inline void mark(const LaunchHook *hook, int stage) {
    if (hook && hook->fn) hook->fn(hook->user, stage);
}

template <int SRC>
cudaError_t launch_chain_src(const ChainArgs &a, cudaStream_t s, const LaunchHook *hook) {
    const bool vec = (a.dim % 8) == 0 && (SRC != SRC_Q8 || a.dim % 32 == 0);
    const bool has_qk = (a.w_q && a.q) || (a.w_k && a.k);
    const bool has_rope = a.rope_mode != 0 && (a.q || a.k);
    // q/k norms or pair-mode RoPE go through the row-staged stream kernel.
    const bool qk_stream = has_qk || (has_rope && a.rope_mode == 2);
    const bool qk_ok = ((a.head | a.q_dim | a.kv_dim) & 3) == 0 && a.head > 0 &&
                       (a.rope_mode != 1 || (a.head & 7) == 0) &&
                       (a.rope_mode != 2 || (a.q_dim % a.head == 0 && a.kv_dim % a.head == 0));
    const bool streams_vec = ((a.half | a.q_dim | a.kv_dim | a.hidden) & 3) == 0;
    const bool any_stream = has_qk || has_rope || a.gate;
    const bool fq_pipe = a.w_final != nullptr && vec && a.dim % 32 == 0;
    const bool split = (a.w_final == nullptr || fq_pipe) &&
                       (!any_stream || (qk_stream ? qk_ok && (a.hidden & 3) == 0 : streams_vec));
    if (!split) {
        mark(hook, STAGE_FUSED);
        const cudaError_t e = launch_chain_src_fused<SRC>(a, s);
        mark(hook, STAGE_END);
        return e;
    }
    cudaError_t e = cudaSuccess;
    // Gathered bf16 / f32 rows ahead of the streams: the two-pass norm stage,
    // its writes a ticket type of the streams' kernel.
    const bool two_pass = (SRC == SRC_BF16 || SRC == SRC_F32) && a.tokens && a.ticket && a.row_scale && !a.w_final &&
                          (a.xb || a.x_out) && any_stream && !qk_stream && streams_vec && vec && al16(a.table) &&
                          (!a.xb || al16(a.xb)) && (!a.x_out || al16(a.x_out)) && (!a.resid || al16(a.resid)) &&
                          al16(a.w_att);
    if (two_pass) {
        mark(hook, STAGE_NORM);
        if constexpr (SRC == SRC_BF16 || SRC == SRC_F32) {
            static bool attr_set[64] = {false};
            int dev = 0;
            cudaGetDevice(&dev);
            if (dev < 0 || dev >= 64) dev = 0;
            if (!attr_set[dev]) {
                e = cudaFuncSetAttribute(k_row_scales<SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScaleSmem);
                attr_set[dev] = e == cudaSuccess;
            }
            if (e == cudaSuccess) {
                k_row_scales<SRC><<<(unsigned)((a.rows + 31) / 32), 32, kScaleSmem, s>>>(a, a.row_scale);
                e = launched();
            }
        }
    } else if (fq_pipe) {
        mark(hook, STAGE_NORM);
        // f32 x rows: the column-tiled pipeline (32 rows' sums in flight);
        // whole staged rows of f32 leave room for fewer
        const bool done = (SRC == SRC_X && try_norm_cols<false, true>(a, s, &e)) || try_norm_rows<SRC, true>(a, s, &e);
        if (!done) e = launch_norm_pipe<SRC, true, false, true>(a, s);
    } else if (a.xb || a.x_out) {
        mark(hook, STAGE_NORM);
        // f32 x rows: a CTA per row for a few, else the column-tiled pipeline
        // keeps more rows' sums in flight
        const bool done =
            vec && (SRC == SRC_X ? (try_norm_small<false>(a, s, &e) || try_norm_cols<false, false>(a, s, &e))
                                 : (try_norm_small_emb<SRC>(a, s, &e) || try_norm_rows<SRC, false>(a, s, &e)));
        if (!done) e = vec ? launch_norm_pipe<SRC, true>(a, s) : launch_norm_pipe<SRC, false>(a, s);
    }
    if (e != cudaSuccess) return e;
    if (any_stream && qk_stream) {
        const QkLaunch c = qk_launch_config(k_stream_qk, a.q_dim > a.kv_dim ? a.q_dim : a.kv_dim, a.head, a.rows);
        if (!c.warps) return cudaErrorInvalidValue;
        // the grid also covers SwiGLU: use every resident CTA slot
        int per_sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_stream_qk, c.warps * 32, c.smem);
        const unsigned grid = (unsigned)(device_sms() * (per_sm > 0 ? per_sm : 1));
        mark(hook, STAGE_STREAM);
        k_stream_qk<<<grid, c.warps * 32, c.smem, s>>>(a, c.smf);
        e = launched();
    } else if (any_stream) {
        static unsigned grid[64] = {0}, grid_dyn[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) dev = 0;
        if (!grid[dev]) {
            int per_sm = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_stream<2>, kThreads, 0);
            grid[dev] = (unsigned)(device_sms() * (per_sm > 0 ? per_sm : 1));
            per_sm = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_stream_dyn<-1, 2>, kThreads, 0);
            grid_dyn[dev] = (unsigned)(device_sms() * (per_sm > 0 ? per_sm : 1));
        }
        mark(hook, STAGE_STREAM);
        if (a.ticket) {
            const bool rope = a.rope_mode == 1;
            const unsigned n_silu = a.gate ? (unsigned)(((size_t)a.rows * a.hidden + kSpanElems - 1) / kSpanElems) : 0;
            const unsigned n_rows = (unsigned)((a.rows + kSpanRows - 1) / kSpanRows);
            const unsigned n_q = rope && a.q ? n_rows : 0, n_k = rope && a.k ? n_rows : 0;
            if (two_pass) {
                const unsigned n_norm = (unsigned)((a.rows + kNormRows - 1) / kNormRows);
                if constexpr (SRC == SRC_BF16 || SRC == SRC_F32)
                    k_stream_dyn<SRC, 2><<<grid_dyn[dev], kThreads, 0, s>>>(a, a.row_scale, n_norm, n_silu, n_q, n_k);
            } else {
                k_stream_dyn<-1, 2><<<grid_dyn[dev], kThreads, 0, s>>>(a, nullptr, 0, n_silu, n_q, n_k);
            }
        } else {
            k_stream<2><<<grid[dev], kThreads, 0, s>>>(a);
        }
        e = launched();
    }
    mark(hook, STAGE_END);
    return e;
}

template <int SRC>
cudaError_t launch_chain_src_fused(const ChainArgs &a, cudaStream_t s) {
    const bool vec = (a.dim % 8) == 0 && (SRC != SRC_Q8 || a.dim % 32 == 0);
    const bool fq = a.w_final != nullptr;
    if (fq) return vec ? launch_chain_t<SRC, true, true>(a, s) : launch_chain_t<SRC, true, false>(a, s);
    return vec ? launch_chain_t<SRC, false, true>(a, s) : launch_chain_t<SRC, false, false>(a, s);
}

}  // namespace

// SM count of the current device, cached per device.
int device_sms() {
    static int sms[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!sms[dev]) {
        int n = 148;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = n > 0 ? n : 148;
    }
    return sms[dev];
}

cudaError_t launch_embed_gather(int kind, bool vec, const GatherArgs &a, cudaStream_t s) {
    if (a.n <= 0) return cudaSuccess;
    const unsigned grid = grid_for((size_t)a.n * 32, kThreads);
    switch (kind) {
    case SRC_BF16:
        if (vec) k_embed_gather<SRC_BF16, true><<<grid, kThreads, 0, s>>>(a);
        else k_embed_gather<SRC_BF16, false><<<grid, kThreads, 0, s>>>(a);
        break;
    case SRC_Q8:
        if (vec) k_embed_gather<SRC_Q8, true><<<grid, kThreads, 0, s>>>(a);
        else k_embed_gather<SRC_Q8, false><<<grid, kThreads, 0, s>>>(a);
        break;
    default:
        if (vec) k_embed_gather<SRC_F32, true><<<grid, kThreads, 0, s>>>(a);
        else k_embed_gather<SRC_F32, false><<<grid, kThreads, 0, s>>>(a);
        break;
    }
    return launched();
}

size_t chain_smem_bytes(int src, const ChainArgs &a, int rows_per_cta) {
    const bool fq = a.w_final != nullptr;
    switch (src) {
    case SRC_BF16: return chain_layout<SRC_BF16>(a, fq, rows_per_cta).smem;
    case SRC_Q8: return chain_layout<SRC_Q8>(a, fq, rows_per_cta).smem;
    case SRC_F32: return chain_layout<SRC_F32>(a, fq, rows_per_cta).smem;
    default: return chain_layout<SRC_X>(a, fq, rows_per_cta).smem;
    }
}

cudaError_t launch_chain(int src, const ChainArgs &a, cudaStream_t s, const LaunchHook *hook) {
    if (a.rows <= 0) return cudaSuccess;
    switch (src) {
    case SRC_BF16: return launch_chain_src<SRC_BF16>(a, s, hook);
    case SRC_Q8: return launch_chain_src<SRC_Q8>(a, s, hook);
    case SRC_F32: return launch_chain_src<SRC_F32>(a, s, hook);
    default: return launch_chain_src<SRC_X>(a, s, hook);
    }
}

cudaError_t launch_qk_norm(float *v, int rows, int width, int head, const float *w, float eps,
                           cudaStream_t s) {
    if (rows <= 0 || width / head == 0) return cudaSuccess;
    const QkLaunch c = qk_launch_config(k_qk_norm_smem, width, head, rows);
    if (c.warps) {
        k_qk_norm_smem<<<c.grid, c.warps * 32, c.smem, s>>>(v, rows, width, head, w, eps, c.smf);
        return launched();
    }
    k_qk_norm<<<grid_for((size_t)rows * 32, kThreads), kThreads, 0, s>>>(v, rows, width, head, w, eps);
    return launched();
}

cudaError_t launch_rope(float *q, float *k, int q_width, int kv_width, int rows, int head,
                        const int32_t *pos, const float *cos_t, const float *sin_t, int max_pos,
                        int interleaved, int *err, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    // up to 8 warps per row while the rows alone would not fill the SMs
    int wpr = 1;
    while (wpr < 8 && (long)rows * 32 * wpr * 2 <= (long)device_sms() * kThreads) wpr *= 2;
    k_rope<<<grid_for((size_t)rows * 32 * wpr, kThreads), kThreads, 0, s>>>(
        q, k, q_width, kv_width, rows, head, pos, cos_t, sin_t, max_pos, interleaved, err, wpr);
    return launched();
}

cudaError_t launch_rope_kv(float *q, float *k, int q_width, int kv_width, int rows, int head, const int32_t *pos,
                           const float *cos_t, const float *sin_t, int max_pos, int *err, const float *v, float *kc,
                           float *vc, const int32_t *dst_rows, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (head <= 0 || kv_width % head != 0) return cudaErrorInvalidValue;
    int wpr = 1;
    while (wpr < 8 && (long)rows * 32 * wpr * 2 <= (long)device_sms() * kThreads) wpr *= 2;
    k_rope_kv<<<grid_for((size_t)rows * 32 * wpr, kThreads), kThreads, 0, s>>>(
        q, k, q_width, kv_width, rows, head, pos, cos_t, sin_t, max_pos, err, wpr, v, kc, vc, dst_rows);
    return launched();
}

cudaError_t launch_add_rms_norm(const ChainArgs &a, cudaStream_t s) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.dim % 8 != 0) return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    if (try_norm_small<true>(a, s, &e) || try_norm_cols<true, false>(a, s, &e))
        return e;
    return launch_norm_pipe<SRC_X, true, true, false>(a, s);
}

cudaError_t launch_qk_rope(float *q, float *k, int q_width, int kv_width, int rows, int head, const float *wq,
                           const float *wk, float eps, const int32_t *pos, const float *cos_t, const float *sin_t,
                           int max_pos, int interleaved, int *err, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    // float4 runs of a half head need head % 8; interleaved pairs need whole heads
    const bool whole = (head & 7) == 0 && (!interleaved || (q_width % head == 0 && kv_width % head == 0));
    const QkLaunch c = whole ? qk_launch_config(k_qk_rope_smem, q_width > kv_width ? q_width : kv_width, head, rows)
                             : QkLaunch{};
    if (c.warps && ((q_width | kv_width) & 3) == 0) {
        k_qk_rope_smem<<<c.grid, c.warps * 32, c.smem, s>>>(q, k, q_width, kv_width, rows, head, wq, wk, eps, pos,
                                                           cos_t, sin_t, max_pos, interleaved, err, c.smf);
        return launched();
    }
    k_qk_rope<<<grid_for((size_t)rows * 32, kThreads), kThreads, 0, s>>>(q, k, q_width, kv_width, rows, head, wq, wk,
                                                                          eps, pos, cos_t, sin_t, max_pos,
                                                                          interleaved, err);
    return launched();
}

cudaError_t launch_mul_strided(float *out, const float *a, const float *b, long long so, long long sa, long long sb,
                               int len, int count, cudaStream_t s) {
    if (len <= 0 || count <= 0) return cudaSuccess;
    k_mul_strided<<<stream_grid((size_t)len * count), kThreads, 0, s>>>(out, a, b, so, sa, sb, len, count);
    return launched();
}

cudaError_t launch_silu_mul(float *g, const float *u, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_silu_mul<<<stream_grid(n), kThreads, 0, s>>>(g, u, n);
    return launched();
}

cudaError_t launch_add(float *d, const float *src, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_add<<<stream_grid(n), kThreads, 0, s>>>(d, src, n);
    return launched();
}

cudaError_t launch_mul(float *o, const float *a, const float *b, size_t n, bool sequential,
                       cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (sequential) k_mul_sequential<<<1, 1, 0, s>>>(o, a, b, n);
    else k_mul<<<stream_grid(n), kThreads, 0, s>>>(o, a, b, n);
    return launched();
}

// The row-tiled kernels for K = 2..4 (float4 channels when dim and the
// pointers allow), the per-element kernel for other sizes.
// `rows` output rows of `dim` channels; `args` are the kernel's arguments.
template <int K, int V, int RT, typename Kern, typename... Args>
cudaError_t launch_conv_tiled(Kern kern, int rows, int dim, cudaStream_t s, Args... args) {
    const size_t threads = (size_t)(dim / V) * (size_t)((rows + RT - 1) / RT);
    kern<<<grid_for(threads, kThreads), kThreads, 0, s>>>(args...);
    return launched();
}

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

cudaError_t launch_conv_prefill(float *out, const float *x, const float *w, int rows, int dim, int k,
                                cudaStream_t s) {
    if (rows <= 0 || dim <= 0) return cudaSuccess;
    const bool v4 = dim % 4 == 0 && aligned16(out) && aligned16(x);
    constexpr int RT = 8;
#define KRT_CONV(KK)                                                                                        \
    if (k == KK)                                                                                            \
        return v4 ? launch_conv_tiled<KK, 4, RT>(k_conv_prefill_tiled<KK, 4, RT>, rows, dim, s, out, x, w, rows, dim) \
                  : launch_conv_tiled<KK, 1, RT>(k_conv_prefill_tiled<KK, 1, RT>, rows, dim, s, out, x, w, rows, dim);
    KRT_CONV(2)
    KRT_CONV(3)
    KRT_CONV(4)
#undef KRT_CONV
    k_conv_prefill<<<grid_for((size_t)rows * dim, kThreads), kThreads, 0, s>>>(out, x, w, rows, dim, k);
    return launched();
}

cudaError_t launch_conv_decode(float *out, const float *x, const float *w, float *state, int dim, int k,
                               cudaStream_t s) {
    if (dim <= 0) return cudaSuccess;
    k_conv_decode<<<grid_for((size_t)dim, kThreads), kThreads, 0, s>>>(out, x, w, state, dim, k);
    return launched();
}

cudaError_t launch_lfm2_conv_block(const float *bcx, const float *w, float *ring, float *cy, int rows,
                                   int dim, int k, cudaStream_t s, int lead) {
    if (rows <= 0 || dim <= 0) return cudaSuccess;
    const bool v4 = dim % 4 == 0 && aligned16(bcx) && aligned16(cy) && (!ring || aligned16(ring));
    constexpr int RT = 4;
    // threads cover the output rows only
#define KRT_CONV(KK)                                                                                           \
    if (k == KK)                                                                                               \
        return v4 ? launch_conv_tiled<KK, 4, RT>(k_lfm2_conv_block_tiled<KK, 4, RT>, rows - lead, dim, s, bcx, w, \
                                                 ring, cy, lead, rows, dim)                                    \
                  : launch_conv_tiled<KK, 1, RT>(k_lfm2_conv_block_tiled<KK, 1, RT>, rows - lead, dim, s, bcx, w, \
                                                 ring, cy, lead, rows, dim);
    KRT_CONV(2)
    KRT_CONV(3)
    KRT_CONV(4)
#undef KRT_CONV
    k_lfm2_conv_block<<<grid_for((size_t)(rows - lead) * dim, kThreads), kThreads, 0, s>>>(bcx, w, ring, cy, lead,
                                                                                           rows, dim, k);
    return launched();
}

cudaError_t launch_quantize_q8(const float *x, int rows, int dim, int8_t *codes, float *scales,
                               uint16_t *scales16, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (dim % 32 == 0 && ((uintptr_t)x & 31) == 0 && ((uintptr_t)codes & 7) == 0) {
        const size_t items = (size_t)rows * dim / 8;
        k_quantize_q8v8<2><<<stream_grid((size_t)rows * dim / 4), kThreads, 0, s>>>(x, items, codes, scales,
                                                                                   scales16);
        return launched();
    }
    if (dim % 32 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)codes & 3) == 0) {
        const size_t items = (size_t)rows * dim / 4;
        k_quantize_q8v<4><<<stream_grid((size_t)rows * dim / 4), kThreads, 0, s>>>(x, items, codes, scales,
                                                                                  scales16);
        return launched();
    }
    k_quantize_q8<<<grid_for((size_t)rows * 32, kThreads), kThreads, 0, s>>>(x, rows, dim, codes, scales,
                                                                              scales16);
    return launched();
}

cudaError_t launch_wait_selftest(int *err, long long limit, int complete, cudaStream_t s) {
    k_wait_selftest<<<1, 32, 0, s>>>(err, limit, complete);
    return launched();
}

cudaError_t launch_widen_f32(int dtype, const uint16_t *src, float *dst, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (dtype != 1 && dtype != 2) return cudaErrorInvalidValue;
    k_widen_f32<<<stream_grid(n), kThreads, 0, s>>>(dtype, src, dst, n);
    return launched();
}

cudaError_t launch_narrow_bf16(const float *src, uint16_t *dst, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_narrow_bf16<<<stream_grid(n), kThreads, 0, s>>>(src, dst, n);
    return launched();
}

cudaError_t launch_f16_scales_to_f32(const uint16_t *src, float *dst, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_f16_scales_to_f32<<<stream_grid(n), kThreads, 0, s>>>(src, dst, n);
    return launched();
}

cudaError_t launch_q8x4_to_row_major(const uint8_t *blocks, int out_dim, int in_dim, int8_t *quants,
                                     float *scales, cudaStream_t s) {
    const size_t n = (size_t)out_dim * (in_dim / 32);
    if (n == 0) return cudaSuccess;
    k_q8x4_to_row_major<<<grid_for(n, kThreads), kThreads, 0, s>>>(blocks, out_dim, in_dim, quants, scales);
    return launched();
}

}  // namespace krt
