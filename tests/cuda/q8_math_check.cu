// Exhaustive check of the Q8_0 block arithmetic in kernrt_b200/csrc/q8_math.cuh
// over all 2^32 f32 bit patterns:
//   q8_scale(a) == a / 127 (correctly rounded) for every a >= +0, +inf included;
//   q8_inv(d)   == 1 / d   (correctly rounded) for every d > 0, +inf included;
//   q8_code(v)  == the float-clamp form of quant.rs:871 for every v;
//   q8_inv_block(q8_scale(a)) == (d > 0 ? 1 / d : 0) for every a >= +0;
//   |q8_round(a * inv)| <= 127 for every finite a > 0 whose block needs no
//   clamp (q8_needs_clamp), inv = q8_inv_block(q8_scale(a)): the largest
//   product of a block, so the clamp-free codes of the kernels are in range.
// Prints the mismatch counts and exits 0 only when all are zero.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../kernrt_b200/csrc/q8_math.cuh"

__device__ __forceinline__ int8_t code_by_float_clamp(float v) {
    float r = roundf(v);
    r = (r < -127.0f) ? -127.0f : r;
    r = (r > 127.0f) ? 127.0f : r;
    return (r != r) ? (int8_t)0 : (int8_t)__float2int_rz(r);
}

__device__ unsigned long long g_bad[5];
__device__ unsigned int g_first[5];

__device__ __forceinline__ void bad(int k, uint32_t bits) {
    if (atomicAdd(&g_bad[k], 1ull) == 0) g_first[k] = bits;
}

__global__ void check(uint64_t base) {
    const uint64_t i = base + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    if (i > 0xffffffffull) return;
    const uint32_t bits = (uint32_t)i;
    const float a = __uint_as_float(bits);
    if (a == a) {
        if (a >= 0.0f && bits != 0x80000000u &&
            __float_as_uint(krt::q8_scale(a)) != __float_as_uint(__fdiv_rn(a, 127.0f)))
            bad(0, bits);
        if (a > 0.0f && __float_as_uint(krt::q8_inv(a)) != __float_as_uint(__fdiv_rn(1.0f, a))) bad(1, bits);
        if (a >= 0.0f && bits != 0x80000000u) {
            const float d = krt::q8_scale(a);
            const float want = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const float inv = krt::q8_inv_block(d);
            if (__float_as_uint(inv) != __float_as_uint(want)) bad(3, bits);
            if (a > 0.0f && a < __int_as_float(0x7f800000) && !krt::q8_needs_clamp(d)) {
                const int c = krt::q8_round(__fmul_rn(a, inv));
                if (c > 127 || c < -127) bad(4, bits);
            }
        }
    }
    if (krt::q8_code(a) != code_by_float_clamp(a)) bad(2, bits);
}

int main() {
    const int threads = 256;
    const uint64_t chunk = 1ull << 30;
    for (uint64_t b = 0; b < (1ull << 32); b += chunk) check<<<(unsigned)(chunk / threads), threads>>>(b);
    const cudaError_t e = cudaDeviceSynchronize();
    unsigned long long n[5] = {0, 0, 0, 0, 0};
    unsigned int f[5] = {0, 0, 0, 0, 0};
    cudaMemcpyFromSymbol(n, g_bad, sizeof(n));
    cudaMemcpyFromSymbol(f, g_first, sizeof(f));
    const char *what[5] = {"q8_scale", "q8_inv", "q8_code", "q8_inv_block", "q8_round bound"};
    for (int k = 0; k < 5; ++k) printf("%s mismatches %llu first 0x%08x\n", what[k], n[k], n[k] ? f[k] : 0u);
    printf("cuda %s\n", cudaGetErrorString(e));
    return (e == cudaSuccess && n[0] == 0 && n[1] == 0 && n[2] == 0 && n[3] == 0 && n[4] == 0) ? 0 : 1;
}
