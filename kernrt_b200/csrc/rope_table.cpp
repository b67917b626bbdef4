// RoPE cos/sin tables, built on the host with the libm calls KernRT's scalar
// backend makes per element (src/backends/reference.rs:225-228, 246-248):
//   freq  = 1.0f / powf(theta, (float)(2*j) / (float)head)
//   angle = (float)pos * freq
//   (sin, cos) = (sinf(angle), cosf(angle))
// The interleaved style's exponent head_dim/head with head_dim = 2j is the
// same float, so one table serves both styles.  The device then only applies
// the rotation; the table is prepared once per (theta, head) like a weight.
//
// Compiled by the host compiler with -ffp-contract=off and without fast-math
// or the sin/cos builtins, so every call is the platform libm's (the same
// glibc entry points Rust's f32::powf / sin / cos reach on Linux).
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <math.h>
#include <vector>

namespace krt {

void build_rope_table(float theta, int head, size_t max_pos, float *cos_out, float *sin_out) {
    const int half = head / 2;
    std::vector<float> freq((size_t)half);
    for (int j = 0; j < half; ++j) freq[(size_t)j] = 1.0f / ::powf(theta, (float)(2 * j) / (float)head);
    for (size_t pos = 0; pos < max_pos; ++pos) {
        const float p = (float)(uint64_t)pos;
        for (int j = 0; j < half; ++j) {
            const float angle = p * freq[(size_t)j];
            cos_out[pos * (size_t)half + (size_t)j] = ::cosf(angle);
            sin_out[pos * (size_t)half + (size_t)j] = ::sinf(angle);
        }
    }
}

}  // namespace krt
