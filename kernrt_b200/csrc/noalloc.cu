// kernrt_cuda_embed_rows_noalloc: the embedding gather for callers that may
// not allocate device memory.
//
// The regular gather (kernrt_cuda_embed) keeps each call's token ids and row
// offsets in scratch that the backend context allocates.  Some callers cannot
// let a library allocate: a host runtime that owns every byte of device memory
// through its own pre-reserved pool, or a serving loop that must never hit the
// device-wide synchronisation cudaMalloc/cudaFree can cause.  This entry point
// serves them from a fixed scratch array compiled into the library instead; it
// needs no context, and the caller passes the table and the output rows.
#include "../../include/kernrt_cuda.h"
#include "kernels.cuh"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

namespace krt {
void set_last_error(const std::string &msg);  // backend.cu: the thread's kernrt_cuda_last_error
}

namespace {

constexpr size_t kMaxRows = KERNRT_NOALLOC_MAX_ROWS;
constexpr int kMaxDevices = 64;

// The scratch: kMaxRows int32 token ids (256 KiB).  Every device that loads
// the library holds one copy until the process exits.  All calls on a device
// share it; a call writes every entry it later reads, so nothing needs
// clearing.  Output rows are addressed as row * dim inside the gather, so a
// call that overwrites the ids while another call's gather runs gives that
// call wrong rows of the table, never a write outside its own `out`.
static __device__ __align__(256) int32_t g_gather_ids[kMaxRows];

std::mutex g_setup_mu;
void *g_ids_addr[kMaxDevices];  // device address of g_gather_ids, per device

int fail(int code, const std::string &msg) {
    krt::set_last_error("kernrt_cuda_embed_rows_noalloc: " + msg);
    return code;
}

}  // namespace

extern "C" int kernrt_cuda_embed_rows_noalloc(int device, int kind, const void *table, const float *scales,
                                              size_t vocab, size_t dim, const int32_t *tokens, size_t n,
                                              float *out, void *stream) {
    if (n > kMaxRows)
        return fail(KERNRT_E_INVALID, std::to_string(n) + " rows exceed the fixed scratch of " +
                                          std::to_string(kMaxRows) + " rows; split the call");
    if (kind != KERNRT_F32 && kind != KERNRT_BF16 && kind != KERNRT_Q8_0)
        return fail(KERNRT_E_INVALID, "storage kind must be f32, bf16 or q8_0 (store Q8_0x4 row-major first)");
    if (!table || !out || vocab == 0 || dim == 0) return fail(KERNRT_E_INVALID, "empty table or null output");
    if (vocab > (size_t)INT32_MAX || dim > (size_t)INT32_MAX / 4)
        return fail(KERNRT_E_INVALID, "table too large");
    if (kind == KERNRT_Q8_0 && (dim % 32 != 0 || !scales))
        return fail(KERNRT_E_INVALID, "Q8_0 rows need whole 32-element blocks and their scales");
    if (n == 0) return KERNRT_OK;
    if (!tokens) return fail(KERNRT_E_INVALID, "null token ids");
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || (size_t)tokens[i] >= vocab)
            return fail(KERNRT_E_INVALID, "token " + std::to_string(tokens[i]) + " at row " + std::to_string(i) +
                                              " out of range for vocab " + std::to_string(vocab));
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count || device >= kMaxDevices) {
        cudaGetLastError();
        return fail(KERNRT_E_NO_DEVICE, "CUDA device " + std::to_string(device) + " not present");
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device && cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return fail(KERNRT_E_CUDA, "cudaSetDevice failed");
    }

    // Set-up, once per device and with that device current: the host-side
    // name of the array is only a stand-in, so fetch its device address.
    void *base = nullptr;
    cudaError_t e = cudaSuccess;
    {
        std::lock_guard<std::mutex> lock(g_setup_mu);
        if (!g_ids_addr[device]) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_gather_ids);
            if (e == cudaSuccess) g_ids_addr[device] = p;
        }
        base = g_ids_addr[device];
    }
    if (e == cudaSuccess && base) {
        int32_t *tok = static_cast<int32_t *>(base);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        e = cudaMemcpyAsync(tok, tokens, n * sizeof(int32_t), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
            krt::GatherArgs a{};
            a.table = table;
            a.tscales = scales;
            a.vocab = (int)vocab;
            a.dim = (int)dim;
            a.tokens = tok;
            a.dst_off = nullptr;  // row r at out + r * dim
            a.dst = out;
            a.n = (int)n;
            a.err = nullptr;  // ids were checked above
            const bool aligned = (((uintptr_t)table | (uintptr_t)out) & 15) == 0 && dim % 4 == 0;
            const bool vec = aligned && (kind == KERNRT_BF16 ? dim % 8 == 0 : kind == KERNRT_Q8_0 ? dim % 16 == 0 : true);
            e = krt::launch_embed_gather(kind, vec, a, s);
        }
    } else if (e == cudaSuccess) {
        e = cudaErrorInvalidSymbol;
    }
    // Leave no stale error behind for the caller's next launch check.
    if (e != cudaSuccess) cudaGetLastError();
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return fail(KERNRT_E_CUDA, cudaGetErrorString(e));
    return KERNRT_OK;
}
