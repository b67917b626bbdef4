// The `cuda` backend: a C++ mirror of KernRT's `Backend` trait
// (src/backends/mod.rs:264-404) over the sm_100a kernels, exported through the
// C ABI of include/kernrt_cuda.h.
//
// Ownership follows the trait: the backend owns every activation buffer and
// hands out handles (`Buf(usize)`, mod.rs:40-42); buffers live until the
// backend is destroyed.  Work is enqueued on one non-blocking CUDA stream per
// backend; nothing waits except `read`/`synchronize`, the trait's single
// barrier (mod.rs:262-263).  Host slices the trait borrows only for the call
// (positions, token ids) are copied into a pinned staging ring at call time.
// Consecutive `embed` calls are coalesced into one gather launch, flushed by
// the next other op or barrier.
//
// Misuse that the reference turns into a panic (index out of range, aliasing
// buffers that must be distinct) is detected on the host before any launch
// and returned as KERNRT_E_INVALID with a message.
#include "../../include/kernrt_cuda.h"
#include "kernels.cuh"
#include "safetensors.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <cstdlib>
#include <fcntl.h>
#include <unistd.h>
#include <cstring>
#include <string>
#include <thread>
#include <utility>
#include <vector>

namespace krt {

void build_rope_table(float theta, int head, size_t max_pos, float *cos_out, float *sin_out);

struct Error {
    int code;
    std::string msg;
};

[[noreturn]] static void fail(int code, const std::string &msg) { throw Error{code, msg}; }

static void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) fail(KERNRT_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static const char *kind_name(int kind) {
    switch (kind) {
    case KERNRT_BF16: return "bf16";
    case KERNRT_Q8_0: return "q8_0";
    case KERNRT_Q8_0X4: return "q8_0x4";
    default: return "f32";
    }
}

class Backend {
public:
    explicit Backend(int device) : device_(device) {
        check(cudaSetDevice(device_), "cudaSetDevice");
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaMalloc(&d_err_, sizeof(int)), "cudaMalloc(error word)");
        check(cudaMemsetAsync(d_err_, 0, sizeof(int), stream_), "cudaMemset");
        check(cudaMalloc(&d_ticket_, sizeof(unsigned)), "cudaMalloc(stream ticket)");
        check(cudaMemsetAsync(d_ticket_, 0, sizeof(unsigned), stream_), "cudaMemset");
        check(cudaMallocHost(&h_err_, sizeof(int)), "cudaMallocHost");
        grow_staging(1 << 20);
        check(cudaStreamCreateWithFlags(&h2d_, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaStreamCreateWithFlags(&d2h_, cudaStreamNonBlocking), "cudaStreamCreate");
        for (auto &set : sets_)
            for (cudaEvent_t *e : {&set.h2d_done, &set.comp_done, &set.d2h_done})
                check(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate");
    }

    ~Backend() {
        cudaSetDevice(device_);
        cudaStreamSynchronize(stream_);
        for (auto &b : bufs_) cudaFree(b.ptr);
        for (auto &t : ropes_) {
            cudaFree(t.cos);
            cudaFree(t.sin);
        }
        cudaFree(emb_data_);
        cudaFree(emb_scales_);
        for (auto &m : mats_) {
            cudaFree(m.data);
            cudaFree(m.scales);
        }
        cudaFree(kc_);
        cudaFree(vc_);
        cudaFree(att_scratch_);
        cudaFree(d_err_);
        cudaFree(d_ticket_);
        cudaFree(split_);
        cudaFree(row_scales_);
        cudaFreeHost(h_err_);
        cudaFreeHost(stage_host_);
        cudaFree(stage_dev_);
        for (auto &r : retired_) {
            cudaFreeHost(r.first);
            cudaFree(r.second);
        }
        for (auto e : events_) cudaEventDestroy(e);
        for (auto e : stage_ev_)
            if (e) cudaEventDestroy(e);
        for (int k = 0; k < 2; ++k) {
            if (file_ev_[k]) cudaEventDestroy(file_ev_[k]);
            cudaFreeHost(file_pin_[k]);
        }
        cudaStreamSynchronize(h2d_);
        cudaStreamSynchronize(d2h_);
        for (auto &set : sets_) {
            cudaFree(set.arena);
            cudaEventDestroy(set.h2d_done);
            cudaEventDestroy(set.comp_done);
            cudaEventDestroy(set.d2h_done);
        }
        cudaStreamDestroy(h2d_);
        cudaStreamDestroy(d2h_);
        cudaStreamDestroy(stream_);
    }

    const char *storage() const { return storage_; }
    cudaStream_t stream() const { return stream_; }
    void activate() const { check(cudaSetDevice(device_), "cudaSetDevice"); }

    // ---- Backend::prepare: the token embedding in its stored format -------
    void prepare_embedding(int kind, const void *data, const float *scales, size_t vocab, size_t dim) {
        if (!data || vocab == 0 || dim == 0) fail(KERNRT_E_INVALID, "empty embedding table");
        if (kind < KERNRT_F32 || kind > KERNRT_Q8_0X4) fail(KERNRT_E_INVALID, "unknown storage kind");
        if ((kind == KERNRT_Q8_0 || kind == KERNRT_Q8_0X4) && dim % 32 != 0)
            fail(KERNRT_E_INVALID, "Q8_0 rows must be a whole number of 32-element blocks");
        if (kind == KERNRT_Q8_0X4 && vocab % 4 != 0)
            fail(KERNRT_E_INVALID, "Q8_0x4 tables hold a multiple of four rows");
        if (kind == KERNRT_Q8_0 && !scales) fail(KERNRT_E_INVALID, "Q8_0 table needs its scales");
        if (vocab * dim > (size_t)INT32_MAX * 4 || vocab > (size_t)INT32_MAX || dim > (1u << 24))
            fail(KERNRT_E_INVALID, "embedding table too large");
        flush();
        check(cudaStreamSynchronize(stream_), "synchronize");
        cudaFree(emb_data_);
        cudaFree(emb_scales_);
        emb_data_ = nullptr;
        emb_scales_ = nullptr;
        const size_t n = vocab * dim;
        if (kind == KERNRT_F32 || kind == KERNRT_BF16) {
            const size_t bytes = n * (kind == KERNRT_F32 ? 4 : 2);
            check(cudaMalloc(&emb_data_, bytes), "cudaMalloc(embedding)");
            check(cudaMemcpy(emb_data_, data, bytes, cudaMemcpyHostToDevice), "upload embedding");
            emb_src_ = kind == KERNRT_F32 ? SRC_F32 : SRC_BF16;
        } else {
            check(cudaMalloc(&emb_data_, n), "cudaMalloc(embedding)");
            check(cudaMalloc(&emb_scales_, (n / 32) * sizeof(float)), "cudaMalloc(embedding scales)");
            if (kind == KERNRT_Q8_0) {
                check(cudaMemcpy(emb_data_, data, n, cudaMemcpyHostToDevice), "upload embedding");
                check(cudaMemcpy(emb_scales_, scales, (n / 32) * sizeof(float), cudaMemcpyHostToDevice),
                      "upload embedding scales");
            } else {
                // Q8_0x4 (quant.rs:102-117): 136 bytes per (4 rows x 32 columns),
                // de-interleaved here to the row-major Q8_0 the kernels read.
                const size_t blk_bytes = (vocab / 4) * (dim / 32) * 136;
                void *tmp = nullptr;
                check(cudaMalloc(&tmp, blk_bytes), "cudaMalloc(q8_0x4 staging)");
                cudaError_t e = cudaMemcpy(tmp, data, blk_bytes, cudaMemcpyHostToDevice);
                if (e == cudaSuccess)
                    e = launch_q8x4_to_row_major(static_cast<const uint8_t *>(tmp), (int)vocab, (int)dim,
                                                 static_cast<int8_t *>(emb_data_), emb_scales_, stream_);
                if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
                cudaFree(tmp);
                check(e, "Q8_0x4 de-interleave");
            }
            emb_src_ = SRC_Q8;
        }
        emb_kind_ = kind;
        vocab_ = vocab;
        dim_ = dim;
        storage_ = kind_name(kind);
    }

    // Backend::prepare's embedding read from a safetensors file
    // (hf.rs:141-191 take_matrix_raw / matrix_from_raw over the raw reader,
    // safetensors.rs:129-135): the tensor's payload goes from the file to the
    // device as stored (page-locked chunks, reads overlapped with the copies)
    // and is converted there into the storage the reference's rules pick:
    // bf16 bits as they are for bf16 storage; bf16 widened and quantised for
    // block-aligned Q8_0 / Q8_0x4; f32 or f16 widened, then kept as f32,
    // quantised for aligned Q8_0x4, and otherwise narrowed to bf16 by
    // dropping the low half.
    void prepare_embedding_file(const char *path, const char *name, int storage) {
        if (!path || !name) fail(KERNRT_E_INVALID, "null path or tensor name");
        if (storage < KERNRT_F32 || storage > KERNRT_Q8_0X4) fail(KERNRT_E_INVALID, "unknown storage kind");
        StHeader h;
        const std::string err = st_read_header(path, &h);
        if (!err.empty()) fail(KERNRT_E_INVALID, err);
        const auto it = h.tensors.find(name);
        if (it == h.tensors.end()) fail(KERNRT_E_INVALID, "weight file is missing \"" + std::string(name) + "\"");
        const StTensor &t = it->second;
        if (t.shape.size() != 2) fail(KERNRT_E_INVALID, "a weight matrix was not rank 2");
        const size_t vocab = (size_t)t.shape[0], dim = (size_t)t.shape[1];
        if (vocab == 0 || dim == 0) fail(KERNRT_E_INVALID, "empty embedding table");
        if (vocab > (size_t)INT32_MAX || dim > (1u << 24) || vocab * dim > (size_t)INT32_MAX * 4)
            fail(KERNRT_E_INVALID, "embedding table too large");
        const bool aligned_q8 = dim % 32 == 0, aligned_q8x4 = aligned_q8 && vocab % 4 == 0;
        enum { BF16_BITS, TO_F32, TO_Q8, TO_Q8X4, TO_BF16 } route;
        if (t.dtype == ST_BF16 && storage == KERNRT_BF16) route = BF16_BITS;
        else if (t.dtype == ST_BF16 && storage == KERNRT_Q8_0 && aligned_q8) route = TO_Q8;
        else if (t.dtype == ST_BF16 && storage == KERNRT_Q8_0X4 && aligned_q8x4) route = TO_Q8X4;
        else if (storage == KERNRT_F32) route = TO_F32;
        else if (storage == KERNRT_Q8_0X4 && aligned_q8x4) route = TO_Q8X4;
        else route = TO_BF16;

        flush();
        check(cudaStreamSynchronize(stream_), "synchronize");
        const size_t n = vocab * dim, nb = n / 32;
        struct Dev {
            void *p = nullptr;
            ~Dev() { cudaFree(p); }
        } payload, wide, table, scales, scales16;
        check(cudaMalloc(&payload.p, std::max<size_t>(t.end - t.start, 16)), "cudaMalloc(file payload)");
        read_file(path, h.data_offset + t.start, t.end - t.start, payload.p);
        // f32 values of the table, where the route needs them
        const float *f = nullptr;
        if (route != BF16_BITS) {
            if (t.dtype == ST_F32) {
                f = static_cast<const float *>(payload.p);
            } else {
                check(cudaMalloc(&wide.p, n * sizeof(float)), "cudaMalloc(widened table)");
                check(launch_widen_f32(t.dtype == ST_BF16 ? 1 : 2, static_cast<const uint16_t *>(payload.p),
                                       static_cast<float *>(wide.p), n, stream_),
                      "widen table");
                f = static_cast<const float *>(wide.p);
            }
        }
        int kind, src;
        switch (route) {
        case BF16_BITS:
            std::swap(table.p, payload.p);
            kind = KERNRT_BF16, src = SRC_BF16;
            break;
        case TO_F32:
            if (f == payload.p) std::swap(table.p, payload.p);
            else std::swap(table.p, wide.p);
            kind = KERNRT_F32, src = SRC_F32;
            break;
        case TO_BF16:
            check(cudaMalloc(&table.p, n * 2), "cudaMalloc(embedding)");
            check(launch_narrow_bf16(f, static_cast<uint16_t *>(table.p), n, stream_), "narrow table");
            kind = KERNRT_BF16, src = SRC_BF16;
            break;
        default:  // TO_Q8, TO_Q8X4: Q8Vec::quantize's blocks (quant.rs:544-557, 124-165)
            check(cudaMalloc(&table.p, n), "cudaMalloc(embedding)");
            check(cudaMalloc(&scales.p, nb * sizeof(float)), "cudaMalloc(embedding scales)");
            check(cudaMalloc(&scales16.p, nb * sizeof(uint16_t)), "cudaMalloc(f16 scales)");
            check(launch_quantize_q8(f, (int)vocab, (int)dim, static_cast<int8_t *>(table.p),
                                     static_cast<float *>(scales.p), static_cast<uint16_t *>(scales16.p), stream_),
                  "quantize table");
            // Q8_0x4 keeps f16 scales and widens them on read (quant.rs:198-220, 764-769)
            if (route == TO_Q8X4)
                check(launch_f16_scales_to_f32(static_cast<const uint16_t *>(scales16.p),
                                               static_cast<float *>(scales.p), nb, stream_),
                      "widen f16 scales");
            kind = route == TO_Q8 ? KERNRT_Q8_0 : KERNRT_Q8_0X4, src = SRC_Q8;
            break;
        }
        check(cudaStreamSynchronize(stream_), "load embedding");
        cudaFree(emb_data_);
        cudaFree(emb_scales_);
        emb_data_ = table.p;
        emb_scales_ = static_cast<float *>(scales.p);
        table.p = scales.p = nullptr;
        emb_src_ = src;
        emb_kind_ = kind;
        vocab_ = vocab;
        dim_ = dim;
        storage_ = kind_name(kind);
    }

    // `bytes` of `path` from `offset` into device memory through two
    // page-locked 64 MB chunks (allocated on the first load and kept): each
    // chunk is filled by several reader threads while the other's copy runs.
    static constexpr size_t kFileChunk = 64u << 20;

    void read_file(const char *path, uint64_t offset, uint64_t bytes, void *dst) {
        if (bytes == 0) return;
        const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
        if (fd < 0) fail(KERNRT_E_INVALID, std::string("i/o error: ") + std::strerror(errno));
        std::string why;
        int code = KERNRT_E_CUDA;
        for (int k = 0; k < 2 && why.empty(); ++k) {
            if (!file_pin_[k] && cudaHostAlloc(&file_pin_[k], kFileChunk, cudaHostAllocDefault) != cudaSuccess) {
                file_pin_[k] = nullptr;
                why = "cudaHostAlloc(file staging)";
            } else if (!file_ev_[k] && cudaEventCreateWithFlags(&file_ev_[k], cudaEventDisableTiming) != cudaSuccess) {
                file_ev_[k] = nullptr;
                why = "cudaEventCreate";
            }
        }
        const unsigned hw = std::thread::hardware_concurrency();
        const int nthreads = (int)std::max(1u, std::min(8u, hw ? hw : 1u));
        // pread [lo, lo + len) of the file into p; false on a short read
        auto fill = [&](char *p, uint64_t lo, size_t len) {
            std::vector<std::thread> pool;
            std::vector<char> ok((size_t)nthreads, 1);
            const size_t part = (len + nthreads - 1) / nthreads;
            for (int t = 0; t < nthreads; ++t) {
                const size_t a = std::min(len, (size_t)t * part), z = std::min(len, a + part);
                if (a >= z) break;
                pool.emplace_back([&, t, a, z] {
                    size_t got = a;
                    while (got < z) {
                        const ssize_t r = ::pread(fd, p + got, z - got, (off_t)(lo + got));
                        if (r < 0 && errno == EINTR) continue;
                        if (r <= 0) break;
                        got += (size_t)r;
                    }
                    ok[(size_t)t] = got == z;
                });
            }
            for (auto &th : pool) th.join();
            for (char c : ok)
                if (!c) return false;
            return true;
        };
        bool used[2] = {false, false};
        uint64_t done = 0;
        for (int k = 0; why.empty() && done < bytes; k ^= 1) {
            const size_t len = (size_t)std::min<uint64_t>(bytes - done, kFileChunk);
            if (used[k] && cudaEventSynchronize(file_ev_[k]) != cudaSuccess) {
                why = "file staging copy";
                break;
            }
            if (!fill(static_cast<char *>(file_pin_[k]), offset + done, len)) {
                why = "i/o error: short read of a tensor payload";
                code = KERNRT_E_INVALID;
                break;
            }
            if (cudaMemcpyAsync(static_cast<char *>(dst) + done, file_pin_[k], len, cudaMemcpyHostToDevice,
                                stream_) != cudaSuccess ||
                cudaEventRecord(file_ev_[k], stream_) != cudaSuccess) {
                why = "upload of a tensor payload";
                break;
            }
            used[k] = true;
            done += len;
        }
        const cudaError_t e = cudaStreamSynchronize(stream_);
        if (why.empty() && e != cudaSuccess) why = "upload of a tensor payload";
        ::close(fd);
        if (!why.empty()) fail(code, why);
    }

    // ---- buffers ------------------------------------------------------------
    kernrt_buf alloc_bytes(size_t bytes) {
        Buffer b;
        b.bytes = bytes;
        // Fault injection for tests: KERNRT_CUDA_FAIL_ALLOC=n makes this
        // context's n-th buffer allocation fail as an exhausted device would.
        if (++allocs_ == fail_alloc_at_) check(cudaErrorMemoryAllocation, "cudaMalloc");
        check(cudaMalloc(&b.ptr, std::max<size_t>(bytes, 16)), "cudaMalloc");
        check(cudaMemsetAsync(b.ptr, 0, std::max<size_t>(bytes, 16), stream_), "cudaMemset");
        bufs_.push_back(b);
        return (kernrt_buf)bufs_.size();  // handle = index + 1; 0 means "none"
    }

    kernrt_buf upload(const float *data, size_t len) {
        if (len && !data) fail(KERNRT_E_INVALID, "null upload source");
        const kernrt_buf h = alloc_bytes(len * sizeof(float));
        write_bytes(h, 0, data, len * sizeof(float));
        return h;
    }

    void write_bytes(kernrt_buf h, size_t off, const void *src, size_t bytes) {
        Buffer &b = buf(h);
        if (off > b.bytes || bytes > b.bytes - off) fail(KERNRT_E_INVALID, "write past the end of the buffer");
        if (bytes == 0) return;
        if (!src) fail(KERNRT_E_INVALID, "null write source");
        flush();
        check(cudaMemcpyAsync(b.ptr + off, src, bytes, cudaMemcpyHostToDevice, stream_), "cudaMemcpyAsync");
        // A pageable source may be read after return; page-locked memory is the
        // caller's to keep alive until the next barrier.
        cudaPointerAttributes attr{};
        if (cudaPointerGetAttributes(&attr, src) != cudaSuccess || attr.type != cudaMemoryTypeHost) {
            cudaGetLastError();
            check(cudaStreamSynchronize(stream_), "synchronize");
        }
    }

    void read_bytes(kernrt_buf h, size_t off, void *dst, size_t bytes) {
        Buffer &b = buf(h);
        if (off > b.bytes || bytes > b.bytes - off) fail(KERNRT_E_INVALID, "read past the end of the buffer");
        flush();
        if (bytes) {
            if (!dst) fail(KERNRT_E_INVALID, "null read destination");
            check(cudaMemcpyAsync(dst, b.ptr + off, bytes, cudaMemcpyDeviceToHost, stream_), "cudaMemcpyAsync");
        }
        barrier();
    }

    void *device_ptr(kernrt_buf h) { return buf(h).ptr; }

    // Completes deferred work and surfaces device-reported input errors.
    void barrier() {
        flush();
        check(cudaMemcpyAsync(h_err_, d_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_), "error word");
        check(cudaStreamSynchronize(stream_), "synchronize");
        for (auto &r : retired_) {
            cudaFreeHost(r.first);
            cudaFree(r.second);
        }
        retired_.clear();
        const int e = *h_err_;
        if (e) {
            check(cudaMemsetAsync(d_err_, 0, sizeof(int), stream_), "cudaMemset");
            check(cudaStreamSynchronize(stream_), "synchronize");
            std::string m = "device reported:";
            if (e & ERR_TOKEN) m += " token id out of range of the embedding table;";
            if (e & ERR_POSITION) m += " position outside the prepared RoPE table;";
            if (e & ERR_TIMEOUT) m += " a kernel's wait for its staged rows timed out;";
            fail(KERNRT_E_DEVICE, m);
        }
    }

    // The pipelines' bounded wait exercised on its own: after `cycles` SM
    // cycles without the phase completing, the error word reports a timeout,
    // which barrier() turns into KERNRT_E_DEVICE; the context stays usable.
    void selftest_wait(uint64_t cycles, int complete) {
        if (cycles > (1ull << 31)) fail(KERNRT_E_INVALID, "wait limit above 2^31 cycles");
        flush();
        launch_or_fail(launch_wait_selftest(d_err_, (long long)cycles, complete ? 1 : 0, stream_), "wait self-test");
        barrier();
    }

    // ---- Backend::embed (deferred, coalesced) --------------------------------
    void embed(size_t token, kernrt_buf out, size_t offset) {
        if (emb_kind_ < 0) fail(KERNRT_E_STATE, "prepare() runs before compute");
        if (token >= vocab_) fail(KERNRT_E_INVALID, "token " + std::to_string(token) + " out of range for vocab " + std::to_string(vocab_));
        const Buffer &b = buf(out);
        if (offset > b.bytes / 4 || dim_ > b.bytes / 4 - offset) fail(KERNRT_E_INVALID, "embed writes past the end of the buffer");
        flush_deferred();
        if (!pending_.empty() && pending_.back().out != out) flush();
        pending_.push_back({(int32_t)token, out, (int64_t)offset});
    }

    // ---- contractions (reference.rs:151-159, 259-306, 402-416) ---------------
    struct DevMatrix {
        int src = SRC_F32;
        void *data = nullptr;
        float *scales = nullptr;
        size_t out_dim = 0, in_dim = 0;
    };

    // A weight matrix [out_dim, in_dim] in its stored format, kept on the
    // device in the form the kernels read (Q8_0x4 de-interleaved to Q8_0 with
    // widened scales, the repack quant.rs:646-652 gives device backends).
    uint64_t prepare_matrix(int kind, const void *data, const float *scales, size_t out_dim, size_t in_dim) {
        if (!data || out_dim == 0 || in_dim == 0) fail(KERNRT_E_INVALID, "empty matrix");
        if (kind < KERNRT_F32 || kind > KERNRT_Q8_0X4) fail(KERNRT_E_INVALID, "unknown storage kind");
        if ((kind == KERNRT_Q8_0 || kind == KERNRT_Q8_0X4) && in_dim % 32 != 0)
            fail(KERNRT_E_INVALID, "Q8_0 rows must be a whole number of 32-element blocks");
        if (kind == KERNRT_Q8_0X4 && out_dim % 4 != 0) fail(KERNRT_E_INVALID, "Q8_0x4 matrices hold a multiple of four rows");
        if (kind == KERNRT_Q8_0 && !scales) fail(KERNRT_E_INVALID, "Q8_0 matrix needs its scales");
        if (out_dim > (size_t)INT32_MAX || in_dim > (size_t)INT32_MAX || out_dim * in_dim > ((size_t)1 << 40))
            fail(KERNRT_E_INVALID, "matrix too large");
        flush();
        DevMatrix m;
        m.out_dim = out_dim;
        m.in_dim = in_dim;
        const size_t n = out_dim * in_dim;
        try {
            if (kind == KERNRT_F32 || kind == KERNRT_BF16) {
                const size_t bytes = n * (kind == KERNRT_F32 ? 4 : 2);
                check(cudaMalloc(&m.data, bytes), "cudaMalloc(matrix)");
                check(cudaMemcpy(m.data, data, bytes, cudaMemcpyHostToDevice), "upload matrix");
                m.src = kind == KERNRT_F32 ? SRC_F32 : SRC_BF16;
            } else {
                check(cudaMalloc(&m.data, n), "cudaMalloc(matrix)");
                check(cudaMalloc(&m.scales, (n / 32) * sizeof(float)), "cudaMalloc(matrix scales)");
                if (kind == KERNRT_Q8_0) {
                    check(cudaMemcpy(m.data, data, n, cudaMemcpyHostToDevice), "upload matrix");
                    check(cudaMemcpy(m.scales, scales, (n / 32) * sizeof(float), cudaMemcpyHostToDevice),
                          "upload matrix scales");
                } else {
                    const size_t blk_bytes = (out_dim / 4) * (in_dim / 32) * 136;
                    void *tmp = nullptr;
                    check(cudaMalloc(&tmp, blk_bytes), "cudaMalloc(q8_0x4 staging)");
                    cudaError_t e = cudaMemcpy(tmp, data, blk_bytes, cudaMemcpyHostToDevice);
                    if (e == cudaSuccess)
                        e = launch_q8x4_to_row_major(static_cast<const uint8_t *>(tmp), (int)out_dim, (int)in_dim,
                                                     static_cast<int8_t *>(m.data), m.scales, stream_);
                    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
                    cudaFree(tmp);
                    check(e, "Q8_0x4 de-interleave");
                }
                m.src = SRC_Q8;
            }
        } catch (...) {
            cudaFree(m.data);
            cudaFree(m.scales);
            throw;
        }
        mats_.push_back(m);
        return (uint64_t)mats_.size();  // handle = index + 1
    }

    const DevMatrix &mat(uint64_t h) const {
        if (h == 0 || h > mats_.size()) fail(KERNRT_E_INVALID, "invalid matrix handle " + std::to_string(h));
        return mats_[h - 1];
    }

    // Tolerance mode: bf16 projections of at least kTcMinRows rows go to the
    // tensor cores (tc_project.cu) instead of the exact-order kernels.
    static constexpr size_t kTcMinRows = 16;
    bool tc_path(const DevMatrix &m, const float *x, const float *y, size_t rows) const {
        return !exact_ && m.src == SRC_BF16 && rows >= kTcMinRows &&
               project_tc_supported((int)m.out_dim, (int)m.in_dim, m.data, x, y);
    }
    // Tolerance mode: bf16 projections of 1-4 rows (decode) sum each output
    // across a warp instead of in the reference's order (tc_project.cu).
    bool tol_gemv_path(const DevMatrix &m, const float *x, size_t rows) const {
        return !exact_ && m.src == SRC_BF16 && gemv_tol_supported(m.data, x, (int)m.in_dim, (int)rows);
    }
    // x split into bf16 hi and lo halves ([rows, in_dim] each), in scratch
    // grown as needed (cudaFree waits for queued kernels still reading it).
    uint16_t *split_x(const float *x, size_t rows, size_t in_dim) {
        const size_t n = rows * in_dim;
        if (2 * n > split_cap_) {
            cudaFree(split_);
            split_ = nullptr;
            split_cap_ = 0;
            check(cudaMalloc(&split_, 2 * n * sizeof(uint16_t)), "cudaMalloc(split activations)");
            split_cap_ = 2 * n;
        }
        launch_or_fail(launch_split_bf16(x, split_, split_ + n, n, stream_), "project (split)");
        return split_;
    }
    void set_fail_alloc(uint64_t n) { fail_alloc_at_ = n; }
    void set_exact(bool exact) {
        flush();
        exact_ = exact;
    }

    // reference.rs:259-274: y[r, o] = dot(decode_row(W, o), x[r]).
    void project(uint64_t w, kernrt_buf x, kernrt_buf y, size_t rows) {
        const DevMatrix &m = mat(w);
        distinct(x, y);
        Buffer &xb = buf(x), &yb = buf(y);
        span(xb, 0, rows * m.in_dim, "project x");
        span(yb, 0, rows * m.out_dim, "project y");
        fits_int(rows * std::max(m.in_dim, m.out_dim), "project");
        flush();
        if (rows == 0) return;
        if (tc_path(m, f(xb), f(yb), rows)) {
            const uint16_t *hi = split_x(f(xb), rows, m.in_dim);
            launch_or_fail(launch_project_tc(static_cast<const uint16_t *>(m.data), (int)m.out_dim, (int)m.in_dim, hi,
                                             hi + rows * m.in_dim, (int)rows, f(yb), d_err_, stream_),
                           "project (tensor cores)");
            return;
        }
        if (tol_gemv_path(m, f(xb), rows)) {
            const uint16_t *w16 = static_cast<const uint16_t *>(m.data);
            const int out = (int)m.out_dim;
            float *y = f(yb);
            launch_or_fail(launch_gemv_tol(1, &w16, &out, (int)m.in_dim, f(xb), (int)rows, &y, stream_),
                           "project (tolerance)");
            return;
        }
        launch_or_fail(launch_project(m.src, m.data, m.scales, (int)m.out_dim, (int)m.in_dim, f(xb), (int)rows, f(yb),
                                      d_err_, stream_),
                       "project");
    }

    // mod.rs:320-337 project_qkv / project_gate_up: n projections of one x,
    // in one launch where the shapes allow (same storage and in_dim).
    void project_set(int n, const uint64_t *ws, kernrt_buf x, const kernrt_buf *ys, size_t rows) {
        const void *wp[3];
        const float *sp[3];
        int outs[3];
        float *yp[3];
        const DevMatrix &m0 = mat(ws[0]);
        bool same = true;
        for (int i = 0; i < n; ++i) {
            const DevMatrix &m = mat(ws[i]);
            distinct(x, ys[i]);
            for (int j = 0; j < i; ++j)
                if (ys[j] == ys[i]) fail(KERNRT_E_INVALID, "buffers must be distinct");
            same = same && m.src == m0.src && m.in_dim == m0.in_dim;
        }
        if (!same) {
            for (int i = 0; i < n; ++i) project(ws[i], x, ys[i], rows);
            return;
        }
        Buffer &xb = buf(x);
        span(xb, 0, rows * m0.in_dim, "project x");
        for (int i = 0; i < n; ++i) {
            const DevMatrix &m = mat(ws[i]);
            Buffer &yb = buf(ys[i]);
            span(yb, 0, rows * m.out_dim, "project y");
            fits_int(rows * std::max(m.in_dim, m.out_dim), "project");
            wp[i] = m.data;
            sp[i] = m.scales;
            outs[i] = (int)m.out_dim;
            yp[i] = f(yb);
        }
        flush();
        if (rows == 0) return;
        bool tc = true;
        for (int i = 0; i < n; ++i) tc = tc && tc_path(mat(ws[i]), f(xb), yp[i], rows);
        if (tc) {  // one split of x for the n projections
            const uint16_t *hi = split_x(f(xb), rows, m0.in_dim);
            for (int i = 0; i < n; ++i)
                launch_or_fail(launch_project_tc(static_cast<const uint16_t *>(wp[i]), outs[i], (int)m0.in_dim, hi,
                                                 hi + rows * m0.in_dim, (int)rows, yp[i], d_err_, stream_),
                               "project (tensor cores)");
            return;
        }
        bool tol = true;
        for (int i = 0; i < n; ++i) tol = tol && tol_gemv_path(mat(ws[i]), f(xb), rows);
        if (tol) {  // one launch over the n matrices' outputs
            const uint16_t *w16[3];
            for (int i = 0; i < n; ++i) w16[i] = static_cast<const uint16_t *>(wp[i]);
            launch_or_fail(launch_gemv_tol(n, w16, outs, (int)m0.in_dim, f(xb), (int)rows, yp, stream_),
                           "project (tolerance)");
            return;
        }
        launch_or_fail(launch_project_set(m0.src, n, wp, sp, outs, (int)m0.in_dim, f(xb), (int)rows, yp, d_err_,
                                          stream_),
                       "project");
    }

    // reference.rs:402-416: the classifier over row 0 of x.
    void logits(uint64_t w, kernrt_buf x, kernrt_buf y) { project(w, x, y, 1); }

    // The key/value caches, [n_layers][seq_len][kv_dim] f32 each, zeroed
    // (KvSpec, mod.rs:169-177).
    void kv_prepare(size_t n_layers, size_t kv_dim, size_t seq_len) {
        if (n_layers == 0 || kv_dim == 0 || seq_len == 0) fail(KERNRT_E_INVALID, "empty key/value cache");
        if (seq_len > (size_t)INT32_MAX || kv_dim > (size_t)INT32_MAX || n_layers * seq_len > (size_t)INT32_MAX)
            fail(KERNRT_E_INVALID, "key/value cache too large");
        flush();
        check(cudaStreamSynchronize(stream_), "synchronize");
        cudaFree(kc_);
        cudaFree(vc_);
        kc_ = vc_ = nullptr;
        const size_t bytes = n_layers * seq_len * kv_dim * sizeof(float);
        check(cudaMalloc(&kc_, bytes), "cudaMalloc(key cache)");
        check(cudaMalloc(&vc_, bytes), "cudaMalloc(value cache)");
        check(cudaMemsetAsync(kc_, 0, bytes, stream_), "cudaMemset");
        check(cudaMemsetAsync(vc_, 0, bytes, stream_), "cudaMemset");
        kv_layers_ = n_layers;
        kv_dim_ = kv_dim;
        kv_seq_ = seq_len;
    }

    // reference.rs:151-159: row i of k and v into slot slots[i] of `layer`.
    void kv_write(size_t layer, const uint64_t *slots, size_t n_slots, kernrt_buf k, kernrt_buf v, size_t rows) {
        if (!kc_) fail(KERNRT_E_STATE, "kv_prepare() runs before kv_write");
        if (layer >= kv_layers_) fail(KERNRT_E_INVALID, "layer out of range of the key/value cache");
        distinct(k, v);
        rows = std::min(rows, n_slots);
        Buffer &kb = buf(k), &vb = buf(v);
        span(kb, 0, rows * kv_dim_, "kv_write k");
        span(vb, 0, rows * kv_dim_, "kv_write v");
        std::vector<int32_t> dst(rows);
        if (rows > 0) {
            if (!slots) {
                flush();
                fail(KERNRT_E_INVALID, "null slots");
            }
            for (size_t i = 0; i < rows; ++i) {
                if (slots[i] >= kv_seq_) {
                    flush();
                    fail(KERNRT_E_INVALID, "slot " + std::to_string(slots[i]) + " out of range");
                }
                dst[i] = (int32_t)(layer * kv_seq_ + slots[i]);
            }
        }
        // the driver's rope(q, k) right before: one launch for both
        if (prope_.on && rows > 0 && prope_.k == k && prope_.rows == rows && v != prope_.q) {
            PendRope p = std::move(prope_);
            prope_ = PendRope{};
            flush();
            const int32_t *dpos = static_cast<const int32_t *>(stage(p.pos.data(), rows * sizeof(int32_t), true));
            const int32_t *d = static_cast<const int32_t *>(stage(dst.data(), rows * sizeof(int32_t), true));
            launch_or_fail(launch_rope_kv(f(buf(p.q)), f(kb), (int)p.qw, (int)p.kvw, (int)rows, (int)p.head, dpos,
                                          p.cos, p.sin, p.max_pos, d_err_, f(vb), kc_, vc_, d, stream_),
                           "rope+kv_write");
            return;
        }
        flush();
        if (rows == 0) return;
        const int32_t *d = static_cast<const int32_t *>(stage(dst.data(), rows * sizeof(int32_t), true));
        launch_or_fail(launch_kv_write(kc_, vc_, (int)kv_dim_, d, f(kb), f(vb), (int)rows, stream_), "kv_write");
    }

    // reference.rs:276-306: one query row per window; scores to att
    // [row][head][seq_len], output [row][n_heads * head_size].
    void attention(kernrt_buf q, kernrt_buf out, kernrt_buf att, size_t layer, const kernrt_window *windows,
                   size_t n_windows, size_t n_heads, size_t kv_mul, size_t head_size, size_t kv_dim,
                   size_t seq_len) {
        if (!kc_) fail(KERNRT_E_STATE, "kv_prepare() runs before attention");
        if (layer >= kv_layers_) fail(KERNRT_E_INVALID, "layer out of range of the key/value cache");
        if (kv_dim != kv_dim_ || seq_len != kv_seq_) fail(KERNRT_E_INVALID, "attention spec does not match the cache");
        if (n_heads == 0 || head_size == 0 || kv_mul == 0) fail(KERNRT_E_INVALID, "empty attention spec");
        if (((n_heads - 1) / kv_mul + 1) * head_size > kv_dim)
            fail(KERNRT_E_INVALID, "key/value heads exceed kv_dim");
        distinct(q, out);
        if (att == q || att == out) fail(KERNRT_E_INVALID, "buffers must be distinct");
        const size_t width = n_heads * head_size;
        Buffer &qb = buf(q), &ob = buf(out), &ab = buf(att);
        span(qb, 0, n_windows * width, "attention q");
        span(ob, 0, n_windows * width, "attention out");
        span(ab, 0, n_windows * n_heads * seq_len, "attention att");
        fits_int(n_windows * n_heads, "attention");
        flush();
        if (n_windows == 0) return;
        if (!windows) fail(KERNRT_E_INVALID, "null windows");
        std::vector<int32_t> win(4 * n_windows);
        size_t max_count = 0;
        for (size_t i = 0; i < n_windows; ++i) {
            const kernrt_window &w = windows[i];
            if (w.slot < w.att_start || w.shared_end < w.shared_start || w.slot >= seq_len || w.shared_end > seq_len)
                fail(KERNRT_E_INVALID, "window " + std::to_string(i) + " out of range");
            const size_t count = (size_t)(w.shared_end - w.shared_start) + (size_t)(w.slot - w.att_start) + 1;
            if (count > seq_len) fail(KERNRT_E_INVALID, "window " + std::to_string(i) + " longer than seq_len");
            max_count = std::max(max_count, count);
            win[4 * i] = (int32_t)w.att_start;
            win[4 * i + 1] = (int32_t)w.slot;
            win[4 * i + 2] = (int32_t)w.shared_start;
            win[4 * i + 3] = (int32_t)w.shared_end;
        }
        if (attention_smem_bytes((int)head_size, (int)max_count) > 200 * 1024)
            fail(KERNRT_E_INVALID, "attention window too long for one SM's shared memory");
        // Tolerance mode, decode-sized calls (at most 4 windows): the window
        // in chunks summed in parallel (prefill keeps the exact kernels, whose
        // row-tiled scores share key tiles and measured faster there).
        const bool tol_att = !exact_ && n_windows <= 4;
        // raw scores (or the chunks' partial sums) go to a scratch the backend
        // keeps (grown, never shrunk)
        const size_t need =
            (tol_att ? attention_tol_scratch_floats((int)n_windows, (int)n_heads, (int)head_size, (int)max_count)
                     : attention_scratch_floats((int)n_windows, (int)n_heads, (int)max_count)) *
            sizeof(float);
        if (need > att_scratch_bytes_) {
            check(cudaStreamSynchronize(stream_), "synchronize");
            cudaFree(att_scratch_);
            att_scratch_ = nullptr;
            att_scratch_bytes_ = 0;
            check(cudaMalloc(&att_scratch_, need), "cudaMalloc(attention scratch)");
            att_scratch_bytes_ = need;
        }
        // windows that differ only in their last slot map positions alike
        bool shared_map = true;
        for (size_t i = 1; i < n_windows && shared_map; ++i)
            shared_map = win[4 * i] == win[0] && win[4 * i + 2] == win[2] && win[4 * i + 3] == win[3];
        const int32_t *d = static_cast<const int32_t *>(stage(win.data(), win.size() * sizeof(int32_t)));
        if (tol_att) {
            launch_or_fail(launch_attention_tol(f(qb), f(ob), f(ab), kc_, vc_, d, (int)n_windows, (int)n_heads,
                                                (int)kv_mul, (int)head_size, (int)kv_dim, (int)seq_len,
                                                layer * seq_len * kv_dim, (int)max_count, att_scratch_, stream_),
                           "attention (tolerance)");
            return;
        }
        launch_or_fail(launch_attention(f(qb), f(ob), f(ab), kc_, vc_, d, (int)n_windows, (int)n_heads, (int)kv_mul,
                                        (int)head_size, (int)kv_dim, (int)seq_len, layer * seq_len * kv_dim,
                                        (int)max_count, att_scratch_, shared_map, d_err_, stream_),
                       "attention");
    }

    // ---- row ops ----------------------------------------------------------------
    void copy(kernrt_buf src, size_t so, kernrt_buf dst, size_t d_o, size_t len) {
        Buffer &s = buf(src), &d = buf(dst);
        span(s, so, len, "copy source");
        span(d, d_o, len, "copy destination");
        flush();
        if (len == 0) return;
        char *sp = s.ptr + so * 4, *dp = d.ptr + d_o * 4;
        const size_t bytes = len * 4;
        if (src == dst && sp != dp && sp < dp + bytes && dp < sp + bytes) {
            // copy_within: overlapping ranges go through a temporary.
            void *tmp = nullptr;
            check(cudaMallocAsync(&tmp, bytes, stream_), "cudaMallocAsync");
            check(cudaMemcpyAsync(tmp, sp, bytes, cudaMemcpyDeviceToDevice, stream_), "copy");
            check(cudaMemcpyAsync(dp, tmp, bytes, cudaMemcpyDeviceToDevice, stream_), "copy");
            check(cudaFreeAsync(tmp, stream_), "cudaFreeAsync");
        } else if (sp != dp) {
            check(cudaMemcpyAsync(dp, sp, bytes, cudaMemcpyDeviceToDevice, stream_), "copy");
        }
    }

    void rms_norm(kernrt_buf out, kernrt_buf x, kernrt_buf weight, size_t rows, size_t dim, float eps) {
        distinct(out, x);
        Buffer &o = buf(out), &xi = buf(x), &w = buf(weight);
        span(o, 0, rows * dim, "rms_norm out");
        span(xi, 0, rows * dim, "rms_norm x");
        span(w, 0, dim, "rms_norm weight");
        if (rows > 0 && dim > 0 && fuse_embed_rms(out, x, weight, rows, dim, eps)) return;
        if (rows > 0 && dim > 0 && fuse_add_rms(out, x, weight, rows, dim, eps)) return;
        flush();
        if (rows == 0 || dim == 0) return;
        ChainArgs a = blank(rows, dim);
        a.eps = eps;
        a.x_in = f(xi);
        a.xb = f(o);
        a.w_att = f(w);
        a.tol = !exact_ && rows <= 4;  // decode-sized: a block reduction
        launch_or_fail(chain_launch(SRC_X, a), "rms_norm");
    }

    void qk_norm(kernrt_buf v, size_t rows, size_t width, size_t head, kernrt_buf weight, float eps) {
        if (head == 0) fail(KERNRT_E_INVALID, "head_size must be positive");
        Buffer &vb = buf(v), &w = buf(weight);
        span(vb, 0, rows * width, "qk_norm v");
        span(w, 0, head, "qk_norm weight");
        fits_int(rows * width, "qk_norm");
        // Deferred: a following rope over the same rows runs both in one pass.
        if (pqk_.n == 1 && pqk_.rows == rows && pqk_.head == head && pqk_.eps == eps && pqk_.v[0] != v) {
            pqk_.v[1] = v;
            pqk_.width[1] = width;
            pqk_.w[1] = weight;
            pqk_.n = 2;
            return;
        }
        flush();
        pqk_ = PendQK{};
        pqk_.n = 1;
        pqk_.v[0] = v;
        pqk_.width[0] = width;
        pqk_.w[0] = weight;
        pqk_.rows = rows;
        pqk_.head = head;
        pqk_.eps = eps;
    }

    void rope(kernrt_buf q, kernrt_buf k, size_t qw, size_t kvw, size_t rows, const uint64_t *positions,
              size_t n_positions, size_t head, float theta, int interleaved) {
        // a rope still held back launches first: the table lookup below may
        // replace (and free, stream-ordered) the table it reads.  Nothing else
        // is pending beside it.
        if (prope_.on) flush();
        distinct(q, k);
        if (head == 0 || head % 2) fail(KERNRT_E_INVALID, "head_size must be a positive even number");
        if (interleaved && kvw % 2) fail(KERNRT_E_INVALID, "interleaved RoPE needs an even kv width");
        rows = std::min(rows, n_positions);
        Buffer &qb = buf(q), &kb = buf(k);
        span(qb, 0, rows * qw, "rope q");
        span(kb, 0, rows * kvw, "rope k");
        fits_int(rows * std::max(qw, kvw), "rope");
        if (rows == 0) {
            flush();
            return;
        }
        if (!positions) fail(KERNRT_E_INVALID, "null positions");
        std::vector<int32_t> pos(rows);
        uint64_t maxp = 0;
        for (size_t i = 0; i < rows; ++i) {
            if (positions[i] > (uint64_t)INT32_MAX - 1) fail(KERNRT_E_INVALID, "position too large");
            pos[i] = (int32_t)positions[i];
            maxp = std::max(maxp, positions[i]);
        }
        const RopeTable &t = rope_table(theta, head, (size_t)maxp + 1);
        // A pending qk_norm of q and/or k over exactly these rows fuses in.
        const float *wq = nullptr, *wk = nullptr;
        bool fuse = pqk_.n > 0 && pqk_.rows == rows && pqk_.head == head;
        for (int i = 0; fuse && i < pqk_.n; ++i) {
            if (pqk_.v[i] == q && pqk_.width[i] == qw) wq = f(buf(pqk_.w[i]));
            else if (pqk_.v[i] == k && pqk_.width[i] == kvw) wk = f(buf(pqk_.w[i]));
            else fuse = false;
        }
        if (!fuse) wq = wk = nullptr;
        float eps = pqk_.eps;
        if (fuse) pqk_.n = 0;
        flush();
        if (!fuse && !interleaved && kc_ && kvw == kv_dim_ && kvw % head == 0) {
            prope_.on = true;
            prope_.q = q;
            prope_.k = k;
            prope_.qw = qw;
            prope_.kvw = kvw;
            prope_.rows = rows;
            prope_.head = head;
            prope_.pos = std::move(pos);
            prope_.cos = t.cos;
            prope_.sin = t.sin;
            prope_.max_pos = (int)t.max_pos;
            return;
        }
        const int32_t *dpos = static_cast<const int32_t *>(stage(pos.data(), rows * sizeof(int32_t), true));
        if (fuse) {
            launch_or_fail(launch_qk_rope(f(qb), f(kb), (int)qw, (int)kvw, (int)rows, (int)head, wq, wk, eps, dpos,
                                          t.cos, t.sin, (int)t.max_pos, interleaved, d_err_, stream_),
                           "qk_norm+rope");
            return;
        }
        launch_or_fail(launch_rope(f(qb), f(kb), (int)qw, (int)kvw, (int)rows, (int)head, dpos, t.cos, t.sin,
                                   (int)t.max_pos, interleaved, d_err_, stream_),
                       "rope");
    }

    void add_in_place(kernrt_buf dst, kernrt_buf src, size_t len) {
        distinct(dst, src);
        Buffer &d = buf(dst), &s = buf(src);
        span(d, 0, len, "add dst");
        span(s, 0, len, "add src");
        flush();
        // Deferred: a following rms_norm of dst runs both in one pass.
        padd_ = PendAdd{dst, src, len};
    }

    void mul(kernrt_buf out, size_t oo, kernrt_buf a, size_t ao, kernrt_buf b, size_t bo, size_t len) {
        Buffer &ob = buf(out), &ab = buf(a), &bb = buf(b);
        span(ob, oo, len, "mul out");
        span(ab, ao, len, "mul a");
        span(bb, bo, len, "mul b");
        if (len == 0) {
            flush();
            return;
        }
        // Consecutive calls on the same three distinct buffers with constant
        // offset strides (the LFM2 driver's per-row calls) run as one launch.
        if (out != a && out != b) {
            if (pmul_.count > 0 && pmul_.out == out && pmul_.a == a && pmul_.b == b && pmul_.len == len) {
                const long long so = (long long)oo - (long long)pmul_.oo, sa = (long long)ao - (long long)pmul_.ao,
                                sb = (long long)bo - (long long)pmul_.bo;
                const long long c = pmul_.count;
                bool ok;
                if (c == 1) ok = (so >= (long long)len || so <= -(long long)len);
                else ok = so == c * pmul_.so && sa == c * pmul_.sa && sb == c * pmul_.sb;
                if (ok) {
                    if (c == 1) {
                        pmul_.so = so;
                        pmul_.sa = sa;
                        pmul_.sb = sb;
                    }
                    pmul_.count += 1;
                    return;
                }
            }
            flush();
            pmul_ = PendMul{out, a, b, oo, ao, bo, len, 0, 0, 0, 1};
            return;
        }
        flush();
        // A write of one index can feed another index's read only when out
        // shares a buffer with an operand at a different, overlapping offset.
        auto hazard = [&](kernrt_buf x, size_t xo) {
            return x == out && xo != oo && (xo < oo ? oo - xo : xo - oo) < len;
        };
        const bool seq = hazard(a, ao) || hazard(b, bo);
        launch_or_fail(launch_mul(f(ob) + oo, f(ab) + ao, f(bb) + bo, len, seq, stream_), "mul");
    }

    void conv_prefill(kernrt_buf out, kernrt_buf x, kernrt_buf kernel, size_t rows, size_t dim, size_t k) {
        if (k == 0) fail(KERNRT_E_INVALID, "conv kernel size must be positive");
        Buffer &ob = buf(out), &xb = buf(x), &kb = buf(kernel);
        span(ob, 0, rows * dim, "conv out");
        span(xb, 0, rows * dim, "conv x");
        span(kb, 0, dim * k, "conv kernel");
        fits_int(rows * dim, "conv_prefill");
        flush();
        if (rows * dim == 0) return;
        // The reference reads cloned inputs (reference.rs:366-369): an aliased
        // input is snapshotted first.
        const float *xp = f(xb), *kp = f(kb);
        void *tx = nullptr, *tk = nullptr;
        if (x == out) {
            check(cudaMallocAsync(&tx, rows * dim * 4, stream_), "cudaMallocAsync");
            check(cudaMemcpyAsync(tx, xp, rows * dim * 4, cudaMemcpyDeviceToDevice, stream_), "copy");
            xp = static_cast<const float *>(tx);
        }
        if (kernel == out) {
            check(cudaMallocAsync(&tk, dim * k * 4, stream_), "cudaMallocAsync");
            check(cudaMemcpyAsync(tk, kp, dim * k * 4, cudaMemcpyDeviceToDevice, stream_), "copy");
            kp = static_cast<const float *>(tk);
        }
        const cudaError_t e = launch_conv_prefill(f(ob), xp, kp, (int)rows, (int)dim, (int)k, stream_);
        if (tx) cudaFreeAsync(tx, stream_);
        if (tk) cudaFreeAsync(tk, stream_);
        launch_or_fail(e, "conv_prefill");
    }

    void conv_decode(kernrt_buf out, kernrt_buf x, kernrt_buf kernel, kernrt_buf state, size_t dim, size_t k) {
        if (k == 0) fail(KERNRT_E_INVALID, "conv kernel size must be positive");
        if (state == out || state == x || state == kernel)
            fail(KERNRT_E_INVALID, "conv_decode state must be distinct from out, x and kernel");
        if (kernel == out) fail(KERNRT_E_INVALID, "conv_decode kernel must be distinct from out");
        Buffer &ob = buf(out), &xb = buf(x), &kb = buf(kernel), &sb = buf(state);
        span(ob, 0, dim, "conv_decode out");
        span(xb, 0, dim, "conv_decode x");
        span(kb, 0, dim * k, "conv_decode kernel");
        span(sb, 0, (k - 1) * dim, "conv_decode state");
        fits_int(dim * k, "conv_decode");
        flush();
        launch_or_fail(launch_conv_decode(f(ob), f(xb), f(kb), f(sb), (int)dim, (int)k, stream_), "conv_decode");
    }

    void silu_mul(kernrt_buf gate, kernrt_buf up, size_t len) {
        distinct(gate, up);
        Buffer &g = buf(gate), &u = buf(up);
        span(g, 0, len, "silu gate");
        span(u, 0, len, "silu up");
        flush();
        launch_or_fail(launch_silu_mul(f(g), f(u), len, stream_), "silu_mul");
    }

    // ---- Q8_0 -----------------------------------------------------------------
    void quantize_q8_0(kernrt_buf x, size_t rows, size_t dim, kernrt_buf codes, kernrt_buf scales,
                       kernrt_buf scales16) {
        Buffer &xb = buf(x);
        span(xb, 0, rows * dim, "quantize x");
        int8_t *c;
        float *s;
        uint16_t *h;
        q8_outputs(rows, dim, codes, scales, scales16, &c, &s, &h);
        fits_int(rows * dim, "quantize");
        flush();
        launch_or_fail(launch_quantize_q8(f(xb), (int)rows, (int)dim, c, s, h, stream_), "quantize_q8_0");
    }

    void rms_norm_q8_0(kernrt_buf x, kernrt_buf weight, size_t rows, size_t dim, float eps, kernrt_buf codes,
                       kernrt_buf scales, kernrt_buf scales16) {
        Buffer &xb = buf(x), &w = buf(weight);
        span(xb, 0, rows * dim, "rms_norm_q8_0 x");
        span(w, 0, dim, "rms_norm_q8_0 weight");
        ChainArgs a = blank(rows, dim);
        q8_outputs(rows, dim, codes, scales, scales16, &a.codes, &a.scales, &a.scales16);
        flush();
        if (rows == 0 || dim == 0) return;
        a.eps = eps;
        a.final_eps = eps;
        a.x_in = f(xb);
        a.w_final = f(w);
        launch_or_fail(chain_launch(SRC_X, a), "rms_norm_q8_0");
    }

    // ---- fused chains -------------------------------------------------------------
    void rope_prepare(float theta, size_t head, size_t max_pos) {
        if (head == 0 || head % 2) fail(KERNRT_E_INVALID, "head_size must be a positive even number");
        flush();
        rope_table(theta, head, max_pos);
    }

    void layer_chain(const kernrt_chain_args &c) {
        const size_t rows = c.rows, dim = c.dim;
        if (rows == 0) return;
        if (dim == 0) fail(KERNRT_E_INVALID, "chain dim must be positive");
        fits_int(rows * std::max({dim, c.q_dim, c.kv_dim, c.hidden}), "layer_chain");
        ChainArgs a = blank(rows, dim);
        a.eps = c.eps;
        a.final_eps = c.final_eps;
        int src = SRC_X;
        if (!c.x) fail(KERNRT_E_INVALID, "chain needs x");
        Buffer &xb = buf(c.x);
        span(xb, 0, rows * dim, "chain x");
        if (c.tokens) {
            if (emb_kind_ < 0) fail(KERNRT_E_STATE, "prepare() runs before compute");
            if (dim != dim_) fail(KERNRT_E_INVALID, "chain dim differs from the embedding width");
            Buffer &tb = buf(c.tokens);
            if (tb.bytes < rows * 4) fail(KERNRT_E_INVALID, "chain tokens buffer too small");
            src = emb_src_;
            a.table = emb_data_;
            a.tscales = emb_scales_;
            a.vocab = (int)vocab_;
            a.tokens = reinterpret_cast<const int32_t *>(tb.ptr);
            a.x_out = f(xb);
            a.row_scale = row_scales(rows);
        } else {
            a.x_in = f(xb);
            if (c.resid) a.x_out = f(xb);
        }
        if (!c.w_att) fail(KERNRT_E_INVALID, "chain needs w_att");
        a.w_att = f(buf(c.w_att));
        span(buf(c.w_att), 0, dim, "chain w_att");
        if (c.xb) {
            if (c.xb == c.x) fail(KERNRT_E_INVALID, "buffers must be distinct (xb, x)");
            span(buf(c.xb), 0, rows * dim, "chain xb");
            a.xb = f(buf(c.xb));
        }
        if (c.resid) {
            if (c.resid == c.x) fail(KERNRT_E_INVALID, "buffers must be distinct (resid, x)");
            span(buf(c.resid), 0, rows * dim, "chain resid");
            a.resid = f(buf(c.resid));
        }
        const size_t head = c.head_size;
        if (c.q || c.k || c.w_q || c.w_k) {
            if (head == 0 || head % 2) fail(KERNRT_E_INVALID, "head_size must be a positive even number");
            if (c.q && c.k && c.q == c.k) fail(KERNRT_E_INVALID, "buffers must be distinct (q, k)");
            if (c.interleaved && c.kv_dim % 2) fail(KERNRT_E_INVALID, "interleaved RoPE needs an even kv width");
            a.head = (int)head;
            a.half = (int)(head / 2);
            a.q_dim = (int)c.q_dim;
            a.kv_dim = (int)c.kv_dim;
            if (c.q) { span(buf(c.q), 0, rows * c.q_dim, "chain q"); a.q = f(buf(c.q)); }
            if (c.k) { span(buf(c.k), 0, rows * c.kv_dim, "chain k"); a.k = f(buf(c.k)); }
            if (c.w_q) { span(buf(c.w_q), 0, head, "chain w_q"); a.w_q = f(buf(c.w_q)); }
            if (c.w_k) { span(buf(c.w_k), 0, head, "chain w_k"); a.w_k = f(buf(c.w_k)); }
            if ((c.q || c.k) && c.positions) {
                Buffer &pb = buf(c.positions);
                if (pb.bytes < rows * 4) fail(KERNRT_E_INVALID, "chain positions buffer too small");
                const RopeTable *t = find_rope(c.theta, head);
                if (!t) fail(KERNRT_E_STATE, "kernrt_cuda_rope_prepare runs before a chain with RoPE");
                a.pos = reinterpret_cast<const int32_t *>(pb.ptr);
                a.cos_t = t->cos;
                a.sin_t = t->sin;
                a.max_pos = (int)t->max_pos;
                a.rope_mode = c.interleaved ? 2 : 1;
            }
        }
        if (c.gate) {
            if (!c.up || c.up == c.gate) fail(KERNRT_E_INVALID, "buffers must be distinct (gate, up)");
            span(buf(c.gate), 0, rows * c.hidden, "chain gate");
            span(buf(c.up), 0, rows * c.hidden, "chain up");
            a.gate = f(buf(c.gate));
            a.up = f(buf(c.up));
            a.hidden = (int)c.hidden;
        }
        if (c.w_final) {
            span(buf(c.w_final), 0, dim, "chain w_final");
            a.w_final = f(buf(c.w_final));
            q8_outputs(rows, dim, c.codes, c.scales, c.scales_f16, &a.codes, &a.scales, &a.scales16);
        }
        flush();
        launch_or_fail(chain_launch(src, a), "layer_chain");
    }

    // `halo` (< k) leading rows of bcx belong to the rows before this shard of
    // the sequence: they feed h and give no output; cy gets `rows` rows.  A 0
    // ring handle skips the ring (a shard that does not end the sequence).
    void lfm2_conv_block(kernrt_buf bcx, kernrt_buf kernel, kernrt_buf ring, kernrt_buf cy, size_t rows,
                         size_t dim, size_t k, size_t halo = 0) {
        if (k == 0) fail(KERNRT_E_INVALID, "conv kernel size must be positive");
        if (halo >= k) fail(KERNRT_E_INVALID, "conv block halo must be shorter than the kernel");
        if (cy == bcx || (ring && (ring == bcx || ring == cy))) fail(KERNRT_E_INVALID, "buffers must be distinct");
        if (ring && halo && rows < k - 1) fail(KERNRT_E_INVALID, "a shard that seeds the ring needs k - 1 rows");
        span(buf(bcx), 0, (halo + rows) * 3 * dim, "conv block bcx");
        span(buf(kernel), 0, dim * k, "conv block kernel");
        span(buf(cy), 0, rows * dim, "conv block cy");
        if (ring && k > 1) span(buf(ring), 0, (k - 1) * dim, "conv block ring");
        fits_int((halo + rows) * 3 * dim, "lfm2_conv_block");
        flush();
        if (rows == 0) return;
        launch_or_fail(launch_lfm2_conv_block(f(buf(bcx)), f(buf(kernel)), ring ? f(buf(ring)) : nullptr, f(buf(cy)),
                                              (int)(halo + rows), (int)dim, (int)k, stream_, (int)halo),
                       "lfm2_conv_block");
    }

    // ---- the chain on host buffers, pipelined over row chunks --------------------
    // Chunk i uses device buffer set i % 3: its inputs go up on h2d_, the chain
    // runs on stream_, its outputs come back on d2h_, each step waiting on the
    // previous one's event for that set; a set is refilled only after its last
    // outputs left (h2d_ waits on d2h_done).  So the copies of chunk i+1 and
    // i-1 overlap the kernels of chunk i.
    void layer_chain_host(const kernrt_chain_host_args &h) {
        const size_t rows = h.rows, dim = h.dim;
        if (rows == 0) return;
        if (dim == 0) fail(KERNRT_E_INVALID, "chain dim must be positive");
        fits_int(rows * std::max({dim, h.q_dim, h.kv_dim, h.hidden}), "layer_chain_host");
        const bool has_q = h.q_in != nullptr, has_k = h.k_in != nullptr, has_g = h.gate_in != nullptr;
        if ((has_q && !h.q_out) || (has_k && !h.k_out) || (has_g && (!h.gate_out || !h.up)))
            fail(KERNRT_E_INVALID, "every streamed input needs its output (and gate needs up)");
        if (!h.tokens && !h.x_in) fail(KERNRT_E_INVALID, "chain needs token ids or x");
        if (!h.w_att) fail(KERNRT_E_INVALID, "chain needs w_att");
        span(buf(h.w_att), 0, dim, "chain w_att");
        const size_t head = h.head_size;
        if (has_q || has_k || h.w_q || h.w_k) {
            if (head == 0 || head % 2) fail(KERNRT_E_INVALID, "head_size must be a positive even number");
            if (h.interleaved && h.kv_dim % 2) fail(KERNRT_E_INVALID, "interleaved RoPE needs an even kv width");
        }
        if (h.w_q) span(buf(h.w_q), 0, head, "chain w_q");
        if (h.w_k) span(buf(h.w_k), 0, head, "chain w_k");
        if (h.w_final) {
            span(buf(h.w_final), 0, dim, "chain w_final");
            if (!h.codes || !h.scales) fail(KERNRT_E_INVALID, "the final Q8_0 stage needs codes and scales");
        }
        if (h.tokens) {
            if (emb_kind_ < 0) fail(KERNRT_E_STATE, "prepare() runs before compute");
            if (dim != dim_) fail(KERNRT_E_INVALID, "chain dim differs from the embedding width");
            for (size_t r = 0; r < rows; ++r)
                if (h.tokens[r] < 0 || (size_t)h.tokens[r] >= vocab_)
                    fail(KERNRT_E_INVALID, "token " + std::to_string(h.tokens[r]) + " at row " + std::to_string(r) +
                                               " out of range for vocab " + std::to_string(vocab_));
        }
        const RopeTable *table = nullptr;
        if (has_q || has_k) {
            if (!h.positions) fail(KERNRT_E_INVALID, "null positions");
            int32_t maxp = 0;
            for (size_t r = 0; r < rows; ++r) {
                if (h.positions[r] < 0) fail(KERNRT_E_INVALID, "negative position");
                maxp = std::max(maxp, h.positions[r]);
            }
            flush();
            table = &rope_table(h.theta, head, (size_t)maxp + 1);
        }
        flush();

        // Per-row bytes of every buffer a set holds, and the chunk size.
        const size_t nb = (dim + 31) / 32;
        struct Part { size_t per_row; size_t off; };
        Part p_tok{h.tokens ? 4u : 0u, 0}, p_pos{(has_q || has_k) ? 4u : 0u, 0}, p_x{4 * dim, 0}, p_xb{h.xb_out ? 4 * dim : 0, 0},
            p_q{has_q ? 4 * h.q_dim : 0, 0}, p_k{has_k ? 4 * h.kv_dim : 0, 0}, p_g{has_g ? 4 * h.hidden : 0, 0},
            p_u{has_g ? 4 * h.hidden : 0, 0}, p_r{h.resid ? 4 * dim : 0, 0}, p_c{h.w_final ? 32 * nb : 0, 0},
            p_s{h.w_final ? 4 * nb : 0, 0}, p_h{(h.w_final && h.scales_f16) ? 2 * nb : 0, 0};
        Part *parts[] = {&p_tok, &p_pos, &p_x, &p_xb, &p_q, &p_k, &p_g, &p_u, &p_r, &p_c, &p_s, &p_h};
        size_t row_bytes = 0;
        for (Part *pt : parts) row_bytes += pt->per_row;
        size_t C = h.chunk_rows;
        // 512 MB of a chunk's buffers by default: large copies keep PCIe busy
        // (measured: 0.50 M rows/s at 64 MB, 0.51-0.52 at 256-512 MB)
        if (C == 0) C = std::max<size_t>(1, ((size_t)512 << 20) / std::max<size_t>(row_bytes, 1));
        C = std::min(C, rows);
        size_t arena = 0;
        for (Part *pt : parts) {
            pt->off = arena;
            arena += (pt->per_row * C + 255) & ~(size_t)255;
        }
        for (auto &set : sets_) {
            if (set.bytes < arena) {
                check(cudaStreamSynchronize(stream_), "synchronize");
                cudaFree(set.arena);
                set.arena = nullptr;
                set.bytes = 0;
                check(cudaMalloc(&set.arena, arena), "cudaMalloc(host pipeline)");
                set.bytes = arena;
            }
            set.used = false;
        }

        // The copy streams start after everything already queued on stream_.
        check(cudaEventRecord(sets_[0].comp_done, stream_), "cudaEventRecord");
        check(cudaStreamWaitEvent(h2d_, sets_[0].comp_done, 0), "cudaStreamWaitEvent");
        try {
            for (size_t i = 0, c0 = 0; c0 < rows; ++i, c0 += C) {
                const size_t n = std::min(C, rows - c0);
                PipeSet &S = sets_[i % 3];
                char *A = static_cast<char *>(S.arena);
                auto dev = [&](const Part &pt) { return pt.per_row ? A + pt.off : nullptr; };
                auto up_rows = [&](const Part &pt, const void *host) {
                    if (pt.per_row && host)
                        check(cudaMemcpyAsync(A + pt.off, static_cast<const char *>(host) + c0 * pt.per_row,
                                              n * pt.per_row, cudaMemcpyHostToDevice, h2d_),
                              "cudaMemcpyAsync(h2d)");
                };
                auto down_rows = [&](const Part &pt, void *host) {
                    if (pt.per_row && host)
                        check(cudaMemcpyAsync(static_cast<char *>(host) + c0 * pt.per_row, A + pt.off,
                                              n * pt.per_row, cudaMemcpyDeviceToHost, d2h_),
                              "cudaMemcpyAsync(d2h)");
                };
                if (S.used) check(cudaStreamWaitEvent(h2d_, S.d2h_done, 0), "cudaStreamWaitEvent");
                up_rows(p_tok, h.tokens);
                up_rows(p_pos, h.positions);
                if (!h.tokens) up_rows(p_x, h.x_in);
                up_rows(p_q, h.q_in);
                up_rows(p_k, h.k_in);
                up_rows(p_g, h.gate_in);
                up_rows(p_u, h.up);
                up_rows(p_r, h.resid);
                check(cudaEventRecord(S.h2d_done, h2d_), "cudaEventRecord");

                check(cudaStreamWaitEvent(stream_, S.h2d_done, 0), "cudaStreamWaitEvent");
                ChainArgs a = blank(n, dim);
                a.eps = h.eps;
                a.final_eps = h.final_eps;
                int src = SRC_X;
                if (h.tokens) {
                    src = emb_src_;
                    a.table = emb_data_;
                    a.tscales = emb_scales_;
                    a.vocab = (int)vocab_;
                    a.tokens = reinterpret_cast<const int32_t *>(dev(p_tok));
                    a.x_out = reinterpret_cast<float *>(dev(p_x));
                    a.row_scale = row_scales(n);
                } else {
                    a.x_in = reinterpret_cast<const float *>(dev(p_x));
                    if (h.resid) a.x_out = reinterpret_cast<float *>(dev(p_x));
                }
                a.w_att = f(buf(h.w_att));
                a.xb = reinterpret_cast<float *>(dev(p_xb));
                a.resid = reinterpret_cast<const float *>(dev(p_r));
                if (has_q || has_k || h.w_q || h.w_k) {
                    a.head = (int)head;
                    a.half = (int)(head / 2);
                    a.q_dim = (int)h.q_dim;
                    a.kv_dim = (int)h.kv_dim;
                    a.q = reinterpret_cast<float *>(dev(p_q));
                    a.k = reinterpret_cast<float *>(dev(p_k));
                    a.w_q = h.w_q ? f(buf(h.w_q)) : nullptr;
                    a.w_k = h.w_k ? f(buf(h.w_k)) : nullptr;
                    if (table) {
                        a.pos = reinterpret_cast<const int32_t *>(dev(p_pos));
                        a.cos_t = table->cos;
                        a.sin_t = table->sin;
                        a.max_pos = (int)table->max_pos;
                        a.rope_mode = h.interleaved ? 2 : 1;
                    }
                }
                if (has_g) {
                    a.gate = reinterpret_cast<float *>(dev(p_g));
                    a.up = reinterpret_cast<const float *>(dev(p_u));
                    a.hidden = (int)h.hidden;
                }
                if (h.w_final) {
                    a.w_final = f(buf(h.w_final));
                    a.codes = reinterpret_cast<int8_t *>(dev(p_c));
                    a.scales = reinterpret_cast<float *>(dev(p_s));
                    a.scales16 = reinterpret_cast<uint16_t *>(dev(p_h));
                }
                launch_or_fail(chain_launch(src, a), "layer_chain_host");
                check(cudaEventRecord(S.comp_done, stream_), "cudaEventRecord");

                check(cudaStreamWaitEvent(d2h_, S.comp_done, 0), "cudaStreamWaitEvent");
                down_rows(p_x, h.x_out);
                down_rows(p_xb, h.xb_out);
                down_rows(p_q, h.q_out);
                down_rows(p_k, h.k_out);
                down_rows(p_g, h.gate_out);
                down_rows(p_c, h.codes);
                down_rows(p_s, h.scales);
                down_rows(p_h, h.scales_f16);
                check(cudaEventRecord(S.d2h_done, d2h_), "cudaEventRecord");
                S.used = true;
            }
        } catch (...) {
            cudaStreamSynchronize(h2d_);
            cudaStreamSynchronize(stream_);
            cudaStreamSynchronize(d2h_);
            throw;
        }
        check(cudaStreamSynchronize(h2d_), "synchronize");
        check(cudaStreamSynchronize(d2h_), "synchronize");
        barrier();
    }

    // ---- stage timing: CUDA events around each kernel of a chain launch --------
    void stage_timing(bool on) {
        flush();
        check(cudaStreamSynchronize(stream_), "synchronize");
        timing_ = on;
        marks_.clear();
        used_events_ = 0;
    }

    // Per stage: total device milliseconds and launch count since timing began.
    void stage_times(double *ms, uint64_t *launches) {
        barrier();
        for (int i = 0; i < STAGE_COUNT; ++i) {
            ms[i] = 0.0;
            launches[i] = 0;
        }
        for (size_t i = 0; i + 1 < marks_.size(); ++i) {
            const int st = marks_[i].stage;
            if (st < 0 || st >= STAGE_COUNT) continue;
            float t = 0.0f;
            check(cudaEventElapsedTime(&t, marks_[i].ev, marks_[i + 1].ev), "cudaEventElapsedTime");
            ms[st] += t;
            launches[st] += 1;
        }
    }

    // Launch whatever is deferred: pending embeds, or the one pending op.
    void flush() {
        flush_embeds();
        flush_deferred();
    }

    void flush_deferred() {
        if (prope_.on) {
            prope_.on = false;
            const int32_t *dpos =
                static_cast<const int32_t *>(stage(prope_.pos.data(), prope_.rows * sizeof(int32_t), true));
            launch_or_fail(launch_rope(f(buf(prope_.q)), f(buf(prope_.k)), (int)prope_.qw, (int)prope_.kvw,
                                       (int)prope_.rows, (int)prope_.head, dpos, prope_.cos, prope_.sin,
                                       prope_.max_pos, 0, d_err_, stream_),
                           "rope");
        }
        if (padd_.len) {
            const PendAdd p = padd_;
            padd_ = PendAdd{};
            launch_or_fail(launch_add(f(buf(p.dst)), f(buf(p.src)), p.len, stream_), "add_in_place");
        }
        if (pqk_.n) {
            const PendQK p = pqk_;
            pqk_.n = 0;
            for (int i = 0; i < p.n; ++i)
                launch_or_fail(launch_qk_norm(f(buf(p.v[i])), (int)p.rows, (int)p.width[i], (int)p.head,
                                              f(buf(p.w[i])), p.eps, stream_),
                               "qk_norm");
        }
        if (pmul_.count) {
            const PendMul p = pmul_;
            pmul_.count = 0;
            launch_or_fail(launch_mul_strided(f(buf(p.out)) + p.oo, f(buf(p.a)) + p.ao, f(buf(p.b)) + p.bo,
                                              p.count > 1 ? p.so : 0, p.count > 1 ? p.sa : 0,
                                              p.count > 1 ? p.sb : 0, (int)p.len, (int)p.count, stream_),
                           "mul");
        }
    }

    // rms_norm right after a run of embeds that wrote exactly rows 0..rows-1
    // of x: gather, normalise and keep x in one pass.
    bool fuse_embed_rms(kernrt_buf out, kernrt_buf x, kernrt_buf weight, size_t rows, size_t dim, float eps) {
        if (pending_.size() != rows || dim != dim_ || rows > (size_t)INT32_MAX) return false;
        for (size_t r = 0; r < rows; ++r)
            if (pending_[r].out != x || pending_[r].offset != (int64_t)(r * dim)) return false;
        std::vector<int32_t> tok(rows);
        for (size_t r = 0; r < rows; ++r) tok[r] = pending_[r].token;
        pending_.clear();
        ChainArgs a = blank(rows, dim);
        a.eps = eps;
        a.tol = !exact_ && rows <= 4;  // decode-sized: a block reduction
        a.table = emb_data_;
        a.tscales = emb_scales_;
        a.vocab = (int)vocab_;
        a.tokens = static_cast<const int32_t *>(stage(tok.data(), rows * sizeof(int32_t), true));
        a.x_out = f(buf(x));
        a.xb = f(buf(out));
        a.w_att = f(buf(weight));
        launch_or_fail(chain_launch(emb_src_, a), "embed+rms_norm");
        return true;
    }

    // rms_norm of x right after add_in_place(x, src): add, normalise, one pass.
    bool fuse_add_rms(kernrt_buf out, kernrt_buf x, kernrt_buf weight, size_t rows, size_t dim, float eps) {
        if (!padd_.len || padd_.dst != x || padd_.len != rows * dim || padd_.src == out || dim % 8 != 0)
            return false;
        const PendAdd p = padd_;
        padd_ = PendAdd{};
        flush_embeds();
        ChainArgs a = blank(rows, dim);
        a.eps = eps;
        a.x_in = f(buf(x));
        a.x_out = f(buf(x));
        a.resid = f(buf(p.src));
        a.xb = f(buf(out));
        a.w_att = f(buf(weight));
        a.tol = !exact_ && rows <= 4;  // decode-sized: a block reduction
        launch_or_fail(launch_add_rms_norm(a, stream_), "add_in_place+rms_norm");
        return true;
    }

    // Launch all pending embeds (one gather per run of calls into one buffer).
    void flush_embeds() {
        if (pending_.empty()) return;
        const kernrt_buf out = pending_.front().out;
        const size_t n = pending_.size();
        std::vector<int32_t> tok(n);
        std::vector<int64_t> off(n);
        bool aligned = true;
        for (size_t i = 0; i < n; ++i) {
            tok[i] = pending_[i].token;
            off[i] = pending_[i].offset;
            aligned = aligned && (off[i] % 4 == 0);
        }
        pending_.clear();
        // One staging call per launch: offsets then token ids in one block.
        std::vector<unsigned char> packed(n * (sizeof(int64_t) + sizeof(int32_t)));
        std::memcpy(packed.data(), off.data(), n * sizeof(int64_t));
        std::memcpy(packed.data() + n * sizeof(int64_t), tok.data(), n * sizeof(int32_t));
        unsigned char *dev = static_cast<unsigned char *>(stage(packed.data(), packed.size(), true));
        GatherArgs g{};
        g.table = emb_data_;
        g.tscales = emb_scales_;
        g.vocab = (int)vocab_;
        g.dim = (int)dim_;
        g.dst_off = reinterpret_cast<const int64_t *>(dev);
        g.tokens = reinterpret_cast<const int32_t *>(dev + n * sizeof(int64_t));
        g.dst = f(buf(out));
        g.n = (int)n;
        g.err = d_err_;
        const bool vec = aligned && (emb_src_ == SRC_BF16 ? dim_ % 8 == 0 : emb_src_ == SRC_Q8 ? dim_ % 16 == 0 : dim_ % 4 == 0);
        launch_or_fail(launch_embed_gather(emb_src_, vec, g, stream_), "embed");
    }

private:
    struct Buffer {
        char *ptr = nullptr;
        size_t bytes = 0;
    };
    struct RopeTable {
        float theta;
        size_t head;
        size_t max_pos;
        float *cos = nullptr;
        float *sin = nullptr;
    };
    struct Pending {
        int32_t token;
        kernrt_buf out;
        int64_t offset;
    };

    Buffer &buf(kernrt_buf h) {
        if (h == 0 || h > bufs_.size()) fail(KERNRT_E_INVALID, "invalid buffer handle " + std::to_string(h));
        return bufs_[h - 1];
    }
    static float *f(Buffer &b) { return reinterpret_cast<float *>(b.ptr); }
    static void span(const Buffer &b, size_t off, size_t len, const char *what) {
        const size_t n = b.bytes / 4;
        if (off > n || len > n - off)
            fail(KERNRT_E_INVALID, std::string(what) + ": range [" + std::to_string(off) + ", " +
                                       std::to_string(off + len) + ") outside a buffer of " + std::to_string(n));
    }
    static void distinct(kernrt_buf a, kernrt_buf b) {
        if (a == b) fail(KERNRT_E_INVALID, "buffers must be distinct");
    }
    static void fits_int(size_t n, const char *what) {
        if (n > (size_t)INT32_MAX) fail(KERNRT_E_INVALID, std::string(what) + ": too many elements for one launch");
    }
    static void launch_or_fail(cudaError_t e, const char *what) { check(e, what); }

    // Scratch for `rows` row scales of a chain on stream_, grown as needed
    // (cudaFree waits for queued kernels that may still read the old one).
    float *row_scales(size_t rows) {
        if (rows > row_scales_cap_) {
            cudaFree(row_scales_);
            row_scales_ = nullptr;
            row_scales_cap_ = 0;
            check(cudaMalloc(&row_scales_, rows * sizeof(float)), "cudaMalloc(row scales)");
            row_scales_cap_ = rows;
        }
        return row_scales_;
    }

    ChainArgs blank(size_t rows, size_t dim) const {
        ChainArgs a{};
        a.rows = (int)rows;
        a.dim = (int)dim;
        a.err = d_err_;
        a.ticket = d_ticket_;  // every chain launches on stream_
        return a;
    }

    void q8_outputs(size_t rows, size_t dim, kernrt_buf codes, kernrt_buf scales, kernrt_buf scales16,
                    int8_t **c, float **s, uint16_t **h) {
        const size_t nb = (dim + 31) / 32;
        Buffer &cb = buf(codes), &sb = buf(scales);
        if (cb.bytes < rows * nb * 32) fail(KERNRT_E_INVALID, "codes buffer too small");
        if (sb.bytes < rows * nb * 4) fail(KERNRT_E_INVALID, "scales buffer too small");
        *c = reinterpret_cast<int8_t *>(cb.ptr);
        *s = reinterpret_cast<float *>(sb.ptr);
        *h = nullptr;
        if (scales16) {
            Buffer &hb = buf(scales16);
            if (hb.bytes < rows * nb * 2) fail(KERNRT_E_INVALID, "f16 scales buffer too small");
            *h = reinterpret_cast<uint16_t *>(hb.ptr);
        }
    }

    const RopeTable *find_rope(float theta, size_t head) const {
        for (const auto &t : ropes_)
            if (t.theta == theta && t.head == head) return &t;
        return nullptr;
    }

    // The table for (theta, head) covering positions < need, built or grown.
    const RopeTable &rope_table(float theta, size_t head, size_t need) {
        RopeTable *t = nullptr;
        for (auto &r : ropes_)
            if (r.theta == theta && r.head == head) t = &r;
        if (t && t->max_pos >= need) return *t;
        size_t cap = std::max<size_t>(need, 4096);
        if (t) cap = std::max(cap, 2 * t->max_pos);
        const size_t half = head / 2, n = cap * half;
        std::vector<float> hc(n), hs(n);
        build_rope_table(theta, (int)head, cap, hc.data(), hs.data());
        if (!t) {
            ropes_.push_back(RopeTable{theta, head, 0, nullptr, nullptr});
            t = &ropes_.back();
        }
        // Stream-ordered: the old table is freed after the work that may
        // still read it, the new one is allocated and filled in order, and
        // nothing waits on the host (the copies from pageable vectors return
        // once their source is staged).
        if (t->cos) check(cudaFreeAsync(t->cos, stream_), "cudaFreeAsync(rope)");
        if (t->sin) check(cudaFreeAsync(t->sin, stream_), "cudaFreeAsync(rope)");
        t->cos = t->sin = nullptr;
        t->max_pos = 0;
        check(cudaMallocAsync(reinterpret_cast<void **>(&t->cos), n * 4, stream_), "cudaMallocAsync(rope)");
        check(cudaMallocAsync(reinterpret_cast<void **>(&t->sin), n * 4, stream_), "cudaMallocAsync(rope)");
        check(cudaMemcpyAsync(t->cos, hc.data(), n * 4, cudaMemcpyHostToDevice, stream_), "upload rope table");
        check(cudaMemcpyAsync(t->sin, hs.data(), n * 4, cudaMemcpyHostToDevice, stream_), "upload rope table");
        t->max_pos = cap;
        return *t;
    }

    // Copy a host slice into the pinned ring and enqueue its upload; returns
    // the device address.  With `in_place`, a slice of a few values (a decode
    // step's token id, position or cache slot, which its kernel reads about
    // once per row) is not uploaded: the kernel reads it from the pinned ring
    // through the ring's device mapping, which saves the copy call on the host
    // and the copy in the stream ahead of the kernel.  Slices that kernels read
    // many times over (attention windows) are always uploaded: each of those
    // reads would cross PCIe.  Each launch takes its staged data from one call,
    // made right before the launch, so when a call starts, the consumers of
    // everything staged before it are enqueued.  The ring is cut into
    // kStageSegs segments: leaving a segment records an event after those
    // consumers, and entering a segment waits for the event recorded when the
    // ring last left it (a whole ring earlier, normally long complete), so a
    // region is never rewritten while a copy from it or a kernel reading it
    // may be pending, and the stream is never drained.  A slice larger than a
    // segment grows the ring; the old one is retired, not freed, until the
    // next barrier.
    static constexpr int kStageSegs = 8;
    static constexpr size_t kStageMapped = 64;  // slices read in place through the mapping
    void *stage(const void *src, size_t bytes, bool in_place = false) {
        const size_t need = (bytes + 255) & ~(size_t)255;
        size_t seg = stage_cap_ / kStageSegs;
        if (need > seg) {
            grow_staging(kStageSegs * std::max<size_t>(2 * need, 1 << 17));
            seg = stage_cap_ / kStageSegs;
        }
        // The segment in use is kept apart from the offset in it: a slice
        // that ends exactly at a segment's end leaves the offset at the end,
        // and the next slice then moves on through the event hand-over (an
        // offset taken from one running head would slip into the next
        // segment, or past the ring's end, without it).
        if (stage_off_ + need > seg) {  // into the next segment
            const size_t next = (stage_seg_ + 1) % kStageSegs;
            check(cudaEventRecord(stage_ev_[stage_seg_], stream_), "cudaEventRecord(staging)");
            stage_ev_set_[stage_seg_] = true;
            if (stage_ev_set_[next]) check(cudaEventSynchronize(stage_ev_[next]), "staging ring");
            stage_ev_set_[next] = false;
            stage_seg_ = next;
            stage_off_ = 0;
        }
        const size_t at = stage_seg_ * seg + stage_off_;
        stage_off_ += need;
        char *h = stage_host_ + at;
        char *d = stage_dev_ + at;
        std::memcpy(h, src, bytes);
        if (in_place && bytes <= kStageMapped && stage_map_) return stage_map_ + at;
        check(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, stream_), "stage");
        return d;
    }

    void grow_staging(size_t cap) {
        if (stage_host_ || stage_dev_) retired_.push_back({stage_host_, stage_dev_});
        stage_host_ = nullptr;
        stage_dev_ = nullptr;
        check(cudaHostAlloc(&stage_host_, cap, cudaHostAllocMapped), "cudaHostAlloc(staging)");
        check(cudaMalloc(&stage_dev_, cap), "cudaMalloc(staging)");
        void *map = nullptr;
        stage_map_ = nullptr;
        if (cudaHostGetDevicePointer(&map, stage_host_, 0) == cudaSuccess) stage_map_ = static_cast<char *>(map);
        else cudaGetLastError();  // no mapping: every slice is uploaded
        stage_cap_ = cap;
        stage_seg_ = 0;
        stage_off_ = 0;
        for (int i = 0; i < kStageSegs; ++i) {  // a new ring: every segment free
            if (!stage_ev_[i]) check(cudaEventCreateWithFlags(&stage_ev_[i], cudaEventDisableTiming), "cudaEventCreate");
            stage_ev_set_[i] = false;
        }
    }

    struct Mark {
        int stage;
        cudaEvent_t ev;
    };
    static void on_stage(void *self, int stage) {
        auto *b = static_cast<Backend *>(self);
        if (b->used_events_ == b->events_.size()) {
            cudaEvent_t e = nullptr;
            check(cudaEventCreate(&e), "cudaEventCreate");
            b->events_.push_back(e);
        }
        cudaEvent_t e = b->events_[b->used_events_++];
        check(cudaEventRecord(e, b->stream_), "cudaEventRecord");
        b->marks_.push_back({stage, e});
    }
    cudaError_t chain_launch(int src, const ChainArgs &a) {
        if (!timing_) return launch_chain(src, a, stream_);
        const LaunchHook hook{&Backend::on_stage, this};
        return launch_chain(src, a, stream_, &hook);
    }

    struct PendAdd {
        kernrt_buf dst = 0, src = 0;
        size_t len = 0;
    };
    struct PendQK {
        int n = 0;
        kernrt_buf v[2] = {0, 0};
        size_t width[2] = {0, 0};
        kernrt_buf w[2] = {0, 0};
        size_t rows = 0, head = 0;
        float eps = 0.0f;
    };
    struct PendMul {
        kernrt_buf out = 0, a = 0, b = 0;
        size_t oo = 0, ao = 0, bo = 0, len = 0;
        long long so = 0, sa = 0, sb = 0;
        long long count = 0;
    };
    // A half-split rope held back for one call: a kv_write of its k rows that
    // follows runs with it in one launch (k_rope_kv).  The positions stay on
    // the host until the launch stages them.
    struct PendRope {
        bool on = false;
        kernrt_buf q = 0, k = 0;
        size_t qw = 0, kvw = 0, rows = 0, head = 0;
        std::vector<int32_t> pos;
        const float *cos = nullptr, *sin = nullptr;
        int max_pos = 0;
    };
    PendAdd padd_;
    PendQK pqk_;
    PendMul pmul_;
    PendRope prope_;

    struct PipeSet {
        void *arena = nullptr;
        size_t bytes = 0;
        bool used = false;
        cudaEvent_t h2d_done = nullptr, comp_done = nullptr, d2h_done = nullptr;
    };
    PipeSet sets_[3];
    cudaStream_t h2d_ = nullptr, d2h_ = nullptr;

    bool timing_ = false;
    std::vector<cudaEvent_t> events_;
    size_t used_events_ = 0;
    std::vector<Mark> marks_;
    int device_;
    cudaStream_t stream_ = nullptr;
    std::vector<Buffer> bufs_;
    std::vector<RopeTable> ropes_;
    std::vector<Pending> pending_;
    std::vector<DevMatrix> mats_;
    float *kc_ = nullptr, *vc_ = nullptr;
    float *att_scratch_ = nullptr;
    size_t att_scratch_bytes_ = 0;
    size_t kv_layers_ = 0, kv_dim_ = 0, kv_seq_ = 0;
    int emb_kind_ = -1;
    int emb_src_ = SRC_F32;
    size_t vocab_ = 0, dim_ = 0;
    void *emb_data_ = nullptr;
    float *emb_scales_ = nullptr;
    void *file_pin_[2] = {nullptr, nullptr};  // page-locked file staging, kept across loads
    cudaEvent_t file_ev_[2] = {nullptr, nullptr};
    const char *storage_ = "f32";
    int *d_err_ = nullptr;
    unsigned *d_ticket_ = nullptr;  // the chain streams' work counter on stream_ (zero between launches)
    bool exact_ = true;             // false: tolerance-mode tensor-core projections (KERNRT_CUDA_EXACT=0)
    uint64_t allocs_ = 0;           // buffer allocations so far
    uint64_t fail_alloc_at_ = 0;    // the allocation to fail (KERNRT_CUDA_FAIL_ALLOC; 0 = none)
    uint16_t *split_ = nullptr;     // bf16 hi / lo halves of a projection's x
    size_t split_cap_ = 0;          // elements
    float *row_scales_ = nullptr;   // the two-pass norm stage's row scales (chains on stream_)
    size_t row_scales_cap_ = 0;
    int *h_err_ = nullptr;
    char *stage_host_ = nullptr;
    char *stage_dev_ = nullptr;
    char *stage_map_ = nullptr;  // stage_host_ as the device addresses it
    std::vector<std::pair<char *, char *>> retired_;  // grown-out staging rings, freed at the next barrier
    cudaEvent_t stage_ev_[kStageSegs] = {};  // per staging segment: recorded when the ring last left it
    bool stage_ev_set_[kStageSegs] = {};
    size_t stage_cap_ = 0, stage_seg_ = 0, stage_off_ = 0;  // the ring, its segment in use, the offset in it
};

}  // namespace krt

// =============================================================================
// C ABI
// =============================================================================

struct kernrt_cuda_ctx {
    krt::Backend *b;
};

static thread_local std::string g_last_error;

namespace krt {
void set_last_error(const std::string &msg) { g_last_error = msg; }
}  // namespace krt

template <class F>
static int guard(kernrt_cuda_ctx *ctx, F &&fn) {
    if (!ctx || !ctx->b) {
        g_last_error = "null kernrt_cuda context";
        return KERNRT_E_INVALID;
    }
    try {
        ctx->b->activate();
        fn(*ctx->b);
        return KERNRT_OK;
    } catch (const krt::Error &e) {
        g_last_error = e.msg;
        return e.code;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return KERNRT_E_CUDA;
    }
}

extern "C" {

const char *kernrt_cuda_last_error(void) { return g_last_error.c_str(); }

int kernrt_cuda_safetensors_tensor(const char *path, const char *name, kernrt_st_tensor *out) {
    if (!path || !name || !out) {
        g_last_error = "null argument";
        return KERNRT_E_INVALID;
    }
    krt::StHeader h;
    const std::string err = krt::st_read_header(path, &h);
    if (!err.empty()) {
        g_last_error = err;
        return KERNRT_E_INVALID;
    }
    const auto it = h.tensors.find(name);
    if (it == h.tensors.end()) {
        g_last_error = "weight file is missing \"" + std::string(name) + "\"";
        return KERNRT_E_INVALID;
    }
    const krt::StTensor &t = it->second;
    std::memset(out, 0, sizeof *out);
    out->dtype = t.dtype;
    out->rank = (int)t.shape.size();
    for (size_t i = 0; i < t.shape.size() && i < 8; ++i) out->shape[i] = t.shape[i];
    out->file_offset = h.data_offset + t.start;
    out->bytes = t.end - t.start;
    return KERNRT_OK;
}

int kernrt_cuda_set_exact(kernrt_cuda_ctx *ctx, int exact) {
    return guard(ctx, [&](krt::Backend &b) { b.set_exact(exact != 0); });
}

int kernrt_cuda_selftest_wait(kernrt_cuda_ctx *ctx, uint64_t cycles, int complete) {
    return guard(ctx, [&](krt::Backend &b) { b.selftest_wait(cycles, complete); });
}

int kernrt_cuda_prepare_embedding_file(kernrt_cuda_ctx *ctx, const char *path, const char *name, int storage) {
    return guard(ctx, [&](krt::Backend &b) { b.prepare_embedding_file(path, name, storage); });
}

int kernrt_cuda_kernel_launches(uint64_t *count) {
    if (!count) {
        g_last_error = "null output pointer";
        return KERNRT_E_INVALID;
    }
    *count = krt::kernel_launches();
    return KERNRT_OK;
}

int kernrt_cuda_device_count(int *count) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    if (count) *count = n;
    return KERNRT_OK;
}

int kernrt_cuda_create(int device, kernrt_cuda_ctx **out) {
    if (!out) {
        g_last_error = "null output pointer";
        return KERNRT_E_INVALID;
    }
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        g_last_error = "no CUDA device";
        return KERNRT_E_NO_DEVICE;
    }
    if (device < 0) {
        const char *env = std::getenv("KERNRT_CUDA_DEVICE");
        device = env && *env ? std::atoi(env) : 0;
    }
    if (device >= n) {
        g_last_error = "CUDA device " + std::to_string(device) + " not present (" + std::to_string(n) + " visible)";
        return KERNRT_E_NO_DEVICE;
    }
    try {
        auto *c = new kernrt_cuda_ctx{new krt::Backend(device)};
        // KERNRT_CUDA_EXACT=0: tolerance-mode tensor-core projections
        const char *exact = std::getenv("KERNRT_CUDA_EXACT");
        if (exact && exact[0] == '0' && exact[1] == '\0') c->b->set_exact(false);
        // test hook, off unless set: fail this context's n-th buffer allocation
        const char *fail_at = std::getenv("KERNRT_CUDA_FAIL_ALLOC");
        if (fail_at && *fail_at) c->b->set_fail_alloc(std::strtoull(fail_at, nullptr, 10));
        *out = c;
        return KERNRT_OK;
    } catch (const krt::Error &e) {
        g_last_error = e.msg;
        return e.code;
    }
}

int kernrt_cuda_destroy(kernrt_cuda_ctx *ctx) {
    if (!ctx) return KERNRT_OK;
    delete ctx->b;
    delete ctx;
    return KERNRT_OK;
}

const char *kernrt_cuda_name(const kernrt_cuda_ctx *) { return "cuda"; }

const char *kernrt_cuda_storage(const kernrt_cuda_ctx *ctx) {
    return ctx && ctx->b ? ctx->b->storage() : "f32";
}

int kernrt_cuda_stream(kernrt_cuda_ctx *ctx, void **stream) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!stream) krt::fail(KERNRT_E_INVALID, "null output pointer");
        *stream = (void *)b.stream();
    });
}

int kernrt_cuda_prepare_embedding(kernrt_cuda_ctx *ctx, int kind, const void *data, const float *scales,
                                  size_t vocab, size_t dim) {
    return guard(ctx, [&](krt::Backend &b) { b.prepare_embedding(kind, data, scales, vocab, dim); });
}

int kernrt_cuda_alloc(kernrt_cuda_ctx *ctx, size_t len, kernrt_buf *out) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!out) krt::fail(KERNRT_E_INVALID, "null output pointer");
        *out = b.alloc_bytes(len * sizeof(float));
    });
}

int kernrt_cuda_alloc_bytes(kernrt_cuda_ctx *ctx, size_t bytes, kernrt_buf *out) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!out) krt::fail(KERNRT_E_INVALID, "null output pointer");
        *out = b.alloc_bytes(bytes);
    });
}

int kernrt_cuda_upload(kernrt_cuda_ctx *ctx, const float *data, size_t len, kernrt_buf *out) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!out) krt::fail(KERNRT_E_INVALID, "null output pointer");
        *out = b.upload(data, len);
    });
}

int kernrt_cuda_read(kernrt_cuda_ctx *ctx, kernrt_buf src, float *out, size_t len) {
    return guard(ctx, [&](krt::Backend &b) { b.read_bytes(src, 0, out, len * sizeof(float)); });
}

int kernrt_cuda_write_bytes(kernrt_cuda_ctx *ctx, kernrt_buf dst, size_t off, const void *src, size_t bytes) {
    return guard(ctx, [&](krt::Backend &b) { b.write_bytes(dst, off, src, bytes); });
}

int kernrt_cuda_read_bytes(kernrt_cuda_ctx *ctx, kernrt_buf src, size_t off, void *dst, size_t bytes) {
    return guard(ctx, [&](krt::Backend &b) { b.read_bytes(src, off, dst, bytes); });
}

int kernrt_cuda_device_ptr(kernrt_cuda_ctx *ctx, kernrt_buf h, void **ptr) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!ptr) krt::fail(KERNRT_E_INVALID, "null output pointer");
        *ptr = b.device_ptr(h);
    });
}

int kernrt_cuda_synchronize(kernrt_cuda_ctx *ctx) {
    return guard(ctx, [&](krt::Backend &b) { b.barrier(); });
}

int kernrt_cuda_flush(kernrt_cuda_ctx *ctx) {
    return guard(ctx, [&](krt::Backend &b) { b.flush(); });
}

int kernrt_cuda_embed(kernrt_cuda_ctx *ctx, size_t token, kernrt_buf out, size_t offset) {
    return guard(ctx, [&](krt::Backend &b) { b.embed(token, out, offset); });
}

int kernrt_cuda_copy(kernrt_cuda_ctx *ctx, kernrt_buf src, size_t so, kernrt_buf dst, size_t d_o, size_t len) {
    return guard(ctx, [&](krt::Backend &b) { b.copy(src, so, dst, d_o, len); });
}

int kernrt_cuda_rms_norm(kernrt_cuda_ctx *ctx, kernrt_buf out, kernrt_buf x, kernrt_buf weight, size_t rows,
                         size_t dim, float eps) {
    return guard(ctx, [&](krt::Backend &b) { b.rms_norm(out, x, weight, rows, dim, eps); });
}

int kernrt_cuda_qk_norm(kernrt_cuda_ctx *ctx, kernrt_buf v, size_t rows, size_t width, size_t head,
                        kernrt_buf weight, float eps) {
    return guard(ctx, [&](krt::Backend &b) { b.qk_norm(v, rows, width, head, weight, eps); });
}

int kernrt_cuda_rope(kernrt_cuda_ctx *ctx, kernrt_buf q, kernrt_buf k, size_t qw, size_t kvw, size_t rows,
                     const uint64_t *positions, size_t n_positions, size_t head, float theta, int interleaved) {
    return guard(ctx, [&](krt::Backend &b) {
        b.rope(q, k, qw, kvw, rows, positions, n_positions, head, theta, interleaved);
    });
}

int kernrt_cuda_add_in_place(kernrt_cuda_ctx *ctx, kernrt_buf dst, kernrt_buf src, size_t len) {
    return guard(ctx, [&](krt::Backend &b) { b.add_in_place(dst, src, len); });
}

int kernrt_cuda_mul(kernrt_cuda_ctx *ctx, kernrt_buf out, size_t oo, kernrt_buf a, size_t ao, kernrt_buf bb,
                    size_t bo, size_t len) {
    return guard(ctx, [&](krt::Backend &b) { b.mul(out, oo, a, ao, bb, bo, len); });
}

int kernrt_cuda_conv_prefill(kernrt_cuda_ctx *ctx, kernrt_buf out, kernrt_buf x, kernrt_buf kernel, size_t rows,
                             size_t dim, size_t k) {
    return guard(ctx, [&](krt::Backend &b) { b.conv_prefill(out, x, kernel, rows, dim, k); });
}

int kernrt_cuda_conv_decode(kernrt_cuda_ctx *ctx, kernrt_buf out, kernrt_buf x, kernrt_buf kernel,
                            kernrt_buf state, size_t dim, size_t k) {
    return guard(ctx, [&](krt::Backend &b) { b.conv_decode(out, x, kernel, state, dim, k); });
}

int kernrt_cuda_silu_mul(kernrt_cuda_ctx *ctx, kernrt_buf gate, kernrt_buf up, size_t len) {
    return guard(ctx, [&](krt::Backend &b) { b.silu_mul(gate, up, len); });
}

int kernrt_cuda_quantize_q8_0(kernrt_cuda_ctx *ctx, kernrt_buf x, size_t rows, size_t dim, kernrt_buf codes,
                              kernrt_buf scales, kernrt_buf scales_f16) {
    return guard(ctx, [&](krt::Backend &b) { b.quantize_q8_0(x, rows, dim, codes, scales, scales_f16); });
}

int kernrt_cuda_rms_norm_q8_0(kernrt_cuda_ctx *ctx, kernrt_buf x, kernrt_buf weight, size_t rows, size_t dim,
                              float eps, kernrt_buf codes, kernrt_buf scales, kernrt_buf scales_f16) {
    return guard(ctx, [&](krt::Backend &b) { b.rms_norm_q8_0(x, weight, rows, dim, eps, codes, scales, scales_f16); });
}

int kernrt_cuda_rope_prepare(kernrt_cuda_ctx *ctx, float theta, size_t head, size_t max_pos) {
    return guard(ctx, [&](krt::Backend &b) { b.rope_prepare(theta, head, max_pos); });
}

int kernrt_cuda_layer_chain(kernrt_cuda_ctx *ctx, const kernrt_chain_args *args) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!args) krt::fail(KERNRT_E_INVALID, "null chain arguments");
        b.layer_chain(*args);
    });
}

int kernrt_cuda_layer_chain_host(kernrt_cuda_ctx *ctx, const kernrt_chain_host_args *args) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!args) krt::fail(KERNRT_E_INVALID, "null chain arguments");
        b.layer_chain_host(*args);
    });
}

int kernrt_cuda_stage_timing(kernrt_cuda_ctx *ctx, int enable) {
    return guard(ctx, [&](krt::Backend &b) { b.stage_timing(enable != 0); });
}

int kernrt_cuda_stage_times(kernrt_cuda_ctx *ctx, double *ms, uint64_t *launches) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!ms || !launches) krt::fail(KERNRT_E_INVALID, "null output pointer");
        b.stage_times(ms, launches);
    });
}

int kernrt_cuda_lfm2_conv_block(kernrt_cuda_ctx *ctx, kernrt_buf bcx, kernrt_buf kernel, kernrt_buf ring,
                                kernrt_buf cy, size_t rows, size_t dim, size_t k) {
    return guard(ctx, [&](krt::Backend &b) {
        if (!ring && k > 1) krt::fail(KERNRT_E_INVALID, "conv block needs its ring");
        b.lfm2_conv_block(bcx, kernel, ring, cy, rows, dim, k);
    });
}

int kernrt_cuda_lfm2_conv_block_halo(kernrt_cuda_ctx *ctx, kernrt_buf bcx, kernrt_buf kernel, kernrt_buf ring,
                                     kernrt_buf cy, size_t rows, size_t dim, size_t k, size_t halo) {
    return guard(ctx, [&](krt::Backend &b) { b.lfm2_conv_block(bcx, kernel, ring, cy, rows, dim, k, halo); });
}

int kernrt_cuda_prepare_matrix(kernrt_cuda_ctx *ctx, int kind, const void *data, const float *scales, size_t out_dim,
                               size_t in_dim, kernrt_mat *out) {
    if (!out) {
        g_last_error = "null output pointer";
        return KERNRT_E_INVALID;
    }
    return guard(ctx, [&](krt::Backend &b) { *out = b.prepare_matrix(kind, data, scales, out_dim, in_dim); });
}

int kernrt_cuda_project(kernrt_cuda_ctx *ctx, kernrt_mat w, kernrt_buf x, kernrt_buf y, size_t rows) {
    return guard(ctx, [&](krt::Backend &b) { b.project(w, x, y, rows); });
}

int kernrt_cuda_project_qkv(kernrt_cuda_ctx *ctx, kernrt_mat wq, kernrt_mat wk, kernrt_mat wv, kernrt_buf x,
                            kernrt_buf q, kernrt_buf k, kernrt_buf v, size_t rows) {
    return guard(ctx, [&](krt::Backend &b) {
        const uint64_t ws[3] = {wq, wk, wv};
        const kernrt_buf ys[3] = {q, k, v};
        b.project_set(3, ws, x, ys, rows);
    });
}

int kernrt_cuda_project_gate_up(kernrt_cuda_ctx *ctx, kernrt_mat wg, kernrt_mat wu, kernrt_buf x, kernrt_buf gate,
                                kernrt_buf up, size_t rows) {
    return guard(ctx, [&](krt::Backend &b) {
        const uint64_t ws[2] = {wg, wu};
        const kernrt_buf ys[2] = {gate, up};
        b.project_set(2, ws, x, ys, rows);
    });
}

int kernrt_cuda_logits(kernrt_cuda_ctx *ctx, kernrt_mat w, kernrt_buf x, kernrt_buf y) {
    return guard(ctx, [&](krt::Backend &b) { b.logits(w, x, y); });
}

int kernrt_cuda_kv_prepare(kernrt_cuda_ctx *ctx, size_t n_layers, size_t kv_dim, size_t seq_len) {
    return guard(ctx, [&](krt::Backend &b) { b.kv_prepare(n_layers, kv_dim, seq_len); });
}

int kernrt_cuda_kv_write(kernrt_cuda_ctx *ctx, size_t layer, const uint64_t *slots, size_t n_slots, kernrt_buf k,
                         kernrt_buf v, size_t rows) {
    return guard(ctx, [&](krt::Backend &b) { b.kv_write(layer, slots, n_slots, k, v, rows); });
}

int kernrt_cuda_attention(kernrt_cuda_ctx *ctx, kernrt_buf q, kernrt_buf out, kernrt_buf att, size_t layer,
                          const kernrt_window *windows, size_t n_windows, size_t n_heads, size_t kv_mul,
                          size_t head_size, size_t kv_dim, size_t seq_len) {
    return guard(ctx, [&](krt::Backend &b) {
        b.attention(q, out, att, layer, windows, n_windows, n_heads, kv_mul, head_size, kv_dim, seq_len);
    });
}

}  // extern "C"
