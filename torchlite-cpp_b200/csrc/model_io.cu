// TLMD model files (src/model_io.cpp:7-94 of torchlite-cpp) read straight
// into, and written straight from, device memory.
//
// Format (little-endian, as the reference writes it on x86):
//   "TLMD" | int32 version = 1 | int64 count | per tensor: int64 ndim,
//   int64 shape[ndim], float data[numel] (row-major).
//
// Loading checks the header and each tensor's ndim and shape against the
// caller's tensors, in order, with the reference's error texts
// (TLC_ERR_IO, the reference's std::runtime_error).  Tensor data streams
// through two page-locked staging buffers: while one chunk's host-to-device
// copy runs on the stream, the next chunk is read from the file into the
// other buffer.  Saving is the mirror image (device-to-host copies into the
// staging buffers, written as they land).
//
// Deliberate differences from the reference: a file that ends early is an
// error ("load_model: file truncated"; the reference leaves the rest of the
// tensor unread without noticing), and a failed write is an error.
#include "common.cuh"

#include <cstdio>
#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace tlc {
namespace {

constexpr char kMagic[4] = {'T', 'L', 'M', 'D'};
constexpr int32_t kVersion = 1;
constexpr size_t kChunk = size_t(16) << 20;  // bytes per staging buffer

struct File {
    std::FILE* f = nullptr;
    ~File() {
        if (f) std::fclose(f);
    }
};

bool read_exact(std::FILE* f, void* p, size_t n) { return std::fread(p, 1, n, f) == n; }

// Two page-locked staging buffers and the events that say when each is free.
struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaStream_t s;
    explicit Staging(cudaStream_t st) : s(st) {}
    int init() {
        for (int i = 0; i < 2; ++i) {
            TLC_CUDA_TRY(cudaMallocHost(&buf[i], kChunk));
            TLC_CUDA_TRY(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        return TLC_OK;
    }
    ~Staging() {
        cudaStreamSynchronize(s);  // no copy may still use a buffer being freed
        for (int i = 0; i < 2; ++i) {
            if (done[i]) cudaEventDestroy(done[i]);
            if (buf[i]) cudaFreeHost(buf[i]);
        }
    }
};

int64_t numel_of(const tlc_tensor& t) {
    int64_t n = 1;
    for (int i = 0; i < t.ndim; ++i) n *= t.sizes[i];
    return n;
}

bool is_contiguous(const tlc_tensor& t) {
    if (numel_of(t) == 0) return true;  // no data: strides of empty tensors vary
    int64_t e = 1;
    for (int i = t.ndim - 1; i >= 0; --i) {
        if (t.sizes[i] != 1 && t.strides[i] != e) return false;
        e *= t.sizes[i];
    }
    return true;
}

int check_tensors(int32_t count, const tlc_tensor* ts, const char* what) {
    if (count < 0) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(what) + ": negative count");
    if (count > 0 && !ts) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(what) + ": tensors is NULL");
    for (int32_t i = 0; i < count; ++i) {
        if (ts[i].ndim < 0 || ts[i].ndim > TLC_MAX_DIMS)
            return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(what) + ": bad ndim");
        for (int d = 0; d < ts[i].ndim; ++d)
            if (ts[i].sizes[d] < 0) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(what) + ": negative size");
        if (numel_of(ts[i]) > 0 && !ts[i].data)
            return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(what) + ": NULL data");
    }
    return TLC_OK;
}

int load(const char* path, int32_t count, const tlc_tensor* dst, cudaStream_t s) {
    TLC_TRY(check_tensors(count, dst, "load_model"));
    for (int32_t i = 0; i < count; ++i)
        if (!is_contiguous(dst[i]))
            return set_error(TLC_ERR_INVALID_ARGUMENT, "load_model: destination tensors must be contiguous");
    const std::string p = path ? path : "";
    File file;
    file.f = std::fopen(p.c_str(), "rb");
    if (!file.f) return set_error(TLC_ERR_IO, "load_model: cannot open file: " + p);
    char magic[4] = {};
    if (!read_exact(file.f, magic, 4) || std::memcmp(magic, kMagic, 4) != 0)
        return set_error(TLC_ERR_IO, "load_model: no TLMD magic header in " + p);
    int32_t version = 0;
    if (!read_exact(file.f, &version, sizeof(version)) || version != kVersion)
        return set_error(TLC_ERR_IO, "load_model: unsupported version");
    int64_t n = 0;
    if (!read_exact(file.f, &n, sizeof(n)) || n != count)
        return set_error(TLC_ERR_IO, "load_model: tensor count mismatch");
    std::unique_ptr<Staging> st;  // set up at the first tensor with data
    int which = 0;
    for (int32_t i = 0; i < count; ++i) {
        int64_t ndim = -1;
        if (!read_exact(file.f, &ndim, sizeof(ndim)) || ndim != dst[i].ndim)
            return set_error(TLC_ERR_IO, "load_model: ndim mismatch");
        std::vector<int64_t> shape((size_t)ndim);
        if (ndim && !read_exact(file.f, shape.data(), sizeof(int64_t) * (size_t)ndim))
            return set_error(TLC_ERR_IO, "load_model: file truncated");
        for (int64_t d = 0; d < ndim; ++d)
            if (shape[(size_t)d] != dst[i].sizes[d]) return set_error(TLC_ERR_IO, "load_model: shape mismatch");
        size_t left = sizeof(float) * (size_t)numel_of(dst[i]);
        char* out = reinterpret_cast<char*>(dst[i].data);
        if (left && !st) {
            st.reset(new Staging(s));
            TLC_TRY(st->init());
        }
        while (left) {
            const size_t c = std::min(left, kChunk);
            TLC_CUDA_TRY(cudaEventSynchronize(st->done[which]));  // its previous copy finished
            if (!read_exact(file.f, st->buf[which], c)) return set_error(TLC_ERR_IO, "load_model: file truncated");
            TLC_CUDA_TRY(cudaMemcpyAsync(out, st->buf[which], c, cudaMemcpyHostToDevice, s));
            TLC_CUDA_TRY(cudaEventRecord(st->done[which], s));
            out += c;
            left -= c;
            which ^= 1;
        }
    }
    if (st) TLC_CUDA_TRY(cudaStreamSynchronize(s));
    return TLC_OK;
}

int save(const char* path, int32_t count, const tlc_tensor* src, cudaStream_t s) {
    TLC_TRY(check_tensors(count, src, "save_model"));
    const std::string p = path ? path : "";
    File file;
    file.f = std::fopen(p.c_str(), "wb");
    if (!file.f) return set_error(TLC_ERR_IO, "save_model: cannot open file: " + p);
    auto put = [&](const void* q, size_t nb) { return std::fwrite(q, 1, nb, file.f) == nb; };
    const int64_t n = count;
    if (!put(kMagic, 4) || !put(&kVersion, sizeof(kVersion)) || !put(&n, sizeof(n)))
        return set_error(TLC_ERR_IO, "save_model: write failed");
    std::unique_ptr<Staging> st;
    for (int32_t i = 0; i < count; ++i) {
        const int64_t ndim = src[i].ndim;
        if (!put(&ndim, sizeof(ndim)) || (ndim && !put(src[i].sizes, sizeof(int64_t) * (size_t)ndim)))
            return set_error(TLC_ERR_IO, "save_model: write failed");
        const int64_t numel = numel_of(src[i]);
        if (!numel) continue;
        if (!st) {
            st.reset(new Staging(s));
            TLC_TRY(st->init());
        }
        // Tensor::contiguous first, as the reference does (src/model_io.cpp:38)
        const float* base = src[i].data;
        void* dense = nullptr;
        if (!is_contiguous(src[i])) {
            TLC_TRY(scratch_alloc(&dense, sizeof(float) * (size_t)numel, s));
            const int rc = launch_strided_copy(src[i].data, src[i].ndim, src[i].sizes, src[i].strides,
                                               static_cast<float*>(dense), s);
            if (rc != TLC_OK) {
                scratch_free(dense, s);
                return rc;
            }
            base = static_cast<const float*>(dense);
        }
        // chunk k + 1's copy is queued before chunk k is written out
        const char* in = reinterpret_cast<const char*>(base);
        const size_t total = sizeof(float) * (size_t)numel;
        size_t len[2] = {0, 0}, pos = 0;
        int cur = 0, rc = TLC_OK;
        auto queue = [&](int b) {
            len[b] = std::min(total - pos, kChunk);
            if (cudaMemcpyAsync(st->buf[b], in + pos, len[b], cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                cudaEventRecord(st->done[b], s) != cudaSuccess)
                rc = set_error(TLC_ERR_CUDA, "save_model: device-to-host copy failed");
            pos += len[b];
        };
        queue(cur);
        while (rc == TLC_OK) {
            const bool more = pos < total;
            if (more) queue(cur ^ 1);  // its buffer's previous chunk is already written
            if (rc != TLC_OK) break;
            if (cudaEventSynchronize(st->done[cur]) != cudaSuccess) {
                rc = set_error(TLC_ERR_CUDA, "save_model: device-to-host copy failed");
                break;
            }
            if (!put(st->buf[cur], len[cur])) {
                rc = set_error(TLC_ERR_IO, "save_model: write failed");
                break;
            }
            if (!more) break;
            cur ^= 1;
        }
        if (dense) scratch_free(dense, s);
        TLC_TRY(rc);
    }
    if (std::fflush(file.f) != 0) return set_error(TLC_ERR_IO, "save_model: write failed");
    return TLC_OK;
}

}  // namespace
}  // namespace tlc

extern "C" int tlc_load_tlmd(const char* path, int32_t count, const tlc_tensor* dst, void* stream) {
    tlc::clear_error();
    return tlc::load(path, count, dst, static_cast<cudaStream_t>(stream));
}

extern "C" int tlc_save_tlmd(const char* path, int32_t count, const tlc_tensor* src, void* stream) {
    tlc::clear_error();
    return tlc::save(path, count, src, static_cast<cudaStream_t>(stream));
}
