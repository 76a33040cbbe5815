// Shared internals of libtl_cuda: status/error plumbing, the normalised GEMM
// problem the kernels consume, and launch bookkeeping.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <string>

#include "../../include/tlc.h"

namespace tlc {

// ---- errors -----------------------------------------------------------------

// Records `msg` as this thread's last error and returns `status`.
int set_error(int status, const std::string& msg);
void clear_error();

#define TLC_CUDA_TRY(expr)                                                              \
    do {                                                                                \
        cudaError_t e_ = (expr);                                                        \
        if (e_ != cudaSuccess) {                                                        \
            return ::tlc::set_error(e_ == cudaErrorMemoryAllocation ? TLC_ERR_OUT_OF_MEMORY \
                                                                    : TLC_ERR_CUDA,     \
                                    std::string(#expr) + ": " + cudaGetErrorString(e_)); \
        }                                                                               \
    } while (0)

#define TLC_TRY(expr)            \
    do {                         \
        int s_ = (expr);         \
        if (s_ != TLC_OK) return s_; \
    } while (0)

// ---- per-device set-up ---------------------------------------------------------------
//
// Set-up that belongs to a device's CUDA context (kernel attributes, symbol
// addresses, streams) runs once per device and context: again when the
// context is re-created (after cudaDeviceReset), never twice at once from two
// host threads.

// The calling thread's current CUDA context (NULL if none is bound yet).
void* current_context();

struct DeviceOnce {
    std::mutex mu;
    void* ctx[64] = {};
};

// Runs setup(device) unless it already succeeded for the current device's
// current context; *dev_out (if given) receives the device index.
template <class F>
int device_once(DeviceOnce& o, F&& setup, int* dev_out = nullptr) {
    int dev = 0;
    TLC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(TLC_ERR_UNSUPPORTED, "device index above 63");
    if (dev_out) *dev_out = dev;
    std::lock_guard<std::mutex> lk(o.mu);
    void* c = current_context();
    if (c && o.ctx[dev] == c) return TLC_OK;
    const int st = setup(dev);
    if (st == TLC_OK) o.ctx[dev] = current_context();
    return st;
}

// Raises a kernel's dynamic shared-memory limit on the current device.
template <class K>
int smem_limit_once(DeviceOnce& o, K kernel, int bytes) {
    return device_once(o, [&](int) -> int {
        TLC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        return TLC_OK;
    });
}

// ---- launch bookkeeping ----------------------------------------------------------

extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Checks the launch that was just made (configuration errors surface here).
int check_launch(const char* what);

// ---- the GEMM problem --------------------------------------------------------------

constexpr int kMaxBatchDims = 3;

// Normalised batched GEMM: C_b[m,n] = sum_k A_b[m,k] B_b[k,n]; all strides in
// elements.  Either a_cs == 1 (A row-major, "K-major") or a_rs == 1 (A
// column-major, "M-major"); likewise b_cs == 1 (B row-major, "N-major") or
// b_rs == 1 (B column-major, "K-major").  C is row-major (c_cs == 1).
struct Gemm {
    int64_t M, N, K;
    const float* A;
    int64_t a_rs, a_cs;
    const float* B;
    int64_t b_rs, b_cs;
    float* C;
    int64_t c_rs;
    int nb;                           // number of batch dims (0..3)
    int64_t bsz[kMaxBatchDims];       // batch sizes, outermost first
    int64_t abs_[kMaxBatchDims], bbs[kMaxBatchDims], cbs[kMaxBatchDims];
    // Epilogue on each output element, in this order (each one IEEE fp32
    // operation, as the reference's separate tl::scale / tl::add would do):
    // c = c * scale if apply_scale; c = c + bias[n] if bias.
    const float* bias = nullptr;  // [N], contiguous
    float scale = 1.0f;
    int apply_scale = 0;
    int64_t batch() const {
        int64_t n = 1;
        for (int i = 0; i < nb; ++i) n *= bsz[i];
        return n;
    }
};

// Flat batch index -> the three operand offsets (get_broadcast_index,
// src/ops.cpp:32-52, with broadcast dims carrying stride 0).
struct BatchOffsets {
    int nb;
    int64_t bsz[kMaxBatchDims];
    int64_t as[kMaxBatchDims], bs[kMaxBatchDims], cs[kMaxBatchDims];
    __host__ __device__ __forceinline__ void get(int64_t b, int64_t& oa, int64_t& ob,
                                                 int64_t& oc) const {
        oa = ob = oc = 0;
#pragma unroll
        for (int i = kMaxBatchDims - 1; i >= 0; --i) {
            if (i < nb) {
                int64_t idx = b % bsz[i];
                b /= bsz[i];
                oa += idx * as[i];
                ob += idx * bs[i];
                oc += idx * cs[i];
            }
        }
    }
};

inline BatchOffsets batch_offsets(const Gemm& g) {
    BatchOffsets o{};
    o.nb = g.nb;
    for (int i = 0; i < kMaxBatchDims; ++i) {
        o.bsz[i] = i < g.nb ? g.bsz[i] : 1;
        o.as[i] = i < g.nb ? g.abs_[i] : 0;
        o.bs[i] = i < g.nb ? g.bbs[i] : 0;
        o.cs[i] = i < g.nb ? g.cbs[i] : 0;
    }
    return o;
}

// Kernels (each returns a tlc_status).
int gemm_exact(const Gemm& g, cudaStream_t s);
int gemm_tc(const Gemm& g, int mode, cudaStream_t s);
// An implicit-GEMM convolution (stride 1) on the tensor cores: the GEMM
// out[n, g] (M output channels x N output pixels) = A[g] (M x K) . B[n, g],
// K = kH * kW * (32 * cblocks) ordered (kh, kw, channel), where B's column
// j = oh * W_out + ow, row (kh, kw, c) is x[n, oh - pad_h + kh, ow - pad_w + kw,
// g * c_group + c] of the NHWC tensor x (zero outside it).  Batch dim 0 of the
// Gemm is the image, dim 1 the group; its B fields are ignored.  Tiles are
// `rows` output rows of W_out pixels (W_out % 8 == 0, rows * W_out <= 256 and
// a multiple of 16).  X3 needs x_lo: the lo plane of x for the 3xTF32 split.
struct ConvTma {
    const float* x;
    const float* x_lo;
    int N, H, W, C;
    int W_out, rows;
    int kH, kW, pad_h, pad_w;
    int cblocks, c_group;
    const float* row_bias;  // NULL, or one per output row: bias[group * row_bias_group + row]
    int64_t row_bias_group;
};
int gemm_tc_conv(const Gemm& g, const ConvTma& c, int mode, cudaStream_t s);

// The weight gradient of a stride-1 convolution as an implicit GEMM with a
// split K (TF32 / 3xTF32):
//   part[s][g][o][tap * c_pad + c] = sum over the output rows of split s, in
//   32-pixel blocks, of dO[n, g*C_out_g + o, oh, ow] * x[n, oh - pad_h + kh,
//   ow - pad_w + kw, g*C_in_g + c]   (tap = kh * kW + kw, c < c_pad)
// with dO read as NCHW and x as its NHWC copy; a TMA box brings 32 pixels of
// one dO row (the K-major A) and, per 32 channels of one tap, the matching 32
// shifted input pixels (the MN-major B), zero-filled outside the image.
// k-steps past the row's end are not issued, so no product of a pixel outside
// the output enters a sum.  Split s covers output rows (n, oh) s * rows ..
// s * rows + rows - 1 (flattened n * H_out + oh; rows past the last read as
// zeros).
struct ConvDw {
    const float* go;     // dO, dense NCHW [N, C_out, H_out, W_out]
    const float* x;      // the input as dense NHWC [N, H, W, C]
    const float* x_lo;   // 3xTF32: the lo plane of x (NHWC), else NULL
    int N, C, H, W;
    int C_out, H_out, W_out;
    int kH, kW, pad_h, pad_w;
    int groups, C_in_g, C_out_g;
};
// Splits (and rows per split) for this problem on this device; the partial
// buffer holds splits * groups * C_out_g * kH * kW * round32(C_in_g) floats.
int conv_dw_splits(const ConvDw& c, int mode, int* splits, int* rows);
int gemm_tc_conv_dw(const ConvDw& c, int splits, int rows, float* part, int mode, cudaStream_t s);

// out[o,n] = sum over d ascending of in[o,d,n], from init[o,n] (NULL: from 0.0f).
int launch_sum_dim(const float* in, float* out, int64_t outer, int64_t D, int64_t inner,
                   cudaStream_t s, const float* init = nullptr);
int launch_add(const float* a, const float* b, float* out, int64_t n, cudaStream_t s);
int launch_zero_plus(const float* in, float* out, int64_t n, cudaStream_t s);
int launch_strided_copy(const float* src, int nd, const int64_t* sizes, const int64_t* strides,
                        float* dst, cudaStream_t s);
int launch_fill_zero(float* p, int64_t n, cudaStream_t s);
int launch_gather_colblocks(const float* g, float* out, int64_t M, int64_t N, int world,
                            const int64_t* begin, cudaStream_t s);

// Glue kernels (glue.cu).  kind 0: out = a + b, kind 1: out = a * s, over a
// contiguous output of shape sz[0..nd) with operand strides sa / sb (0 on
// broadcast dims).
int launch_elementwise(const float* a, const float* b, float s, float* out, int64_t n, int nd,
                       const int64_t* sz, const int64_t* sa, const int64_t* sb, int kind,
                       cudaStream_t st);
int launch_epilogue(float* C, int64_t rows, int64_t cols, float s, bool apply_scale,
                    const float* bias, cudaStream_t st);
int launch_softmax(const float* x, float* y, int64_t rows, int64_t D, cudaStream_t st);
// Attention forward on the tensor cores (flash_tc.cu): q, k, v, o [heads, S, d]
// contiguous, lse [heads, S] or NULL.
bool flash_tc_supported(int d, const float* q, const float* k, const float* v);
int flash_forward_tc(const float* q, const float* k, const float* v, float* o, float* lse,
                     int64_t heads, int S, int d, float scale, cudaStream_t s);
// Attention backward on the tensor cores (flash_bwd_tc.cu); ptrs: every operand.
bool flash_bwd_tc_supported(int d, const float* const* ptrs, int n);
int flash_backward_tc(const float* dout, const float* q, const float* k, const float* v,
                      const float* o, const float* lse, float* dq, float* dk, float* dv,
                      int64_t heads, int S, int d, float scale, cudaStream_t s);
int launch_softmax_backward(const float* g, const float* y, float* dx, int64_t rows, int64_t D,
                            cudaStream_t st);

// Copy a strided view into a destination with its own strides (same shape).
int launch_strided_copy_to(const float* src, int nd, const int64_t* sizes, const int64_t* sstr,
                           float* dst, const int64_t* dstr, cudaStream_t s);
// Whether the tensor cores read fp32 operands truncated to TF32 on the current
// device (checked once per device by one small product; false while unknown
// and `s` is being captured).
bool tf32_reads_truncated(cudaStream_t s);
// Device error word written by bounded waits inside kernels (0 = none).
int tc_error_word(int** p);
// Launches a kernel whose bounded wait must time out (failure-detection test).
int bounded_wait_selftest(uint64_t timeout_ns, cudaStream_t s);

// Stream-ordered scratch memory from the device's memory pool.
int scratch_alloc(void** p, size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

// A second stream of the calling host thread on the current device (made on
// first use), for work that overlaps the caller's stream.
inline cudaStream_t side_stream() {
    thread_local cudaStream_t streams[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!streams[dev] && cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        streams[dev] = nullptr;
    }
    return streams[dev];
}

// Work forked from `main` onto a side stream; the destructor makes `main`
// wait for it (so anything enqueued on `main` afterwards, frees of the
// buffers it reads included, comes after it), on every return path.
struct Fork {
    cudaStream_t main, side = nullptr;
    cudaEvent_t join = nullptr;
    explicit Fork(cudaStream_t m) : main(m) {}
    // the side stream, ordered after everything enqueued on `main` so far;
    // nullptr when none can be had (the caller then uses `main`)
    cudaStream_t begin() {
        cudaStream_t s = side_stream();
        cudaEvent_t f = nullptr;
        if (!s || cudaEventCreateWithFlags(&f, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        if (cudaEventCreateWithFlags(&join, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventRecord(f, main) != cudaSuccess || cudaStreamWaitEvent(s, f, 0) != cudaSuccess) {
            cudaGetLastError();
            cudaEventDestroy(f);
            if (join) cudaEventDestroy(join);
            join = nullptr;
            return nullptr;
        }
        cudaEventDestroy(f);
        side = s;
        return s;
    }
    ~Fork() {
        if (!side) return;
        cudaEventRecord(join, side);
        cudaStreamWaitEvent(main, join, 0);
        cudaEventDestroy(join);
    }
};

}  // namespace tlc
