/*
 * libtl_cuda: the C ABI under torchlite-cpp's matmul path on B200 (sm_100a).
 *
 * The reference library has no FFI: its operator API for this path is the C++
 * free function  tl::Tensor tl::matmul(const Tensor&, const Tensor&)
 * (include/tl/ops.h:24-26, src/ops.cpp:605-699) and the autograd node
 * MatmulBackward (include/tl/autograd.h:177-182, src/autograd.cpp:341-384).
 * The entry points below are what that C++ code binds to when it runs on the
 * GPU: plain pointers, sizes and strides, status codes instead of exceptions
 * (the C++ layer maps TLC_ERR_INVALID_ARGUMENT back to std::invalid_argument
 * with the reference's message, available from tlc_last_error()).
 *
 * Pointers passed to the compute entry points are device pointers on the
 * current CUDA device unless the function name ends in _host.  Streams are
 * cudaStream_t passed as void* (NULL = the legacy default stream).
 *
 * Precision modes (argument `mode`):
 *   TLC_MODE_EXACT   fp32 FFMA; every output element is the ascending-k chain
 *                    c = fmaf(a[m,k], b[k,n], c) from c = 0, so results are
 *                    bit-identical to the reference's gemm_blocked
 *                    (src/ops.cpp:242-268), which compiles to that chain.
 *   TLC_MODE_TF32    tcgen05 tensor cores, TF32 inputs, fp32 accumulation.
 *   TLC_MODE_3XTF32  tcgen05, each operand split into TF32 hi + lo parts,
 *                    three products accumulated in fp32 (near-fp32 accuracy).
 *   TLC_MODE_DEFAULT the process default: environment variable TL_GEMM_MODE
 *                    (exact | tf32 | 3xtf32), read once; exact if unset.
 */
#ifndef TLC_H
#define TLC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TLC_MAX_DIMS 8

typedef enum tlc_status {
    TLC_OK = 0,
    TLC_ERR_INVALID_ARGUMENT = 1, /* the reference throws std::invalid_argument here */
    TLC_ERR_UNSUPPORTED = 2,
    TLC_ERR_CUDA = 3,
    TLC_ERR_OUT_OF_MEMORY = 4,
    TLC_ERR_TIMEOUT = 5, /* a bounded wait inside a kernel gave up; see tlc_last_error() */
    TLC_ERR_IO = 6       /* file error (the reference throws std::runtime_error here) */
} tlc_status;

typedef enum tlc_mode {
    TLC_MODE_DEFAULT = -1,
    TLC_MODE_EXACT = 0,
    TLC_MODE_TF32 = 1,
    TLC_MODE_3XTF32 = 2
} tlc_mode;

/* A strided fp32 tensor view: the layout of tl::Tensor (include/tl/tensor.h:13-67:
 * sizes_, strides_ in elements, data_ + offset_).  `data` points at element
 * [0,...,0], i.e. storage + storage_offset. */
typedef struct tlc_tensor {
    float* data;
    int32_t ndim;
    int64_t sizes[TLC_MAX_DIMS];
    int64_t strides[TLC_MAX_DIMS];
} tlc_tensor;

/* One batched, strided GEMM: for every batch index b (up to 3 batch dims,
 * row-major order), C_b[m,n] = sum_k A_b[m,k] * B_b[k,n] with
 *   A_b[m,k] = A[off_a(b) + m*a_rs + k*a_cs]     (a_cs == 1: row-major A;
 *   B_b[k,n] = B[off_b(b) + k*b_rs + n*b_cs]      a_rs == 1: transposed view)
 *   C_b[m,n] = C[off_c(b) + m*c_rs + n]
 *   off_x(b) = sum_j idx_j(b) * x_bstride[j]     (0 = broadcast over that dim).
 * Replaces the batch loop + get_broadcast_index + gemm_mt/gemm_tiled dispatch
 * of src/ops.cpp:655-674 and the kernels it reaches (src/ops.cpp:242-602). */
typedef struct tlc_gemm_desc {
    int64_t M, N, K;
    const float* A;
    int64_t a_rs, a_cs;
    const float* B;
    int64_t b_rs, b_cs;
    float* C;
    int64_t c_rs;
    int32_t batch_ndim;
    int64_t batch_sizes[3];
    int64_t a_bstride[3], b_bstride[3], c_bstride[3];
} tlc_gemm_desc;

/* ---- library ---------------------------------------------------------- */

int tlc_version(void);
const char* tlc_status_string(int status);
/* Message of the last failing call on this host thread ("" if none).  For
 * TLC_ERR_INVALID_ARGUMENT it is the reference's exception text. */
const char* tlc_last_error(void);
/* Number of CUDA kernels this library has launched in this process. */
uint64_t tlc_launch_count(void);
/* Parse a mode name ("exact", "tf32", "3xtf32"); -1 if unknown. */
int tlc_mode_from_string(const char* name);
/* The mode TLC_MODE_DEFAULT resolves to. */
int tlc_default_mode(void);

/* ---- device-buffer backing for Tensor storage ----------------------------
 * Storage of tl::Tensor is std::shared_ptr<std::vector<float>>
 * (include/tl/tensor.h:53); these are the device and pinned-host allocation
 * and copy primitives its CUDA backing uses. */
int tlc_device_count(int* count);
int tlc_set_device(int device);
int tlc_get_device(int* device);
int tlc_malloc(void** ptr, size_t bytes);
int tlc_free(void* ptr);
int tlc_malloc_host(void** ptr, size_t bytes); /* page-locked */
int tlc_free_host(void* ptr);
/* kind: 0 host->device, 1 device->host, 2 device->device (async on stream). */
int tlc_memcpy(void* dst, const void* src, size_t bytes, int kind, void* stream);
int tlc_memset_zero(void* dst, size_t bytes, void* stream);
/* Waits for `stream`, then reports (and clears) a timeout that a kernel of
 * this library recorded on the current device: TLC_ERR_TIMEOUT. */
int tlc_stream_synchronize(void* stream);
/* Synchronises the current device and reports (and clears) a recorded
 * in-kernel timeout, like tlc_stream_synchronize. */
int tlc_check_device_errors(void);
/* Failure-detection self test: runs the tensor-core GEMM's bounded wait on an
 * mbarrier that nothing arrives on, with the given limit.  A working bound
 * returns TLC_ERR_TIMEOUT (and leaves the context usable); TLC_OK would mean
 * the wait ended without its barrier completing. */
int tlc_selftest_bounded_wait(uint64_t timeout_ns);

/* ---- tl::matmul ---------------------------------------------------------- */

/* Shape rules of tl::matmul (src/ops.cpp:605-652): 1-D operands are squeezed
 * ([K] -> [1,K] for a, [K] -> [K,1] for b), batch dims broadcast NumPy-style,
 * and the squeezed dims are dropped from the result (src/ops.cpp:676-687).
 * Writes the result rank and sizes.  Errors (TLC_ERR_INVALID_ARGUMENT):
 *   "matmul: requires at least 1D tensors"      (src/ops.cpp:622)
 *   "Incompatible dimensions for matmul"         (src/ops.cpp:635)
 *   "Incompatible dimensions for broadcasting"   (src/ops.cpp:66)
 * Host-only; touches no GPU. */
int tlc_matmul_shape(const tlc_tensor* a, const tlc_tensor* b, int32_t* out_ndim,
                     int64_t* out_sizes);

/* out = tl::matmul(a, b) on the current device (src/ops.cpp:605-699).
 * a and b are any strided views (transposed views are read in place);
 * out must be contiguous with the shape tlc_matmul_shape reports.  K == 0
 * gives zeros, as the reference's zero-initialised output does. */
int tlc_matmul(const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, int mode, void* stream);

/* MatmulBackward::backward (src/autograd.cpp:341-384): given dC = grad (the
 * shape of the matmul result), computes
 *   dA = sum_to(dC . B^T, shape(a)),  dB = sum_to(A^T . dC, shape(b))
 * with sum_to's order (src/autograd.cpp:24-36), then accumulate_grad
 * (src/autograd.cpp:16-22): if `accumulate` is non-zero da/db already hold a
 * gradient and receive da + dA (resp. db + dB); otherwise they are
 * overwritten with 0 + dA.  da / db must be contiguous with the shapes of
 * a / b; pass data == NULL to skip one of them. */
int tlc_matmul_backward(const tlc_tensor* grad, const tlc_tensor* a, const tlc_tensor* b,
                        tlc_tensor* da, tlc_tensor* db, int accumulate, int mode, void* stream);

/* Host-buffer forms for callers whose tensors live in host memory (the
 * unmodified reference Tensor): copies operands to the current device,
 * computes, and copies the result back, all inside the call, which returns
 * once the result is in `out`.  Same shapes and errors as above; views are
 * strided host views (page-locked memory copies fastest).  The work runs on
 * `stream` (NULL = a stream the library keeps per device). */
int tlc_matmul_host(const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, int mode,
                    void* stream);
int tlc_matmul_backward_host(const tlc_tensor* grad, const tlc_tensor* a, const tlc_tensor* b,
                             tlc_tensor* da, tlc_tensor* db, int accumulate, int mode,
                             void* stream);

/* The GEMM core (see tlc_gemm_desc). */
int tlc_gemm(const tlc_gemm_desc* desc, int mode, void* stream);

/* 3xTF32 GEMM that allocates no device memory.  No counterpart in the
 * reference (its CPU path has no device memory to allocate); it exists for
 * callers that may not let this library allocate: an application whose device
 * memory all belongs to its own arena allocator, or a latency-critical loop
 * where an allocation that can block or fail is not allowed.  Same arguments
 * and result as tlc_gemm(desc, TLC_MODE_3XTF32, stream), except:
 *  - the hi / lo split planes live in one 64 MiB device array inside the
 *    library, held on every GPU that loads it until the process exits; A and
 *    B together may span at most 8 Mi floats (minus 64-float padding per
 *    plane); larger problems return TLC_ERR_INVALID_ARGUMENT;
 *  - A and B must be 16-byte aligned with strides that are multiples of 4
 *    floats (else TLC_ERR_UNSUPPORTED);
 *  - the array takes its 64 MiB of device memory when the library's GEMM
 *    code is loaded on a device; with CUDA's lazy module loading (the
 *    default since CUDA 12.2) that is the first GEMM call of any kind on the
 *    device, this entry point included.  A caller whose arena claims the
 *    device's free memory makes one call (any small product) before it
 *    sizes the arena;
 *  - the first call on a device (and the first after its context is re-
 *    created) looks up that array's device address (set-up work), so make it
 *    before any stream capture; the set-up is safe to race from several host
 *    threads;
 *  - all calls share the array: calls that overlap on the GPU race, so
 *    serialise them (each call rewrites every element it reads, so nothing
 *    needs clearing between calls). */
int tlc_gemm_3xtf32_noalloc(const tlc_gemm_desc* desc, void* stream);

/* ---- building blocks of the backward pass --------------------------------- */

/* sum(input, dim, keepdim) of src/ops.cpp:1181-1233 for a contiguous input
 * viewed as [outer, D, inner]: out[o,n] = sum over d ascending, from 0.0f. */
int tlc_sum_dim(const float* in, float* out, int64_t outer, int64_t D, int64_t inner, void* stream);
/* The same sums continued from a running value: out[o,n] = init[o,n] +
 * in[o,0,n] + in[o,1,n] + ... in that order (init == NULL: from 0.0f, as
 * tlc_sum_dim).  A sum over a dim whose entries are spread over devices or
 * ranks in order continues on each one from the previous one's result, which
 * gives the reference's single sequential sum bit for bit. */
int tlc_sum_dim_from(const float* in, const float* init, float* out, int64_t outer, int64_t D,
                     int64_t inner, void* stream);
/* out = a + b element-wise (same shape, contiguous): src/ops.cpp:75-103. */
int tlc_add(const float* a, const float* b, float* out, int64_t n, void* stream);
/* Tensor::contiguous (src/tensor.cpp:174-193): copy a strided view into a
 * dense row-major buffer. */
int tlc_contiguous(const tlc_tensor* src, float* dst, void* stream);

/* ---- the glue around the GEMMs in Linear and attention ---------------------
 * Device tensors; `out` is contiguous with the result's shape.  Element-wise
 * results are bit-identical to the reference except tlc_softmax (see there). */

/* out = scale * (a . b) + bias: tl::matmul fused with the tl::scale and
 * tl::add that follow it in the reference's callers (Linear::forward,
 * src/nn.cpp:77-83: add(matmul(x, W), b); MultiHeadAttention::forward,
 * src/nn.cpp:423-424: scale(matmul(q, k^T), 1/sqrt(d))).  Each output is the
 * product exactly as tlc_matmul computes it, then one fp32 multiply by
 * `scale` (skipped when scale == 1), then one fp32 add of bias[n]: the same
 * rounding as the separate ops.  `bias` is NULL or a 1-D tensor of length N. */
int tlc_matmul_fused(const tlc_tensor* a, const tlc_tensor* b, float scale, const tlc_tensor* bias,
                     tlc_tensor* out, int mode, void* stream);
/* tl::add with NumPy broadcasting (src/ops.cpp:74-103); "Incompatible
 * dimensions for broadcasting" as TLC_ERR_INVALID_ARGUMENT. */
int tlc_add_tensors(const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, void* stream);
/* tl::scale (src/ops.cpp:963-983): out = x * scale. */
int tlc_scale(const tlc_tensor* x, float scale, tlc_tensor* out, void* stream);
/* tl::softmax over the last dim (src/ops.cpp:985-1037).  Same steps and
 * order as the reference (row max, exp(x - max), sequential sum, divide); the
 * exponential is CUDA's expf rather than the C library's, so outputs agree
 * with the reference to a few ulp rather than bit for bit. */
int tlc_softmax(const tlc_tensor* x, tlc_tensor* out, void* stream);
/* SoftmaxBackward (src/autograd.cpp:228-256): dx = y * (grad - sum_j grad_j y_j)
 * per row, with the row dot rounded as the reference's x86-64-v4 build rounds
 * it (blocks of 8 rounded products added in order, the tail fused). */
int tlc_softmax_backward(const tlc_tensor* grad, const tlc_tensor* y, tlc_tensor* dx, void* stream);
/* sum_to (src/autograd.cpp:24-36): `out`'s shape is the target, a reduction of
 * x's shape (leading dims dropped, dims of size 1 kept); sequential sums from
 * 0.0f in the reference's order. */
int tlc_sum_to(const tlc_tensor* x, tlc_tensor* out, void* stream);

/* ---- conv2d ------------------------------------------------------------------
 * conv2d (src/ops.cpp:1443-1548) and Conv2dBackward (src/autograd.cpp:386-517)
 * for NCHW fp32 device tensors: input [N, C_in, H, W], weight
 * [C_out, C_in/groups, kH, kW], bias [C_out] or NULL, out [N, C_out, H_out,
 * W_out] with H_out = (H + 2*padding - kH) / stride + 1 (C++ division).
 * TLC_MODE_TF32 / _3XTF32 at stride 1 (output rows a multiple of 8 wide,
 * channels a multiple of 4): the forward product, the input gradient and the
 * weight gradient (split over output rows, the splits then summed in a fixed
 * order) are implicit GEMMs on the tensor cores reading TMA boxes of NHWC
 * copies (no column buffer); otherwise im2col for all images and groups at
 * once, then one batched GEMM per product in `mode`;
 * exact mode is bit-identical to the reference, backward
 * included (its per-image += order for the weight gradient, col2im's order
 * for the input gradient, its (n, oh, ow) order for the bias gradient).
 * Errors: the reference's ("conv2d: groups must be > 0", "conv2d: groups
 * doesn't divide C_in", "conv2d: groups doesn't divide C_out",
 * "conv2d: weight.sizes()[1] must equal C_in / groups"), plus non-4-D
 * operands and stride < 1 (the reference would index out of range or divide
 * by zero).  Backward outputs are contiguous and overwritten (0 + gradient,
 * as accumulate_grad stores a first gradient); pass NULL to skip one. */
int tlc_conv2d_shape(const tlc_tensor* input, const tlc_tensor* weight, int64_t stride,
                     int64_t padding, int64_t groups, int64_t* out_sizes);
int tlc_conv2d(const tlc_tensor* input, const tlc_tensor* weight, const tlc_tensor* bias,
               int64_t stride, int64_t padding, int64_t groups, tlc_tensor* out, int mode,
               void* stream);
int tlc_conv2d_backward(const tlc_tensor* grad_output, const tlc_tensor* input,
                        const tlc_tensor* weight, int64_t stride, int64_t padding, int64_t groups,
                        tlc_tensor* d_input, tlc_tensor* d_weight, tlc_tensor* d_bias, int mode,
                        void* stream);

/* ---- attention ---------------------------------------------------------------
 * flash_attention (src/ops.cpp:1040-1137): out = softmax(q . k^T * sm_scale) . v
 * for q, k, v, out contiguous [..., S, d] device tensors of one shape (every
 * leading index a separate head; the reference takes one head [S, d]),
 * d <= 128, no S x S buffer.  TLC_MODE_EXACT / _3XTF32: one fused fp32 FFMA
 * kernel with the reference's 64 x 64 tiles and online-softmax update;
 * TLC_MODE_TF32 with 32 <= d <= 64 (d % 4 == 0, 16-byte aligned q, k, v): the
 * same update around tcgen05 TF32 products (scores in tensor memory), within
 * the TF32 tolerance; other TF32 cases run the FFMA kernel.  `lse` ([..., S],
 * contiguous, or NULL) receives L = m + log(l), the reference's L_cache.
 * FlashAttentionBackward (src/autograd.cpp:575-669): d_q, d_k, d_v from
 * grad_out, the forward's inputs, out and lse; outputs are overwritten.
 * TLC_MODE_TF32 with 32 <= d <= 64 (d % 4 == 0, 16-byte aligned operands):
 * two fused tcgen05 kernels (dK / dV per key tile, dQ per query tile), no
 * S x S buffer; otherwise batched GEMMs in `mode` (S x S scratch per head, at
 * most 1 GiB per buffer).  Both agree with the reference to its own bar (1e-4 against
 * the materialised softmax path): expf / logf and the order of the softmax
 * sums differ from the C library's.  Errors: shapes that differ, non-contiguous
 * operands, fewer than 2 dims (TLC_ERR_INVALID_ARGUMENT); d > 128
 * (TLC_ERR_UNSUPPORTED). */
int tlc_flash_attention(const tlc_tensor* q, const tlc_tensor* k, const tlc_tensor* v,
                        float sm_scale, tlc_tensor* out, tlc_tensor* lse, int mode, void* stream);
int tlc_flash_attention_backward(const tlc_tensor* grad_out, const tlc_tensor* q,
                                 const tlc_tensor* k, const tlc_tensor* v, const tlc_tensor* out,
                                 const tlc_tensor* lse, float sm_scale, tlc_tensor* d_q,
                                 tlc_tensor* d_k, tlc_tensor* d_v, int mode, void* stream);

/* ---- TLMD model files straight to / from device memory --------------------
 * load_model / save_model (src/model_io.cpp:7-94): "TLMD", int32 version 1,
 * int64 count, then per tensor int64 ndim, int64 shape[ndim], float data.
 * tlc_load_tlmd checks the header and each tensor's ndim and shape against
 * `dst` (contiguous device tensors, in order) with the reference's messages
 * (TLC_ERR_IO: "load_model: cannot open file: <path>", "... no TLMD magic
 * header in <path>", "... unsupported version", "... tensor count mismatch",
 * "... ndim mismatch", "... shape mismatch"; and "load_model: file truncated"
 * for a file that ends early) and streams the data into device memory through
 * page-locked staging buffers, reads overlapping copies.  tlc_save_tlmd
 * writes device tensors (any strides) in the same format.  Both return when
 * all copies are done. */
int tlc_load_tlmd(const char* path, int32_t count, const tlc_tensor* dst, void* stream);
int tlc_save_tlmd(const char* path, int32_t count, const tlc_tensor* src, void* stream);

/* ---- device groups: one process over several GPUs ----------------------------
 * The reference spreads one matmul over host threads (gemm_mt's row bands,
 * src/ops.cpp:569-587); a group spreads it over GPUs of the box, called from
 * one host thread.  A batched / broadcast product is split over its flattened
 * batch (a broadcast operand goes whole to every GPU); a single product from
 * host buffers over row blocks of A and C; a single product in device memory
 * over output column blocks (A sent to every GPU by one NCCL broadcast, each
 * GPU its own column block of B).  Results are those of the single-device
 * entry points bit for bit: no product's additions are split across GPUs,
 * and the dB of a broadcast B is summed by an ordered chain over the GPUs
 * (tlc_sum_dim_from).  NCCL is loaded at run time; a device may be listed
 * more than once (its shares then run side by side).  Calls on one group are
 * serialised; a call returns when its results are in place (device form: in
 * stream order on `stream`). */
typedef struct tlc_group tlc_group;

/* A group over `devices[0..n)` (1 <= n <= 64): a stream and a worker thread
 * per member, peer access between members, and one NCCL communicator per
 * member when NCCL loads and the devices are distinct. */
int tlc_group_create(const int* devices, int n, tlc_group** out);
int tlc_group_destroy(tlc_group* g);
/* Members, and whether the group holds NCCL communicators (0 / 1). */
int tlc_group_size(const tlc_group* g, int* n, int* uses_nccl);
/* tl::matmul (src/ops.cpp:605-699) on host buffers over the group: each GPU
 * copies in its share, computes, copies its share of `out` back; the
 * multi-GPU form of tlc_matmul_host, same shapes and errors. */
int tlc_group_matmul_host(tlc_group* g, const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out,
                          int mode);
/* MatmulBackward (src/autograd.cpp:341-384) on host buffers over the group:
 * the multi-GPU form of tlc_matmul_backward_host. */
int tlc_group_matmul_backward_host(tlc_group* g, const tlc_tensor* grad, const tlc_tensor* a,
                                   const tlc_tensor* b, tlc_tensor* da, tlc_tensor* db,
                                   int accumulate, int mode);
/* tl::matmul with a, b and out in the memory of the group's first device (the
 * current device) over the group: the multi-GPU form of tlc_matmul, ordered
 * after and before the work of `stream` (on the first device). */
int tlc_group_matmul(tlc_group* g, const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out,
                     int mode, void* stream);

/* ---- multi-GPU partitioning ------------------------------------------------
 * One process per GPU.  A batched GEMM is split over its flattened batch
 * dimension, a single GEMM over output column blocks (operands replicated).
 * These compute a rank's share; the rank then runs tlc_gemm on it. */

/* Contiguous range [*begin, *end) of `count` units for `rank` of `world`
 * (the first count % world ranks get one extra). */
int tlc_shard_range(int64_t count, int world, int rank, int64_t* begin, int64_t* end);
/* Column block of an N-wide output for `rank`, block edges rounded to a
 * multiple of `align` columns (the last rank takes the remainder). */
int tlc_shard_cols(int64_t N, int world, int rank, int64_t align, int64_t* begin, int64_t* end);
/* After an all-gather of per-rank column blocks stored back to back
 * (rank r's block is [M, w_r] row-major at offset M * col_begin[r]), write the
 * row-major [M, N] result.  col_begin has world + 1 entries (col_begin[world] = N). */
int tlc_gather_colblocks(const float* gathered, float* out, int64_t M, int64_t N, int world,
                         const int64_t* col_begin, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TLC_H */
