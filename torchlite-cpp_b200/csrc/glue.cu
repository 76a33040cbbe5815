// Device kernels for the glue around the GEMMs in Linear and attention:
// tl::add with broadcasting (src/ops.cpp:74-103), tl::scale (:963-983),
// tl::softmax (:985-1037), SoftmaxBackward (src/autograd.cpp:228-256), and
// the in-place epilogue (scale, then bias) that the fused GEMM entry point
// applies when K == 0.  All HBM-bound: grid-stride loops, coalesced along the
// contiguous output.
//
// Rounding, element by element:
//  - add, scale, the epilogue: one IEEE fp32 operation each, as in the
//    reference: bit-identical.
//  - softmax: the row max as the reference picks it (first element, then
//    strictly greater: a NaN first element makes the row NaN, later NaNs are
//    skipped), e = expf(x - max), their sum in j order from 0.0f, e / sum
//    (IEEE division).  CUDA's expf is not the C library's, so results agree
//    with the reference to a few ulp, not bit for bit.
//  - SoftmaxBackward: bit-identical to the reference's x86-64-v4 build, whose
//    vectorised row dot product adds rounded products g_j * y_j in order for
//    the first D - D mod 8 elements and contracts the remaining ones into
//    fmaf(g_j, y_j, dot): each warp walks its row in that order (the values
//    reach lane 0 by shuffles), then dx_i = y_i * (g_i - dot).
#include "common.cuh"

#include <algorithm>

namespace tlc {
namespace {

constexpr int kEwMaxDims = TLC_MAX_DIMS;
// Rows from which the many-row kernels (a row per warp, block-shared
// sequential sums) are used.
constexpr int64_t kRowPerThread = 148 * 128;

// Output index -> operand offsets for a contiguous output of shape sz[0..nd).
struct EwIndex {
    int nd;
    int64_t sz[kEwMaxDims];
    int64_t sa[kEwMaxDims], sb[kEwMaxDims];  // element strides, 0 on broadcast dims
    __device__ __forceinline__ void offsets(int64_t i, int64_t& oa, int64_t& ob) const {
        oa = ob = 0;
#pragma unroll
        for (int d = kEwMaxDims - 1; d >= 0; --d) {
            if (d < nd) {
                const int64_t c = i % sz[d];
                i /= sz[d];
                oa += c * sa[d];
                ob += c * sb[d];
            }
        }
    }
};

// kind 0: out = a + b;  kind 1: out = a * s
__global__ void elementwise_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                   float s, float* __restrict__ out, int64_t n, EwIndex ix,
                                   int kind) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t oa, ob;
        ix.offsets(i, oa, ob);
        out[i] = kind == 0 ? __fadd_rn(a[oa], b[ob]) : __fmul_rn(a[oa], s);
    }
}

// The same operation row by row when the innermost (merged) dim is contiguous
// in a and out and a multiple of 4 long: one offset decode per row, float4
// loads and stores along it; b is one value per row (b_unit = 0) or a
// contiguous run (b_unit = 1).  The per-element roundings are the same.
__global__ void elementwise_rows_vec4_kernel(const float* __restrict__ a, const float* __restrict__ b, float s,
                                             float* __restrict__ out, int64_t rows, int L4, EwIndex ix, int kind,
                                             int b_unit) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        int64_t oa, ob;
        ix.offsets(r * (int64_t)L4 * 4, oa, ob);
        const float4* ar = reinterpret_cast<const float4*>(a + oa);
        float4* orow = reinterpret_cast<float4*>(out + r * (int64_t)L4 * 4);
        if (kind == 1) {
            for (int j = threadIdx.x; j < L4; j += blockDim.x) {
                const float4 x = ar[j];
                orow[j] = make_float4(__fmul_rn(x.x, s), __fmul_rn(x.y, s), __fmul_rn(x.z, s), __fmul_rn(x.w, s));
            }
        } else if (b_unit) {
            const float4* br = reinterpret_cast<const float4*>(b + ob);
            for (int j = threadIdx.x; j < L4; j += blockDim.x) {
                const float4 x = ar[j], y = br[j];
                orow[j] = make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z),
                                      __fadd_rn(x.w, y.w));
            }
        } else {
            const float y = b[ob];
            for (int j = threadIdx.x; j < L4; j += blockDim.x) {
                const float4 x = ar[j];
                orow[j] = make_float4(__fadd_rn(x.x, y), __fadd_rn(x.y, y), __fadd_rn(x.z, y), __fadd_rn(x.w, y));
            }
        }
    }
}

// C[r, c] = C[r, c] * s + bias[c] for a contiguous [rows, cols] block
// (the GEMM epilogue on an all-zero product, K == 0).
__global__ void epilogue_kernel(float* __restrict__ C, int64_t rows, int64_t cols, float s,
                                int apply_scale, const float* __restrict__ bias) {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float v = C[i];
        if (apply_scale) v = __fmul_rn(v, s);
        if (bias) v = __fadd_rn(v, bias[i % cols]);
        C[i] = v;
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One warp per row of D (rows contiguous).
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                               int64_t D) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const float* xr = x + r * D;
        float* yr = y + r * D;
        // max over the non-NaN values (fmaxf skips NaN); NaN if the first is NaN
        float m = -INFINITY;
        for (int64_t j = lane; j < D; j += 32) m = fmaxf(m, xr[j]);
        m = warp_max(m);
        const float x0 = xr[0];
        if (x0 != x0) m = x0;
        // e_j = exp(x_j - max), summed in j order from 0.0f as the reference
        // does (every lane carries the same running sum; values by shuffle)
        float s = 0.0f;
        for (int64_t j0 = 0; j0 < D; j0 += 32) {
            const int64_t j = j0 + lane;
            const float e = j < D ? expf(__fsub_rn(xr[j], m)) : 0.0f;
            if (j < D) yr[j] = e;
            const int cnt = D - j0 < 32 ? (int)(D - j0) : 32;
            for (int t = 0; t < cnt; ++t) s = __fadd_rn(s, __shfl_sync(0xffffffffu, e, t));
        }
        __syncwarp();
        for (int64_t j = lane; j < D; j += 32) yr[j] = __fdiv_rn(yr[j], s);
    }
}

// The same for rows of at most 32 * VPL: each lane keeps its VPL values in
// registers (element j = 32 i + lane), so a row is read once and written once.
template <int VPL>
__global__ void softmax_reg_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                                   int D) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const float* xr = x + r * D;
        float v[VPL];
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int j = 32 * i + lane;
            v[i] = j < D ? xr[j] : -INFINITY;
            m = fmaxf(m, v[i]);
        }
        m = warp_max(m);
        const float x0 = __shfl_sync(0xffffffffu, v[0], 0);
        if (x0 != x0) m = x0;
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int j0 = 32 * i;
            v[i] = (j0 + lane < D) ? expf(__fsub_rn(v[i], m)) : 0.0f;
            const int cnt = D - j0 < 32 ? D - j0 : 32;
            for (int t = 0; t < cnt; ++t) s = __fadd_rn(s, __shfl_sync(0xffffffffu, v[i], t));
        }
        float* yr = y + r * D;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int j = 32 * i + lane;
            if (j < D) yr[j] = __fdiv_rn(v[i], s);
        }
    }
}

// SoftmaxBackward for rows of at most 32 * VPL, g and y held in registers.
template <int VPL>
__global__ void softmax_backward_reg_kernel(const float* __restrict__ g, const float* __restrict__ y,
                                            float* __restrict__ dx, int64_t rows, int D) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int nv = D - D % 8;
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        float gv[VPL], yv[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int j = 32 * i + lane;
            gv[i] = j < D ? g[r * D + j] : 0.0f;
            yv[i] = j < D ? y[r * D + j] : 0.0f;
        }
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int j0 = 32 * i;
            const float p = __fmul_rn(gv[i], yv[i]);
            const int cnt = D - j0 < 32 ? D - j0 : 32;
            for (int t = 0; t < cnt; ++t) {
                if (j0 + t < nv) {
                    dot = __fadd_rn(dot, __shfl_sync(0xffffffffu, p, t));
                } else {
                    const float gt = __shfl_sync(0xffffffffu, gv[i], t);
                    const float yt = __shfl_sync(0xffffffffu, yv[i], t);
                    dot = __fmaf_rn(gt, yt, dot);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int j = 32 * i + lane;
            if (j < D) dx[r * D + j] = __fmul_rn(yv[i], __fsub_rn(gv[i], dot));
        }
    }
}

// Many rows of at most 32 * VPL: a block of ROWS warps takes ROWS rows, one
// per warp in registers (read once, written once).  Each warp computes its
// row's max and e = exp(x - max) and parks e in a padded shared tile; lane r
// of warp 0 then adds row r's e in j order (the reference's sequential sum,
// one lane per row instead of a shuffle chain on all 32 lanes), and every
// warp divides its registers by its row's sum.
constexpr int SM_ROWS = 16;
template <int VPL>
__global__ void __launch_bounds__(SM_ROWS * 32) softmax_block_kernel(const float* __restrict__ x,
                                                                     float* __restrict__ y,
                                                                     int64_t rows, int D) {
    extern __shared__ float sm[];
    float* tile = sm;                      // [SM_ROWS][D + 1]
    float* sums = sm + SM_ROWS * (D + 1);  // [SM_ROWS]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t r0 = (int64_t)blockIdx.x * SM_ROWS; r0 < rows; r0 += (int64_t)gridDim.x * SM_ROWS) {
        const int64_t r = r0 + warp;
        const bool valid = r < rows;
        float v[VPL];
        if (valid) {
            const float* xr = x + r * D;
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int j = 32 * i + lane;
                v[i] = j < D ? xr[j] : -INFINITY;
                m = fmaxf(m, v[i]);
            }
            m = warp_max(m);
            const float x0 = __shfl_sync(0xffffffffu, v[0], 0);
            if (x0 != x0) m = x0;
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int j = 32 * i + lane;
                if (j < D) {
                    v[i] = expf(__fsub_rn(v[i], m));
                    tile[warp * (D + 1) + j] = v[i];
                }
            }
        }
        __syncthreads();
        if (warp == 0 && lane < SM_ROWS && r0 + lane < rows) {
            const float* t = tile + lane * (D + 1);
            float s = 0.0f;
            for (int j = 0; j < D; ++j) s = __fadd_rn(s, t[j]);
            sums[lane] = s;
        }
        __syncthreads();
        if (valid) {
            const float s = sums[warp];
            float* yr = y + r * D;
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int j = 32 * i + lane;
                if (j < D) yr[j] = __fdiv_rn(v[i], s);
            }
        }
        __syncthreads();  // the tile and sums are reused by the next rows
    }
}

// Many rows of at most 32 * VPL: SoftmaxBackward with the softmax's block
// layout.  Each warp holds its row's g and y in registers and parks the
// rounded products g_j * y_j (j < D - D mod 8) and the tail's g_j, y_j in
// shared memory; lane r of warp 0 forms row r's dot in the reference build's
// order; every warp then writes dx = y * (g - dot) from its registers.
template <int VPL>
__global__ void __launch_bounds__(SM_ROWS * 32) softmax_backward_block_kernel(
    const float* __restrict__ g, const float* __restrict__ y, float* __restrict__ dx, int64_t rows,
    int D) {
    extern __shared__ float sm[];
    float* tile = sm;                          // [SM_ROWS][D + 1] rounded products
    float* tail_g = sm + SM_ROWS * (D + 1);    // [SM_ROWS][8]
    float* tail_y = tail_g + SM_ROWS * 8;      // [SM_ROWS][8]
    float* dots = tail_y + SM_ROWS * 8;        // [SM_ROWS]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nv = D - D % 8;
    for (int64_t r0 = (int64_t)blockIdx.x * SM_ROWS; r0 < rows; r0 += (int64_t)gridDim.x * SM_ROWS) {
        const int64_t r = r0 + warp;
        const bool valid = r < rows;
        float gv[VPL], yv[VPL];
        if (valid) {
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int j = 32 * i + lane;
                gv[i] = j < D ? g[r * D + j] : 0.0f;
                yv[i] = j < D ? y[r * D + j] : 0.0f;
                if (j < nv) {
                    tile[warp * (D + 1) + j] = __fmul_rn(gv[i], yv[i]);
                } else if (j < D) {
                    tail_g[warp * 8 + (j - nv)] = gv[i];
                    tail_y[warp * 8 + (j - nv)] = yv[i];
                }
            }
        }
        __syncthreads();
        if (warp == 0 && lane < SM_ROWS && r0 + lane < rows) {
            const float* t = tile + lane * (D + 1);
            float dot = 0.0f;
            for (int j = 0; j < nv; ++j) dot = __fadd_rn(dot, t[j]);
            for (int j = nv; j < D; ++j)
                dot = __fmaf_rn(tail_g[lane * 8 + (j - nv)], tail_y[lane * 8 + (j - nv)], dot);
            dots[lane] = dot;
        }
        __syncthreads();
        if (valid) {
            const float dot = dots[warp];
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int j = 32 * i + lane;
                if (j < D) dx[r * D + j] = __fmul_rn(yv[i], __fsub_rn(gv[i], dot));
            }
        }
        __syncthreads();
    }
}

// One warp per row: the reference build's dot order (blocks of 8 rounded
// products added in order, fused tail), then dx = y * (g - dot).
__global__ void softmax_backward_kernel(const float* __restrict__ g, const float* __restrict__ y,
                                        float* __restrict__ dx, int64_t rows, int64_t D) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t nv = D - D % 8;
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const float* gr = g + r * D;
        const float* yr = y + r * D;
        float dot = 0.0f;  // every lane carries the same running value
        for (int64_t j0 = 0; j0 < D; j0 += 32) {
            const int64_t j = j0 + lane;
            const float gv = j < D ? gr[j] : 0.0f;
            const float yv = j < D ? yr[j] : 0.0f;
            const float p = __fmul_rn(gv, yv);
            const int cnt = D - j0 < 32 ? (int)(D - j0) : 32;
            for (int t = 0; t < cnt; ++t) {
                if (j0 + t < nv) {
                    dot = __fadd_rn(dot, __shfl_sync(0xffffffffu, p, t));
                } else {
                    const float gt = __shfl_sync(0xffffffffu, gv, t);
                    const float yt = __shfl_sync(0xffffffffu, yv, t);
                    dot = __fmaf_rn(gt, yt, dot);
                }
            }
        }
        float* o = dx + r * D;
        for (int64_t j = lane; j < D; j += 32) o[j] = __fmul_rn(yr[j], __fsub_rn(gr[j], dot));
    }
}

int grid_for(int64_t n, int per_block) {
    const int64_t b = (n + per_block - 1) / per_block;
    return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 32));
}

}  // namespace

int launch_elementwise(const float* a, const float* b, float s, float* out, int64_t n, int nd,
                       const int64_t* sz, const int64_t* sa, const int64_t* sb, int kind,
                       cudaStream_t st) {
    if (n == 0) return TLC_OK;
    EwIndex ix{};
    // merge adjacent dims that walk both operands as one; drop size-1 dims
    int m = 0;
    for (int d = 0; d < nd; ++d) {
        if (sz[d] == 1) continue;
        if (m > 0 && ix.sa[m - 1] == sa[d] * sz[d] && ix.sb[m - 1] == sb[d] * sz[d]) {
            ix.sz[m - 1] *= sz[d];
            ix.sa[m - 1] = sa[d];
            ix.sb[m - 1] = sb[d];
            continue;
        }
        ix.sz[m] = sz[d];
        ix.sa[m] = sa[d];
        ix.sb[m] = sb[d];
        ++m;
    }
    ix.nd = m;
    // row-wise float4 path: innermost dim contiguous in a, a multiple of 4
    // long, every other a stride a multiple of 4, 16-byte aligned pointers;
    // b one value per row or a contiguous, equally aligned run
    auto al16p = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    bool rows_ok = m >= 1 && ix.sa[m - 1] == 1 && ix.sz[m - 1] % 4 == 0 && ix.sz[m - 1] / 4 <= INT32_MAX &&
                   al16p(a) && al16p(out);
    for (int d = 0; rows_ok && d < m - 1; ++d) rows_ok = ix.sa[d] % 4 == 0;
    int b_unit = 0;
    if (rows_ok && kind == 0) {
        if (ix.sb[m - 1] == 1) {
            b_unit = 1;
            rows_ok = al16p(b);
            for (int d = 0; rows_ok && d < m - 1; ++d) rows_ok = ix.sb[d] % 4 == 0;
        } else {
            rows_ok = ix.sb[m - 1] == 0;
        }
    }
    if (rows_ok) {
        const int64_t L = ix.sz[m - 1], rows = n / L;
        elementwise_rows_vec4_kernel<<<(unsigned)std::min<int64_t>(rows, 148 * 16), 256, 0, st>>>(
            a, b, s, out, rows, (int)(L / 4), ix, kind, b_unit);
        count_launch();
        return check_launch("elementwise");
    }
    elementwise_kernel<<<grid_for(n, 256), 256, 0, st>>>(a, b, s, out, n, ix, kind);
    count_launch();
    return check_launch("elementwise");
}

int launch_epilogue(float* C, int64_t rows, int64_t cols, float s, bool apply_scale,
                    const float* bias, cudaStream_t st) {
    if (rows * cols == 0 || (!apply_scale && !bias)) return TLC_OK;
    epilogue_kernel<<<grid_for(rows * cols, 256), 256, 0, st>>>(C, rows, cols, s, apply_scale ? 1 : 0,
                                                               bias);
    count_launch();
    return check_launch("epilogue");
}


template <int VPL>
int launch_softmax_block(const float* x, float* y, int64_t rows, int D, cudaStream_t st) {
    const size_t smem = sizeof(float) * (SM_ROWS * (size_t)(D + 1) + SM_ROWS);
    static DeviceOnce once;
    TLC_TRY(smem_limit_once(once, softmax_block_kernel<VPL>,
                            (int)(sizeof(float) * (SM_ROWS * 1025 + SM_ROWS))));
    const int64_t groups = (rows + SM_ROWS - 1) / SM_ROWS;
    const int grid = (int)std::min<int64_t>(groups, 148 * 8);
    softmax_block_kernel<VPL><<<grid, SM_ROWS * 32, smem, st>>>(x, y, rows, D);
    count_launch();
    return check_launch("softmax");
}

int launch_softmax(const float* x, float* y, int64_t rows, int64_t D, cudaStream_t st) {
    if (rows == 0 || D == 0) return TLC_OK;
    if (rows >= kRowPerThread && D <= 1024) {
        const int d = (int)D;
        if (D <= 32) return launch_softmax_block<1>(x, y, rows, d, st);
        if (D <= 64) return launch_softmax_block<2>(x, y, rows, d, st);
        if (D <= 128) return launch_softmax_block<4>(x, y, rows, d, st);
        if (D <= 256) return launch_softmax_block<8>(x, y, rows, d, st);
        if (D <= 512) return launch_softmax_block<16>(x, y, rows, d, st);
        return launch_softmax_block<32>(x, y, rows, d, st);
    }
    const int gb = grid_for(rows, 8);
    const int d = (int)std::min<int64_t>(D, 1 << 30);
    if (D <= 32) softmax_reg_kernel<1><<<gb, 256, 0, st>>>(x, y, rows, d);
    else if (D <= 64) softmax_reg_kernel<2><<<gb, 256, 0, st>>>(x, y, rows, d);
    else if (D <= 128) softmax_reg_kernel<4><<<gb, 256, 0, st>>>(x, y, rows, d);
    else if (D <= 256) softmax_reg_kernel<8><<<gb, 256, 0, st>>>(x, y, rows, d);
    else if (D <= 512) softmax_reg_kernel<16><<<gb, 256, 0, st>>>(x, y, rows, d);
    else if (D <= 1024) softmax_reg_kernel<32><<<gb, 256, 0, st>>>(x, y, rows, d);
    else softmax_kernel<<<gb, 256, 0, st>>>(x, y, rows, D);
    count_launch();
    return check_launch("softmax");
}

template <int VPL>
int launch_softmax_backward_block(const float* g, const float* y, float* dx, int64_t rows, int D,
                                  cudaStream_t st) {
    const size_t smem = sizeof(float) * (SM_ROWS * (size_t)(D + 1) + 2 * SM_ROWS * 8 + SM_ROWS);
    static DeviceOnce once;
    TLC_TRY(smem_limit_once(once, softmax_backward_block_kernel<VPL>,
                            (int)(sizeof(float) * (SM_ROWS * 1025 + 2 * SM_ROWS * 8 + SM_ROWS))));
    const int64_t groups = (rows + SM_ROWS - 1) / SM_ROWS;
    const int grid = (int)std::min<int64_t>(groups, 148 * 8);
    softmax_backward_block_kernel<VPL><<<grid, SM_ROWS * 32, smem, st>>>(g, y, dx, rows, D);
    count_launch();
    return check_launch("softmax_backward");
}

int launch_softmax_backward(const float* g, const float* y, float* dx, int64_t rows, int64_t D,
                            cudaStream_t st) {
    if (rows == 0 || D == 0) return TLC_OK;
    if (rows >= kRowPerThread && D <= 1024) {
        const int d = (int)D;
        if (D <= 32) return launch_softmax_backward_block<1>(g, y, dx, rows, d, st);
        if (D <= 64) return launch_softmax_backward_block<2>(g, y, dx, rows, d, st);
        if (D <= 128) return launch_softmax_backward_block<4>(g, y, dx, rows, d, st);
        if (D <= 256) return launch_softmax_backward_block<8>(g, y, dx, rows, d, st);
        if (D <= 512) return launch_softmax_backward_block<16>(g, y, dx, rows, d, st);
        return launch_softmax_backward_block<32>(g, y, dx, rows, d, st);
    }
    const int gb = grid_for(rows, 8);
    const int d = (int)std::min<int64_t>(D, 1 << 30);
    if (D <= 32) softmax_backward_reg_kernel<1><<<gb, 256, 0, st>>>(g, y, dx, rows, d);
    else if (D <= 64) softmax_backward_reg_kernel<2><<<gb, 256, 0, st>>>(g, y, dx, rows, d);
    else if (D <= 128) softmax_backward_reg_kernel<4><<<gb, 256, 0, st>>>(g, y, dx, rows, d);
    else if (D <= 256) softmax_backward_reg_kernel<8><<<gb, 256, 0, st>>>(g, y, dx, rows, d);
    else if (D <= 512) softmax_backward_reg_kernel<16><<<gb, 256, 0, st>>>(g, y, dx, rows, d);
    else if (D <= 1024) softmax_backward_reg_kernel<32><<<gb, 256, 0, st>>>(g, y, dx, rows, d);
    else softmax_backward_kernel<<<gb, 256, 0, st>>>(g, y, dx, rows, D);
    count_launch();
    return check_launch("softmax_backward");
}

}  // namespace tlc
