// Memory-bound helpers of the matmul path: the ordered batch reduction of
// sum_to, the accumulate_grad add, strided->contiguous copies, and the
// column-block reassembly after a multi-GPU all-gather.  All are grid-stride
// loops sized to a multiple of the SM count.
#include "common.cuh"

namespace tlc {
namespace {

int grid_for(int64_t n, int threads) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            sms <= 0)
            sms = 148;
    }
    int64_t want = (n + threads - 1) / threads;
    int64_t cap = (int64_t)sms * 8;
    if (want > cap) want = cap;
    return (int)(want < 1 ? 1 : want);
}

// out[o, n] = ((0 + x[o,0,n]) + x[o,1,n]) + ... : the order of sum()
// (src/ops.cpp:1214-1222).  One thread per output element; threads of a warp
// take consecutive n, so every step of the d loop is a coalesced row read.
__global__ void sum_dim_kernel(const float* __restrict__ in, const float* __restrict__ init,
                               float* __restrict__ out, int64_t outer, int64_t D, int64_t inner) {
    const int64_t total = outer * inner;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = i / inner, n = i - o * inner;
        const float* p = in + o * D * inner + n;
        float acc = init ? init[i] : 0.0f;
        for (int64_t d = 0; d < D; ++d) acc = __fadd_rn(acc, p[d * inner]);
        out[i] = acc;
    }
}

// The same sums when there are few outputs and long chains (e.g. a bias
// gradient: D = 4096 rows into 4096 columns).  A block owns a strip of 32
// consecutive outputs of one `o`; warps 1..7 stage SUM_ROWS rows of the strip
// into a double-buffered shared tile (many loads in flight per thread), and
// warp 0, one lane per output, adds each tile's rows in ascending d.  The
// order of every sum is the reference's.
constexpr int SUM_ROWS = 168;  // rows per tile: 24 per loader warp (2 tiles: 42 KB)
__global__ void __launch_bounds__(256) sum_dim_strip_kernel(const float* __restrict__ in,
                                                            const float* __restrict__ init,
                                                            float* __restrict__ out, int64_t outer,
                                                            int64_t D, int64_t inner) {
    __shared__ float tile[2][SUM_ROWS][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t strips = (inner + 31) / 32;
    const int64_t o = blockIdx.x / strips;
    const int64_t n0 = (blockIdx.x - o * strips) * 32;
    const int64_t n = n0 + lane;
    const bool col_ok = n < inner;
    const float* base = in + o * D * inner + n;
    const int64_t tiles = (D + SUM_ROWS - 1) / SUM_ROWS;
    float acc = (init && col_ok) ? init[o * inner + n] : 0.0f;
    // loaders: warp w (1..7) stages rows w - 1, w + 6, ... of each tile
    auto stage = [&](int64_t t, int buf) {
        const int64_t d0 = t * SUM_ROWS;
        float v[SUM_ROWS / 7];
#pragma unroll
        for (int r = 0; r < SUM_ROWS / 7; ++r) {
            const int64_t d = d0 + (warp - 1) + 7 * r;
            v[r] = (col_ok && d < D) ? base[d * inner] : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < SUM_ROWS / 7; ++r) tile[buf][(warp - 1) + 7 * r][lane] = v[r];
    };
    if (warp > 0 && tiles > 0) stage(0, 0);
    __syncthreads();
    for (int64_t t = 0; t < tiles; ++t) {
        const int buf = (int)(t & 1);
        if (warp > 0) {
            if (t + 1 < tiles) stage(t + 1, buf ^ 1);
        } else {
            const int rows = (int)min((int64_t)SUM_ROWS, D - t * SUM_ROWS);
            for (int r = 0; r < rows; ++r) acc = __fadd_rn(acc, tile[buf][r][lane]);
        }
        __syncthreads();
    }
    if (warp == 0 && col_ok) out[o * inner + n] = acc;
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// out = 0 + in: what accumulate_grad stores into an empty gradient
// (zeros + d, src/autograd.cpp:18-21).  __fadd_rn keeps the add (it maps -0 to +0).
__global__ void zero_plus_kernel(const float* __restrict__ in, float* __restrict__ out,
                                 int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(0.0f, in[i]);
}

struct StridedView {
    int nd;
    int64_t sizes[TLC_MAX_DIMS];
    int64_t strides[TLC_MAX_DIMS];
};

// dst[i] = src[offset of multi-index i]: Tensor::contiguous (src/tensor.cpp:174-193).
__global__ void strided_copy_kernel(const float* __restrict__ src, StridedView v,
                                    float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i, off = 0;
        for (int d = v.nd - 1; d >= 0; --d) {
            const int64_t c = t % v.sizes[d];
            t /= v.sizes[d];
            off += c * v.strides[d];
        }
        dst[i] = src[off];
    }
}

// dst[offset_d(i)] = src[offset_s(i)] over the multi-index i of a shared shape.
__global__ void strided_copy_to_kernel(const float* __restrict__ src, StridedView vs,
                                       float* __restrict__ dst, StridedView vd, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i, os = 0, od = 0;
        for (int d = vs.nd - 1; d >= 0; --d) {
            const int64_t c = t % vs.sizes[d];
            t /= vs.sizes[d];
            os += c * vs.strides[d];
            od += c * vd.strides[d];
        }
        dst[od] = src[os];
    }
}

struct ColBlocks {
    int world;
    int64_t begin[65];
};

// out[m, n] = gathered[M * begin[r] + m * w_r + (n - begin[r])] with r the
// rank whose block holds column n.
__global__ void gather_colblocks_kernel(const float* __restrict__ g, float* __restrict__ out,
                                        int64_t M, int64_t N, ColBlocks cb) {
    const int64_t total = M * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / N, n = i - m * N;
        int r = 0;
        while (r + 1 < cb.world && n >= cb.begin[r + 1]) ++r;
        const int64_t w = cb.begin[r + 1] - cb.begin[r];
        out[i] = g[M * cb.begin[r] + m * w + (n - cb.begin[r])];
    }
}

}  // namespace

int launch_sum_dim(const float* in, float* out, int64_t outer, int64_t D, int64_t inner,
                   cudaStream_t s, const float* init) {
    const int64_t n = outer * inner;
    if (n == 0) return TLC_OK;
    // few outputs and long chains: the strip kernel keeps enough loads in flight
    const int64_t strips = outer * ((inner + 31) / 32);
    if (inner >= 32 && D >= 64 && n < 148 * 1024 && strips < (int64_t(1) << 31)) {
        sum_dim_strip_kernel<<<(unsigned)strips, 256, 0, s>>>(in, init, out, outer, D, inner);
        count_launch();
        return check_launch("sum_dim_strip");
    }
    sum_dim_kernel<<<grid_for(n, 256), 256, 0, s>>>(in, init, out, outer, D, inner);
    count_launch();
    return check_launch("sum_dim");
}

int launch_add(const float* a, const float* b, float* out, int64_t n, cudaStream_t s) {
    if (n == 0) return TLC_OK;
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, b, out, n);
    count_launch();
    return check_launch("add");
}

int launch_zero_plus(const float* in, float* out, int64_t n, cudaStream_t s) {
    if (n == 0) return TLC_OK;
    zero_plus_kernel<<<grid_for(n, 256), 256, 0, s>>>(in, out, n);
    count_launch();
    return check_launch("zero_plus");
}

int launch_strided_copy(const float* src, int nd, const int64_t* sizes, const int64_t* strides,
                        float* dst, cudaStream_t s) {
    StridedView v{};
    v.nd = nd;
    int64_t n = 1;
    for (int i = 0; i < nd; ++i) {
        v.sizes[i] = sizes[i];
        v.strides[i] = strides[i];
        n *= sizes[i];
    }
    if (n == 0) return TLC_OK;
    strided_copy_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, v, dst, n);
    count_launch();
    return check_launch("strided_copy");
}

int launch_strided_copy_to(const float* src, int nd, const int64_t* sizes, const int64_t* sstr,
                           float* dst, const int64_t* dstr, cudaStream_t s) {
    StridedView vs{}, vd{};
    vs.nd = vd.nd = nd;
    int64_t n = 1;
    for (int i = 0; i < nd; ++i) {
        vs.sizes[i] = vd.sizes[i] = sizes[i];
        vs.strides[i] = sstr[i];
        vd.strides[i] = dstr[i];
        n *= sizes[i];
    }
    if (n == 0) return TLC_OK;
    strided_copy_to_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, vs, dst, vd, n);
    count_launch();
    return check_launch("strided_copy_to");
}

int launch_fill_zero(float* p, int64_t n, cudaStream_t s) {
    if (n == 0) return TLC_OK;
    TLC_CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(float) * (size_t)n, s));
    return TLC_OK;
}

int launch_gather_colblocks(const float* g, float* out, int64_t M, int64_t N, int world,
                            const int64_t* begin, cudaStream_t s) {
    if (world < 1 || world > 64)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "gather_colblocks: world must be 1..64");
    ColBlocks cb{};
    cb.world = world;
    for (int r = 0; r <= world; ++r) cb.begin[r] = begin[r];
    if (cb.begin[0] != 0 || cb.begin[world] != N)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "gather_colblocks: blocks must cover [0, N)");
    for (int r = 0; r < world; ++r)
        if (cb.begin[r + 1] < cb.begin[r])
            return set_error(TLC_ERR_INVALID_ARGUMENT, "gather_colblocks: decreasing block edge");
    const int64_t n = M * N;
    if (n == 0) return TLC_OK;
    gather_colblocks_kernel<<<grid_for(n, 256), 256, 0, s>>>(g, out, M, N, cb);
    count_launch();
    return check_launch("gather_colblocks");
}

}  // namespace tlc
