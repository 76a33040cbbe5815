// Exact-mode GEMM: fp32 FFMA on the CUDA cores, bit-identical to the
// reference CPU kernel.
//
// The reference's x86 kernel gemm_blocked (src/ops.cpp:242-268) zeroes C and
// accumulates C[m,n] += A[m,k] * B[k,n] with k ascending per element; compiled
// with its Release flags that is one fused multiply-add per k, i.e. the chain
//     c = 0;  for k = 0 .. K-1:  c = fmaf(A[m,k], B[k,n], c).
// Every output element here is produced by exactly one thread, whose
// accumulator starts at 0 and takes the FFMAs in that same ascending-k order
// (k-tiles ascending, k within a tile ascending), so the result is the same
// bit pattern.  Out-of-range k (the K tail) contributes fmaf(0, 0, c) == c:
// c is never -0 (a chain started from +0 can only reach +0, never -0), so the
// padding cannot change a bit.
//
// Tiling: 128x128 output tile per CTA, k-tiles of 16, 256 threads, each thread
// an 8x8 register tile split 2x2 into 4x4 blocks (rows tm*4 and 32+tm*4 of the
// warp's 64 rows, columns tn*4 and 16+tn*4 of its 32), so every shared-memory
// read is a conflict-free 128-bit load.  Global loads go through registers
// into a double-buffered shared-memory stage, transposing K-major operands on
// the way so both operands sit k-major ([k][m], [k][n]) in shared memory.
// Transposed operand layouts (an M-major A, a K-major B: the transpose views
// MatmulBackward builds, src/autograd.cpp:370-371) are read in place by the
// matching loader; nothing is materialised.
#include "common.cuh"

namespace tlc {
namespace {

constexpr int BM = 128, BN = 128, BK = 16, PAD = 4, NT = 256;
constexpr int LDA_S = BM + PAD;  // shared row pitch (floats); keeps 16-byte alignment
constexpr int LDB_S = BN + PAD;

struct ExactParams {
    const float* A;
    const float* B;
    float* C;
    int64_t M, N, K;
    int64_t a_rs, a_cs, b_rs, b_cs, c_rs;
    BatchOffsets bo;
    int64_t batch;
};

// Loads one operand k-tile into 8 registers.
//  KMAJ = the operand's contiguous dimension is k: thread covers rows
//         r = (tid>>2) + 64*i, k-quad kq = tid&3 (4 consecutive k).
//  else the contiguous dimension is m (or n): thread covers k = (tid>>5) + 8*i,
//         quad q = tid&31 (4 consecutive m/n).
// `base` points at element (row 0, k 0) of this CTA's tile; `rs` is the
// element stride between rows (m or n), `ks` between k.
template <bool KMAJ, bool VEC>
__device__ __forceinline__ void load_tile(float (&r)[8], const float* base, int64_t rs,
                                          int64_t ks, int64_t rows_left, int64_t k_left,
                                          int tid) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        if (KMAJ) {
            const int row = (tid >> 2) + 64 * i;
            const int k = (tid & 3) * 4;
            const float* p = base + row * rs + k;  // ks == 1
            if (VEC) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row < rows_left && k < k_left) v = __ldg(reinterpret_cast<const float4*>(p));
                r[4 * i + 0] = v.x;
                r[4 * i + 1] = v.y;
                r[4 * i + 2] = v.z;
                r[4 * i + 3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    r[4 * i + j] = (row < rows_left && k + j < k_left) ? __ldg(p + j) : 0.f;
            }
        } else {
            const int k = (tid >> 5) + 8 * i;
            const int q = (tid & 31) * 4;
            const float* p = base + k * ks + q;  // rs == 1
            if (VEC) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (k < k_left && q < rows_left) v = __ldg(reinterpret_cast<const float4*>(p));
                r[4 * i + 0] = v.x;
                r[4 * i + 1] = v.y;
                r[4 * i + 2] = v.z;
                r[4 * i + 3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    r[4 * i + j] = (k < k_left && q + j < rows_left) ? __ldg(p + j) : 0.f;
            }
        }
    }
}

// Writes the 8 staged registers into the k-major shared tile s[k][row].
template <bool KMAJ, int LD>
__device__ __forceinline__ void store_tile(const float (&r)[8], float* s, int tid) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        if (KMAJ) {
            const int row = (tid >> 2) + 64 * i;
            const int k = (tid & 3) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) s[(k + j) * LD + row] = r[4 * i + j];
        } else {
            const int k = (tid >> 5) + 8 * i;
            const int q = (tid & 31) * 4;
            *reinterpret_cast<float4*>(&s[k * LD + q]) =
                make_float4(r[4 * i + 0], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
        }
    }
}

template <bool AK, bool BKM, bool VA, bool VB, bool VC>
__global__ void __launch_bounds__(NT, 2) exact_kernel(ExactParams p) {
    __shared__ __align__(16) float As[2][BK * LDA_S];
    __shared__ __align__(16) float Bs[2][BK * LDB_S];

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int wm = warp & 1, wn = warp >> 1;  // 2 x 4 warps of 64 x 32
    const int tm = lane >> 2, tn = lane & 3;  // 8 x 4 lanes of 8 x 8

    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;
    const int64_t nk = (p.K + BK - 1) / BK;

    for (int64_t b = blockIdx.z; b < p.batch; b += gridDim.z) {
        int64_t oa, ob, oc;
        p.bo.get(b, oa, ob, oc);
        // Tile origins: A at (m0, 0), B at (0, n0).
        const float* Ab = p.A + oa + m0 * p.a_rs;
        const float* Bb = p.B + ob + n0 * p.b_cs;
        // Row/k strides as the loaders see them.
        const int64_t a_row = AK ? p.a_rs : 1, a_k = AK ? 1 : p.a_cs;
        const int64_t b_row = BKM ? p.b_cs : 1, b_k = BKM ? 1 : p.b_rs;
        const int64_t m_left = p.M - m0, n_left = p.N - n0;

        float acc[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

        float ra[8], rb[8];
        if (nk > 0) {
            load_tile<AK, VA>(ra, Ab, a_row, a_k, m_left, p.K, tid);
            load_tile<BKM, VB>(rb, Bb, b_row, b_k, n_left, p.K, tid);
            store_tile<AK, LDA_S>(ra, As[0], tid);
            store_tile<BKM, LDB_S>(rb, Bs[0], tid);
        }
        __syncthreads();

        for (int64_t kt = 0; kt < nk; ++kt) {
            const int buf = (int)(kt & 1);
            const bool more = kt + 1 < nk;
            if (more) {
                const int64_t k0 = (kt + 1) * BK;
                load_tile<AK, VA>(ra, Ab + k0 * a_k, a_row, a_k, m_left, p.K - k0, tid);
                load_tile<BKM, VB>(rb, Bb + k0 * b_k, b_row, b_k, n_left, p.K - k0, tid);
            }
            const float* as = As[buf] + wm * 64 + tm * 4;
            const float* bs = Bs[buf] + wn * 32 + tn * 4;
#pragma unroll
            for (int kk = 0; kk < BK; ++kk) {
                const float4 a0 = *reinterpret_cast<const float4*>(as + kk * LDA_S);
                const float4 a1 = *reinterpret_cast<const float4*>(as + kk * LDA_S + 32);
                const float4 b0 = *reinterpret_cast<const float4*>(bs + kk * LDB_S);
                const float4 b1 = *reinterpret_cast<const float4*>(bs + kk * LDB_S + 16);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (more) {
                store_tile<AK, LDA_S>(ra, As[buf ^ 1], tid);
                store_tile<BKM, LDB_S>(rb, Bs[buf ^ 1], tid);
            }
            __syncthreads();
        }

        // Epilogue: rows wm*64 + {tm*4 + i, 32 + tm*4 + i}, cols wn*32 + {tn*4 + j, 16 + tn*4 + j}.
        float* Cb = p.C + oc;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t row = m0 + wm * 64 + (i < 4 ? tm * 4 + i : 32 + tm * 4 + (i - 4));
            if (row >= p.M) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t col = n0 + wn * 32 + h * 16 + tn * 4;
                float* dst = Cb + row * p.c_rs + col;
                if (VC && col + 3 < p.N) {
                    *reinterpret_cast<float4*>(dst) =
                        make_float4(acc[i][4 * h + 0], acc[i][4 * h + 1], acc[i][4 * h + 2],
                                    acc[i][4 * h + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (col + j < p.N) dst[j] = acc[i][4 * h + j];
                }
            }
        }
        __syncthreads();  // shared tiles are reused by the next batch
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <bool AK, bool BKM, bool VA, bool VB, bool VC>
int launch(const ExactParams& p, dim3 grid, cudaStream_t s) {
    exact_kernel<AK, BKM, VA, VB, VC><<<grid, NT, 0, s>>>(p);
    count_launch();
    return check_launch("gemm_exact");
}

template <bool AK, bool BKM>
int dispatch_vec(const ExactParams& p, dim3 grid, bool va, bool vb, bool vc, cudaStream_t s) {
    const int key = (va ? 4 : 0) | (vb ? 2 : 0) | (vc ? 1 : 0);
    switch (key) {
        case 0: return launch<AK, BKM, false, false, false>(p, grid, s);
        case 1: return launch<AK, BKM, false, false, true>(p, grid, s);
        case 2: return launch<AK, BKM, false, true, false>(p, grid, s);
        case 3: return launch<AK, BKM, false, true, true>(p, grid, s);
        case 4: return launch<AK, BKM, true, false, false>(p, grid, s);
        case 5: return launch<AK, BKM, true, false, true>(p, grid, s);
        case 6: return launch<AK, BKM, true, true, false>(p, grid, s);
        default: return launch<AK, BKM, true, true, true>(p, grid, s);
    }
}

}  // namespace

int gemm_exact(const Gemm& g, cudaStream_t s) {
    ExactParams p;
    p.A = g.A;
    p.B = g.B;
    p.C = g.C;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.a_rs = g.a_rs;
    p.a_cs = g.a_cs;
    p.b_rs = g.b_rs;
    p.b_cs = g.b_cs;
    p.c_rs = g.c_rs;
    p.bo = batch_offsets(g);
    p.batch = g.batch();
    if (p.batch == 0 || p.M == 0 || p.N == 0) return TLC_OK;

    const bool ak = g.a_cs == 1;   // else a_rs == 1
    const bool bkm = g.b_rs == 1 && g.b_cs != 1;  // B column-major (K contiguous)
    auto div4 = [](int64_t v) { return (v & 3) == 0; };
    bool bs_ok_a = true, bs_ok_b = true, bs_ok_c = true;
    for (int i = 0; i < g.nb; ++i) {
        bs_ok_a &= div4(g.abs_[i]);
        bs_ok_b &= div4(g.bbs[i]);
        bs_ok_c &= div4(g.cbs[i]);
    }
    // float4 loads need the contiguous extent and every outer stride to be
    // multiples of 4 floats and a 16-byte aligned base.
    const bool va = aligned16(g.A) && bs_ok_a &&
                    (ak ? div4(g.K) && div4(g.a_rs) : div4(g.M) && div4(g.a_cs));
    const bool vb = aligned16(g.B) && bs_ok_b &&
                    (bkm ? div4(g.K) && div4(g.b_cs) : div4(g.N) && div4(g.b_rs));
    const bool vc = aligned16(g.C) && bs_ok_c && div4(g.c_rs);

    const int64_t gx = (g.N + BN - 1) / BN, gy = (g.M + BM - 1) / BM;
    if (gy > 65535) return set_error(TLC_ERR_UNSUPPORTED, "gemm_exact: M too large");
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(p.batch < 65535 ? p.batch : 65535));
    if (ak && !bkm) return dispatch_vec<true, false>(p, grid, va, vb, vc, s);
    if (ak && bkm) return dispatch_vec<true, true>(p, grid, va, vb, vc, s);
    if (!ak && !bkm) return dispatch_vec<false, false>(p, grid, va, vb, vc, s);
    return dispatch_vec<false, true>(p, grid, va, vb, vc, s);
}

}  // namespace tlc
