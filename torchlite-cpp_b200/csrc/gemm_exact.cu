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
// Two kernels, one contract:
//
// exact_tma_kernel (operands TMA-readable: 16-byte aligned, strides multiples
// of 4 floats).  256 threads in 2 x 4 warps; k-tiles of 32 stream into a ring
// of shared-memory stages with cp.async.bulk.tensor, one "full" mbarrier per
// stage, and one "empty" mbarrier per stage that every warp arrives on when
// done with it; thread 0 issues the loads.  The FFMA loop carries no global
// loads, shared stores or address arithmetic, and warps never meet at a CTA
// barrier.  Each operand keeps its memory layout in shared memory:
//   K-major tile ([rows][32 k], a row-major A or the W^T view of a B):
//     128-byte rows with the 128-byte swizzle (16-byte chunk c of row r at
//     c ^ (r % 8)); a thread's 8 rows are 8 apart (its 8 B columns 4 apart),
//     so a warp's 16-byte reads of 4 k-values (8-byte reads of 2 for B) hit
//     distinct chunks: no bank conflicts.
//   MN-major tile ([32 k][rows], an M-major A or a row-major B): dense; a
//     warp reads consecutive 16-byte groups along m / n.
// With an N-major B the inner product runs on sm_100's packed fma.rn.f32x2
// (two IEEE fmaf per instruction, same rounding, so the chains stay
// bit-identical), on 128 x 256 tiles (8 x 16 per thread, one CTA per SM, four
// stages) when N >= 256, else 128 x 128.  With a K-major B (no column pairs in
// its loads) it is scalar FFMA.  128 x 128 tiles run 8 x 8 per thread, two
// CTAs per SM, three stages.
//
// exact_kernel (any other strides).  128x128 tile, k-tiles of 16, 256
// threads, 8x8 per thread; global loads go through registers into a double-
// buffered shared-memory stage, transposing K-major operands on the way so
// both operands sit k-major ([k][m], [k][n]) in shared memory.
//
// Transposed operand layouts (an M-major A, a K-major B: the transpose views
// MatmulBackward builds, src/autograd.cpp:370-371) are read in place by both
// kernels; nothing is materialised.
#include "common.cuh"
#include "tma.cuh"

#include <cstring>

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
    const float* bias;  // epilogue (see Gemm): c * scale if apply_scale, + bias[col]
    float scale;
    int apply_scale;
};

// The GEMM epilogue on one output value: one IEEE fp32 operation per step,
// as the reference's separate tl::scale / tl::add would round it.
__device__ __forceinline__ float epilogue(float v, int64_t col, const float* bias, float scale,
                                          int apply_scale) {
    if (apply_scale) v = __fmul_rn(v, scale);
    if (bias) v = __fadd_rn(v, bias[col]);
    return v;
}

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
                float v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    v[j] = (col + j < p.N)
                               ? epilogue(acc[i][4 * h + j], col + j, p.bias, p.scale, p.apply_scale)
                               : 0.0f;
                if (VC && col + 3 < p.N) {
                    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (col + j < p.N) dst[j] = v[j];
                }
            }
        }
        __syncthreads();  // shared tiles are reused by the next batch
    }
}

// ---- small problems --------------------------------------------------------------------
//
// exact_small_kernel: 32 x 64 output tiles, k-tiles of 16, 128 threads with
// 4 x 4 outputs each.  For products with fewer 128-row tiles than there are
// SMs (a 512^3 GEMM is 8 tiles of 128 x 256, the broadcast A[32,128,64].B[64,128]
// 32 tiles of 128 x 128), whose big-tile kernels leave most SMs idle: 16 to 32
// times as many CTAs, each output still one ascending-k fmaf chain from +0.
// Operands in any strides (one of the two matrix strides of each is 1), loads
// through registers into double-buffered k-major shared tiles, as in
// exact_kernel.
constexpr int SBM = 32, SBN = 64, SBK = 16, SNT = 128;
constexpr int SLDA = SBM + 4, SLDB = SBN + 4;

template <bool AK, bool BKM, bool VC>
__global__ void __launch_bounds__(SNT) exact_small_kernel(ExactParams p) {
    __shared__ __align__(16) float As[2][SBK * SLDA];
    __shared__ __align__(16) float Bs[2][SBK * SLDB];
    const int tid = threadIdx.x;
    const int tr = tid >> 4, tc = tid & 15;  // 8 x 16 threads of 4 x 4 outputs
    const int64_t m0 = (int64_t)blockIdx.y * SBM, n0 = (int64_t)blockIdx.x * SBN;
    const int64_t nk = (p.K + SBK - 1) / SBK;
    // this thread's loads: A 4 values, B 8 values per k-tile
    const int a_row = AK ? tid >> 2 : (tid & 7) * 4, a_k = AK ? (tid & 3) * 4 : tid >> 3;
    const int b_col = BKM ? tid >> 1 : (tid & 7) * 8, b_k = BKM ? (tid & 1) * 8 : tid >> 3;

    for (int64_t b = blockIdx.z; b < p.batch; b += gridDim.z) {
        int64_t oa, ob, oc;
        p.bo.get(b, oa, ob, oc);
        const float* Ab = p.A + oa + m0 * p.a_rs;
        const float* Bb = p.B + ob + n0 * p.b_cs;
        float ra[4], rb[8];
        auto load = [&](int64_t k0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = AK ? a_row : a_row + j, k = AK ? a_k + j : a_k;
                ra[j] = (m0 + r < p.M && k0 + k < p.K) ? __ldg(Ab + r * p.a_rs + (k0 + k) * p.a_cs) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = BKM ? b_col : b_col + j, k = BKM ? b_k + j : b_k;
                rb[j] = (n0 + c < p.N && k0 + k < p.K) ? __ldg(Bb + c * p.b_cs + (k0 + k) * p.b_rs) : 0.f;
            }
        };
        auto store = [&](int buf) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = AK ? a_row : a_row + j, k = AK ? a_k + j : a_k;
                As[buf][k * SLDA + r] = ra[j];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = BKM ? b_col : b_col + j, k = BKM ? b_k + j : b_k;
                Bs[buf][k * SLDB + c] = rb[j];
            }
        };
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        if (nk > 0) {
            load(0);
            store(0);
        }
        __syncthreads();
        for (int64_t kt = 0; kt < nk; ++kt) {
            const int buf = (int)(kt & 1);
            const bool more = kt + 1 < nk;
            if (more) load((kt + 1) * SBK);
#pragma unroll
            for (int kk = 0; kk < SBK; ++kk) {
                const float4 a = *reinterpret_cast<const float4*>(&As[buf][kk * SLDA + tr * 4]);
                const float4 bq = *reinterpret_cast<const float4*>(&Bs[buf][kk * SLDB + tc * 4]);
                const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (more) store(buf ^ 1);
            __syncthreads();
        }
        float* Cb = p.C + oc;
        const int64_t col = n0 + tc * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t row = m0 + tr * 4 + i;
            if (row >= p.M) continue;
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                v[j] = col + j < p.N ? epilogue(acc[i][j], col + j, p.bias, p.scale, p.apply_scale) : 0.f;
            float* dst = Cb + row * p.c_rs + col;
            if (VC && col + 3 < p.N) {
                *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (col + j < p.N) dst[j] = v[j];
            }
        }
        __syncthreads();  // shared tiles are reused by the next batch entry
    }
}

// ---- TMA-fed kernel ------------------------------------------------------------------

constexpr int TBM = 128, TBK = 32;

// Tile shapes.  WIDE (N-major B): 128 x 256 output tile, thread tile 8 x 16,
// one CTA per SM with a 4-stage ring (4 x 48 KB).  Otherwise (K-major B):
// 128 x 128, thread tile 8 x 8, two CTAs per SM with 3-stage rings (3 x 32 KB).
template <bool WIDE>
struct TmaCfg {
    static constexpr int BN = WIDE ? 256 : 128;
    static constexpr int NJ = WIDE ? 16 : 8;     // columns per thread
    static constexpr int WN = BN / 4;            // columns per warp (4 warps across)
    static constexpr int STAGES = WIDE ? 4 : 3;
    static constexpr int MIN_BLOCKS = WIDE ? 1 : 2;
    static constexpr int A_BYTES = TBM * TBK * 4;
    static constexpr int B_BYTES = BN * TBK * 4;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int SMEM = STAGES * STAGE + 256 + 1024;  // + barriers, cursor, alignment slack
};

struct ExactTmaParams {
    CUtensorMap tmA, tmB;
    float* C;
    int64_t c_rs;
    int64_t cbs[kMaxBatchDims];
    int bsz[kMaxBatchDims];
    int a_bc[kMaxBatchDims];  // 1: A indexes this batch dim, 0: broadcast (coordinate 0)
    int b_bc[kMaxBatchDims];
    int nb;
    int M, N, nk;
    int64_t batch;
    uint64_t timeout_ns;
    int* err;
    const float* bias;  // epilogue (see Gemm)
    float scale;
    int apply_scale;
};

// Packed fp32 pairs (sm_100 fma.rn.f32x2: two IEEE fused multiply-adds with
// round-to-nearest in one instruction, each lane exactly fmaf).
__device__ __forceinline__ uint64_t pack2(float x, float y) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& x, float& y) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v));
}
// d = a * b + d, element-wise on the pairs
__device__ __forceinline__ void fma2(uint64_t& d, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}

// Bounded wait for the phase of `bar` with the given parity.  Gives up when
// the CTA's abort flag is raised or the deadline passes (2 s: far above any
// legitimate wait); on expiry it raises the flag and records `site` in the
// device error word.
__device__ __forceinline__ bool exact_wait(uint64_t* bar, uint32_t parity,
                                           volatile int* abort_flag, uint64_t timeout_ns,
                                           int* err, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > timeout_ns) {
                *abort_flag = 1;
                atomicCAS(err, 0, site);
                return false;
            }
        }
    }
}

// Thread 0's load cursor (shared memory: it lives across the k-tile loop but
// only thread 0 touches it, so it should not hold registers in every thread).
struct IssueCursor {
    int64_t entry;   // this CTA's entry number of the next load
    int kt;          // its k-tile
    int slot;        // ring slot of the next load
    uint32_t phase;  // how often the ring wrapped before it (parity)
    uint32_t pend, pend_par;  // slots with a load thread 0 has not seen complete, and their parity
    int ca[kMaxBatchDims], cb[kMaxBatchDims];  // tensor-map batch coordinates of `entry`
};

// AK: A is K-major (row-major [M,K]); BKM: B is K-major ([N,K] storage);
// WIDE: 128 x 256 tiles (N-major B only; see TmaCfg).
//
// Each CTA walks a flat sequence of k-tiles: its batch entries blockIdx.z,
// blockIdx.z + gridDim.z, ..., nk k-tiles each.  k-tile g lives in ring slot
// g % STAGES.  full[s] completes when a slot's loads land; empty[s] when all
// 8 warps finished reading it (one arrival per warp), and thread 0 waits on
// it before reloading the slot.  So warps only wait for data, never for one
// another at a CTA barrier.
//
// Thread (warp wm, wn; lane tm, tn) rows: wm*64 + tm + 8i when A is K-major,
// wm*64 + {tm*4, 32 + tm*4} + 0..3 when M-major.  Columns: wn*WN + 16g +
// tn*4 + 0..3 (g < NJ/4) for an N-major B, wn*32 + tn + 4j for a K-major B.
//
// N-major B (packed): the product runs on fma.rn.f32x2.  acc2[i][jp] holds row
// i, columns 2jp and 2jp + 1 of the thread's NJ as a pair; B's 16-byte groups
// give the column pairs, A's value is duplicated into both halves (one move
// per A value and k, shared by NJ/2 packed FMAs).  A K-major B has no column
// pairs in its loads: scalar FFMA into accs.
template <bool AK, bool BKM, bool VC, bool WIDE>
__global__ void __launch_bounds__(NT, TmaCfg<WIDE>::MIN_BLOCKS)
    exact_tma_kernel(const __grid_constant__ ExactTmaParams p) {
    static_assert(!(WIDE && BKM), "wide tiles need an N-major B");
    constexpr bool PACKED = !BKM;
    using S = TmaCfg<WIDE>;
    constexpr int STAGES = S::STAGES, NJ = S::NJ, NJP = S::NJ / 2;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment: the 128-byte swizzle pattern repeats every 8 rows.
    // Offsetting the shared array itself (no round trip through an integer)
    // keeps the compiler aware that these are shared-memory addresses, so
    // the tile reads compile to 32-bit-addressed shared loads.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE);  // [STAGES]
    uint64_t* empty = full + STAGES;                                        // [STAGES]
    IssueCursor* cur = reinterpret_cast<IssueCursor*>(empty + STAGES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(cur + 1);

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int wm = warp & 1, wn = warp >> 1;  // 2 x 4 warps
    const int tm = lane >> 2, tn = lane & 3;  // 8 x 4 lanes
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NT / 32);
        }
        *abort_flag = 0;
        cur->entry = 0;
        cur->kt = 0;
        cur->slot = 0;
        cur->phase = 0;
        cur->pend = cur->pend_par = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        prefetch_map(&p.tmA);
        prefetch_map(&p.tmB);
    }
    __syncthreads();

    const int m0 = blockIdx.y * TBM, n0 = blockIdx.x * S::BN;
    const int64_t n_entries = (p.batch - 1 - (int64_t)blockIdx.z) / gridDim.z + 1;
    const int64_t total = n_entries * p.nk;

    // Thread 0: load the next k-tile of the sequence into its slot, after the
    // warps released the slot's previous k-tile (`wait_empty`).
    auto issue_next = [&](bool wait_empty) -> bool {
        IssueCursor& c = *cur;
        if (wait_empty && !exact_wait(&empty[c.slot], c.phase ^ 1u, abort_flag, p.timeout_ns, p.err, 12))
            return false;
        if (c.kt == 0) {
            int64_t r = (int64_t)blockIdx.z + c.entry * gridDim.z;
#pragma unroll
            for (int i = kMaxBatchDims - 1; i >= 0; --i) {
                int idx = 0;
                if (i < p.nb) {
                    idx = (int)(r % p.bsz[i]);
                    r /= p.bsz[i];
                }
                c.ca[i] = p.a_bc[i] ? idx : 0;
                c.cb[i] = p.b_bc[i] ? idx : 0;
            }
        }
        const int slot = c.slot;
        uint8_t* sa = smem + slot * S::STAGE;
        mbar_expect_tx(&full[slot], S::STAGE);
        const int k0 = c.kt * TBK;
        if (AK)
            tma_load_5d_local(sa, &p.tmA, &full[slot], k0, m0, c.ca[0], c.ca[1], c.ca[2]);
        else
            tma_load_5d_local(sa, &p.tmA, &full[slot], m0, k0, c.ca[0], c.ca[1], c.ca[2]);
        if (BKM)
            tma_load_5d_local(sa + S::A_BYTES, &p.tmB, &full[slot], k0, n0, c.cb[0], c.cb[1], c.cb[2]);
        else
            tma_load_5d_local(sa + S::A_BYTES, &p.tmB, &full[slot], n0, k0, c.cb[0], c.cb[1], c.cb[2]);
        c.pend |= 1u << slot;
        c.pend_par = (c.pend_par & ~(1u << slot)) | (c.phase << slot);
        if (++c.kt == p.nk) {
            c.kt = 0;
            ++c.entry;
        }
        if (++c.slot == STAGES) {
            c.slot = 0;
            c.phase ^= 1u;
        }
        return true;
    };

    bool ok = true;
    if (tid == 0)
        for (int64_t g = 0; g < STAGES - 1 && g < total; ++g) issue_next(false);  // fresh slots

    uint64_t acc2[PACKED ? 8 : 1][PACKED ? NJP : 1];
    float accs[PACKED ? 1 : 8][PACKED ? 1 : NJ];
    int64_t oc = 0;  // C offset of the current entry
    int kt = 0;
    int64_t entry = 0;
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t g = 0; g < total; ++g) {
        if (kt == 0) {
            if constexpr (PACKED) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int jp = 0; jp < NJP; ++jp) acc2[i][jp] = 0ull;  // +0.0f, +0.0f
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < NJ; ++j) accs[i][j] = 0.f;
            }
            int64_t r = (int64_t)blockIdx.z + entry * gridDim.z;
            oc = 0;
#pragma unroll
            for (int i = kMaxBatchDims - 1; i >= 0; --i) {
                if (i < p.nb) {
                    oc += (r % p.bsz[i]) * p.cbs[i];
                    r /= p.bsz[i];
                }
            }
        }
        // k-tile g + STAGES - 1 reuses the slot of k-tile g - 1
        if (tid == 0 && g + STAGES - 1 < total && !issue_next(g >= 1)) ok = false;
        if (!ok || !exact_wait(&full[slot], phase, abort_flag, p.timeout_ns, p.err, 11)) {
            ok = false;
            break;
        }
        if (tid == 0) cur->pend &= ~(1u << slot);
        {
            const uint8_t* sa = smem + slot * S::STAGE;
            const uint8_t* sb = sa + S::A_BYTES;
#pragma unroll 2
            for (int q = 0; q < TBK / 4; ++q) {  // groups of 4 k, ascending
                // A: a[i][u] = A[row i][4q + u]
                float a[8][4];
                if (AK) {
                    // row r = wm*64 + tm + 8i (r % 8 == tm): 16-byte chunk q of the row
                    const uint8_t* pa = sa + (wm * 64 + tm) * 128 + ((q ^ tm) << 4);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 v = *reinterpret_cast<const float4*>(pa + i * 8 * 128);
                        a[i][0] = v.x;
                        a[i][1] = v.y;
                        a[i][2] = v.z;
                        a[i][3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint8_t* pa = sa + (4 * q + u) * (TBM * 4) + (wm * 64 + tm * 4) * 4;
                        const float4 x = *reinterpret_cast<const float4*>(pa);
                        const float4 y = *reinterpret_cast<const float4*>(pa + 32 * 4);
                        a[0][u] = x.x; a[1][u] = x.y; a[2][u] = x.z; a[3][u] = x.w;
                        a[4][u] = y.x; a[5][u] = y.y; a[6][u] = y.z; a[7][u] = y.w;
                    }
                }
                if constexpr (PACKED) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {  // one k: 8 x NJP packed FMAs
                        const uint8_t* pb = sb + (4 * q + u) * (S::BN * 4) + (wn * S::WN + tn * 4) * 4;
                        uint64_t bp[NJP];
#pragma unroll
                        for (int g4 = 0; g4 < NJ / 4; ++g4) {
                            const float4 x = *reinterpret_cast<const float4*>(pb + g4 * 16 * 4);
                            bp[2 * g4] = pack2(x.x, x.y);
                            bp[2 * g4 + 1] = pack2(x.z, x.w);
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint64_t ad = pack2(a[i][u], a[i][u]);
#pragma unroll
                            for (int jp = 0; jp < NJP; ++jp) fma2(acc2[i][jp], ad, bp[jp]);
                        }
                    }
                } else {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {  // k = 4q + 2h, 4q + 2h + 1
                        // column c = wn*32 + tn + 4j (c % 8 == tn + 4 (j % 2)): 8 bytes of chunk q
                        float bv[8][2];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int c7 = tn + 4 * (j & 1);
                            const float2 v = *reinterpret_cast<const float2*>(
                                sb + (wn * S::WN + tn + 4 * j) * 128 + ((q ^ c7) << 4) + h * 8);
                            bv[j][0] = v.x;
                            bv[j][1] = v.y;
                        }
#pragma unroll
                        for (int t = 0; t < 2; ++t)
#pragma unroll
                            for (int i = 0; i < 8; ++i)
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    accs[i][j] = fmaf(a[i][2 * h + t], bv[j][t], accs[i][j]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done with the slot
        if (++slot == STAGES) {
            slot = 0;
            phase ^= 1u;
        }
        if (++kt < p.nk) continue;
        kt = 0;
        ++entry;

        float* Cb = p.C + oc;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = m0 + wm * 64 + (AK ? tm + 8 * i : (i < 4 ? tm * 4 + i : 32 + tm * 4 + (i - 4)));
            if (row >= p.M) continue;
            float* crow = Cb + (int64_t)row * p.c_rs;
            if constexpr (PACKED) {
#pragma unroll
                for (int g4 = 0; g4 < NJ / 4; ++g4) {
                    float v[4];
                    unpack2(acc2[i][2 * g4], v[0], v[1]);
                    unpack2(acc2[i][2 * g4 + 1], v[2], v[3]);
                    const int col = n0 + wn * S::WN + g4 * 16 + tn * 4;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (col + j < p.N) v[j] = epilogue(v[j], col + j, p.bias, p.scale, p.apply_scale);
                    if (VC && col + 3 < p.N) {
                        *reinterpret_cast<float4*>(crow + col) = make_float4(v[0], v[1], v[2], v[3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (col + j < p.N) crow[col + j] = v[j];
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int col = n0 + wn * S::WN + tn + 4 * j;
                    if (col < p.N) crow[col] = epilogue(accs[i][j], col, p.bias, p.scale, p.apply_scale);
                }
            }
        }
    }
    if (!ok && tid == 0) {
        // Drain: wait (bounded) for loads still in flight into shared memory.
        const uint32_t pend = cur->pend, pend_par = cur->pend_par;
        for (int s = 0; s < STAGES; ++s) {
            if (!(pend & (1u << s))) continue;
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(&full[s], (pend_par >> s) & 1u) &&
                   globaltimer() - t0 < p.timeout_ns) {
            }
        }
    }
}

template <bool AK, bool BKM, bool VC, bool WIDE>
int launch_tma_variant(const ExactTmaParams& p, dim3 grid, cudaStream_t s) {
    using S = TmaCfg<WIDE>;
    auto kernel = exact_tma_kernel<AK, BKM, VC, WIDE>;
    static DeviceOnce once;
    TLC_TRY(smem_limit_once(once, kernel, S::SMEM));
    kernel<<<grid, NT, S::SMEM, s>>>(p);
    count_launch();
    return check_launch("gemm_exact_tma");
}

// The TMA kernel when both operands are TMA-readable in place; returns
// TLC_ERR_UNSUPPORTED (without launching) otherwise.
int gemm_exact_tma(const Gemm& g, bool ak, bool bkm, bool vc, cudaStream_t s) {
    if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX - TBK) return TLC_ERR_UNSUPPORTED;
    for (int i = 0; i < g.nb; ++i)
        if (g.bsz[i] > INT32_MAX) return TLC_ERR_UNSUPPORTED;
    const int64_t a_os = ak ? g.a_rs : g.a_cs, b_os = bkm ? g.b_cs : g.b_rs;
    if (!tma_ok(g.A, a_os, g.abs_, g.nb) || !tma_ok(g.B, b_os, g.bbs, g.nb)) return TLC_ERR_UNSUPPORTED;
    // 256-column tiles for an N-major B at least that wide (a narrower B
    // would leave most of a wide tile idle)
    const bool wide = !bkm && g.N >= 256;
    const int bn = wide ? TmaCfg<true>::BN : TmaCfg<false>::BN;
    int* err = nullptr;
    TLC_TRY(tc_error_word(&err));
    ExactTmaParams p;
    memset(&p, 0, sizeof(p));
    int64_t bsz[kMaxBatchDims];
    for (int i = 0; i < kMaxBatchDims; ++i) bsz[i] = i < g.nb ? g.bsz[i] : 1;
    int64_t abst[kMaxBatchDims] = {}, bbst[kMaxBatchDims] = {};
    for (int i = 0; i < g.nb; ++i) {
        abst[i] = g.abs_[i];
        bbst[i] = g.bbs[i];
    }
    // A K-major: {K, M} boxes {32, 128}, swizzled; M-major: {M, K} boxes {128, 32}.
    // B K-major: {K, N} boxes {32, 128}, swizzled; N-major: {N, K} boxes {256, 32}.
    if (ak)
        TLC_TRY(encode_tiled(&p.tmA, g.A, g.K, g.M, a_os, bsz, abst, TBK, TBM, CU_TENSOR_MAP_SWIZZLE_128B));
    else
        TLC_TRY(encode_tiled(&p.tmA, g.A, g.M, g.K, a_os, bsz, abst, TBM, TBK, CU_TENSOR_MAP_SWIZZLE_NONE));
    if (bkm)
        TLC_TRY(encode_tiled(&p.tmB, g.B, g.K, g.N, b_os, bsz, bbst, TBK, bn, CU_TENSOR_MAP_SWIZZLE_128B));
    else
        TLC_TRY(encode_tiled(&p.tmB, g.B, g.N, g.K, b_os, bsz, bbst, bn, TBK, CU_TENSOR_MAP_SWIZZLE_NONE));
    p.C = g.C;
    p.c_rs = g.c_rs;
    p.nb = g.nb;
    for (int i = 0; i < kMaxBatchDims; ++i) {
        p.bsz[i] = (int)bsz[i];
        p.cbs[i] = i < g.nb ? g.cbs[i] : 0;
        p.a_bc[i] = (i < g.nb && g.abs_[i] != 0 && g.bsz[i] > 1) ? 1 : 0;
        p.b_bc[i] = (i < g.nb && g.bbs[i] != 0 && g.bsz[i] > 1) ? 1 : 0;
    }
    p.M = (int)g.M;
    p.N = (int)g.N;
    p.nk = (int)((g.K + TBK - 1) / TBK);
    p.batch = g.batch();
    p.timeout_ns = 2000000000ull;
    p.err = err;
    p.bias = g.bias;
    p.scale = g.scale;
    p.apply_scale = g.apply_scale;
    const int64_t gx = (g.N + bn - 1) / bn, gy = (g.M + TBM - 1) / TBM;
    if (gy > 65535) return TLC_ERR_UNSUPPORTED;
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(p.batch < 65535 ? p.batch : 65535));
    const int key = (wide ? 8 : 0) | (ak ? 4 : 0) | (bkm ? 2 : 0) | (vc ? 1 : 0);
    switch (key) {
        case 0: return launch_tma_variant<false, false, false, false>(p, grid, s);
        case 1: return launch_tma_variant<false, false, true, false>(p, grid, s);
        case 2: return launch_tma_variant<false, true, false, false>(p, grid, s);
        case 3: return launch_tma_variant<false, true, true, false>(p, grid, s);
        case 4: return launch_tma_variant<true, false, false, false>(p, grid, s);
        case 5: return launch_tma_variant<true, false, true, false>(p, grid, s);
        case 6: return launch_tma_variant<true, true, false, false>(p, grid, s);
        case 7: return launch_tma_variant<true, true, true, false>(p, grid, s);
        case 8: return launch_tma_variant<false, false, false, true>(p, grid, s);
        case 9: return launch_tma_variant<false, false, true, true>(p, grid, s);
        case 12: return launch_tma_variant<true, false, false, true>(p, grid, s);
        default: return launch_tma_variant<true, false, true, true>(p, grid, s);
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
    p.bias = g.bias;
    p.scale = g.scale;
    p.apply_scale = g.apply_scale;
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

    // Few big tiles (fewer than half the SMs): the small-tile kernel.
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t big_tiles = p.batch * ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
    if (p.K > 0 && 2 * big_tiles < sms) {
        const int64_t sx = (g.N + SBN - 1) / SBN, sy = (g.M + SBM - 1) / SBM;
        if (sy <= 65535) {
            dim3 sgrid((unsigned)sx, (unsigned)sy, (unsigned)(p.batch < 65535 ? p.batch : 65535));
            const int key = (ak ? 4 : 0) | (bkm ? 2 : 0) | (vc ? 1 : 0);
            switch (key) {
                case 0: exact_small_kernel<false, false, false><<<sgrid, SNT, 0, s>>>(p); break;
                case 1: exact_small_kernel<false, false, true><<<sgrid, SNT, 0, s>>>(p); break;
                case 2: exact_small_kernel<false, true, false><<<sgrid, SNT, 0, s>>>(p); break;
                case 3: exact_small_kernel<false, true, true><<<sgrid, SNT, 0, s>>>(p); break;
                case 4: exact_small_kernel<true, false, false><<<sgrid, SNT, 0, s>>>(p); break;
                case 5: exact_small_kernel<true, false, true><<<sgrid, SNT, 0, s>>>(p); break;
                case 6: exact_small_kernel<true, true, false><<<sgrid, SNT, 0, s>>>(p); break;
                default: exact_small_kernel<true, true, true><<<sgrid, SNT, 0, s>>>(p); break;
            }
            count_launch();
            return check_launch("gemm_exact_small");
        }
    }
    if (p.K > 0) {
        const int st = gemm_exact_tma(g, ak, bkm, vc, s);
        if (st != TLC_ERR_UNSUPPORTED) return st;
        clear_error();
    }
    const int64_t gx = (g.N + BN - 1) / BN, gy = (g.M + BM - 1) / BM;
    if (gy > 65535) return set_error(TLC_ERR_UNSUPPORTED, "gemm_exact: M too large");
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(p.batch < 65535 ? p.batch : 65535));
    if (ak && !bkm) return dispatch_vec<true, false>(p, grid, va, vb, vc, s);
    if (ak && bkm) return dispatch_vec<true, true>(p, grid, va, vb, vc, s);
    if (!ak && !bkm) return dispatch_vec<false, false>(p, grid, va, vb, vc, s);
    return dispatch_vec<false, true>(p, grid, va, vb, vc, s);
}

}  // namespace tlc
