// FlashAttentionBackward (src/autograd.cpp:575-669 of torchlite-cpp) on the
// tensor cores: TLC_MODE_TF32, head dim 32 <= d <= 64 (d % 4 == 0, 16-byte
// aligned operands), one launch of each kernel below after a small prep.
//
// The reference recomputes, per 64 x 64 tile pair, S = Q_i . K_j^T * scale,
// P = exp(S - L_i), dP = dO_i . V_j^T, dS = P * (dP - D_i) (D = rowsum(dO * O))
// and accumulates dV_j += P^T . dO_i, dK_j += scale * dS^T . Q_i and
// dQ_i += scale * dS . K_j.  Here every product is a tcgen05.mma with fp32
// accumulators in tensor memory; no S x S intermediate leaves the SM.
//
//   fa_bwd_prep_kernel   D = rowsum(dO * O) and L2 = L * log2(e) into
//                        [heads, S_pad] scratch (S_pad = S rounded up to 128),
//                        zero past S.
//   flash_bwd_dkdv_kernel  one CTA per (head, 128 keys).  The CTA's K and V
//                        rows are written once into tensor memory, where the
//                        S^T = K . Q^T and dP^T = V . dO^T products read them
//                        as their A operand (an M = 128, N = 64 product whose
//                        A comes from shared memory runs at about a third of
//                        the rate of one whose A is in TMEM).  Query blocks of
//                        64 stream through a three-stage TMA ring, each as Q and
//                        dO twice (K-major for S^T and dP^T, MN-major for
//                        dV += P^T . dO and dK += dS^T . Q) with their L2, D.
//                        Sixteen elementwise warps (four per TMEM lane
//                        quarter, thread = key, a quarter of the block's
//                        queries) turn S^T,
//                        dP^T into P^T = 2^(S^T * scale * log2 e - L2) and
//                        dS^T = P^T * (dP^T - D) * scale in place in TMEM,
//                        where the next two MMAs read them as their A
//                        operand.  dK, dV accumulate in TMEM over all query
//                        blocks and are written once.
//   flash_bwd_dq_kernel  one CTA per (head, 128 queries): the same with the
//                        roles exchanged, Q and dO rows in TMEM, S = Q . K^T
//                        and dP = dO . V^T per block of 64 keys (K, V K-major
//                        and K MN-major in a four-stage ring), dS in place in
//                        TMEM, dQ += dS . K; three score buffers and two dP
//                        buffers (only the scores are read again by an MMA).
//
// Rows past S: TMA fills Q, K, V, dO rows past S with zeros and the padded
// L2, D are zero there, so every product term that involves such a row is
// zero, and rows past S are not stored.  The one exception is dS for keys
// past S in the dQ kernel, set to zero outright: there exp(-L) could overflow
// (a row whose scores all lie far below zero) and make 0 * inf.
//
// Scores and dP (or their transposes) of a block sit in one of two TMEM
// buffer pairs, so the MMA thread issues block i + 1's products while block
// i's elementwise step and products run.  Both kernels follow the forward kernel's protocol (flash_tc.cu):
// per-buffer full / empty mbarriers, every wait bounded (%globaltimer
// deadline, abort flag, the device error word), MMA completion tracked with
// tcgen05.commit.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace tlc {
namespace {

constexpr int BD = 64;          // head dim of the tiles (d <= 64, zero-filled)
constexpr int TR = 128;         // rows of a CTA's fixed tile = TMEM lanes = MMA M
constexpr int TB = 64;          // rows of a streamed block = MMA N / K
constexpr int EW_WARPS = 16;    // elementwise warps: four per TMEM lane quarter
constexpr int EW_COLS = TB / 4;  // columns (queries, keys or head dims) per elementwise thread
// warps: 0 producer, 1 the first MMA stream, 2.. elementwise, MMA2_WARP.. the
// other MMA streams (dK/dV kernel: S^T, dP^T, dV, dK; dQ kernel: S, dP, dQ)
constexpr int MMA2_WARP = 2 + EW_WARPS;
constexpr int DKV_THREADS = 32 * (MMA2_WARP + 3);
constexpr int DQ_THREADS = 32 * (MMA2_WARP + 2);
constexpr int TILE64 = TB * BD * 4;   // [64 x 64]: 2 boxes / chunks [64 x 32] of 8 KB
constexpr uint32_t kSleep = 100000;   // a waiting thread sleeps up to 100 us per poll
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr int NB = 2;  // score / dP buffer pairs in TMEM
static_assert(BD == TB, "the block width doubles as the head-dim tile in the descriptors");

// kind::tf32, fp32 D, M = 128, N = 64; A K-major (smem or TMEM), B K-major
// (bit 16 clear) or MN-major (bit 16 set).
constexpr uint32_t kIdescKK = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TB >> 3) << 17) |
                              ((uint32_t)(TR >> 4) << 24);
constexpr uint32_t kIdescKM = kIdescKK | (1u << 16);

struct BwdParams {
    CUtensorMap m[6];  // [2..5] used: see each kernel
    const float* L2;  // [heads, S_pad]
    const float* D;   // [heads, S_pad]
    const float* kv0;  // rows kept in TMEM: K (dkdv kernel) / Q (dq kernel)
    const float* kv1;  // V (dkdv kernel) / dO (dq kernel)
    float* out0;       // dK (dkdv kernel) / dQ (dq kernel)
    float* out1;       // dV (dkdv kernel)
    int S, S_pad, d, tiles, nblk;
    float scale;
    int* err;
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ bool wait_b(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                       const BwdParams& p, int site) {
    return wait_bounded(bar, parity, abort_flag, kTimeoutNs, p.err, site, kSleep);
}

// every lane of the warp waits (measured faster than lane 0 polling and
// sharing its result with a shuffle); true only if all succeeded
__device__ __forceinline__ bool warp_wait_b(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                            const BwdParams& p, int site) {
    return warp_wait_bounded(bar, parity, abort_flag, kTimeoutNs, p.err, site, kSleep);
}

// Shared-memory descriptor of k-step s (8 columns of 4 bytes) of a K-major
// tile made of two [rows x 32] SW128 boxes of `box` bytes each.
__device__ __forceinline__ uint64_t kmajor_step(uint64_t desc0, int box, int s) {
    return desc0 + (uint32_t)((((s >> 2) * box) + (s & 3) * 32) >> 4);
}
// k-step s (8 k-rows) of an MN-major tile: +1 KB per step.
__device__ __forceinline__ uint64_t mnmajor_step(uint64_t desc0, int s) {
    return desc0 + (uint32_t)((s * 1024) >> 4);
}

// Row `row` of one head's [S, d] rows (row-major), columns c0 .. c0 + 15,
// into this thread's TMEM lane at `taddr`: zero past S and past d.  d % 4 == 0
// and a 16-byte aligned base (checked on the host).
__device__ __forceinline__ void rows_to_tmem(const float* __restrict__ head_base, int row, int S, int d,
                                             int c0, uint32_t taddr) {
    uint32_t v[EW_COLS];
#pragma unroll
    for (int c = 0; c < EW_COLS; ++c) v[c] = 0u;
    if (row < S) {
        const float4* src = reinterpret_cast<const float4*>(head_base + (int64_t)row * d + c0);
#pragma unroll
        for (int c = 0; c < EW_COLS / 4; ++c)
            if (c0 + 4 * c < d) {
                const float4 x = __ldg(src + c);
                v[4 * c] = __float_as_uint(x.x);
                v[4 * c + 1] = __float_as_uint(x.y);
                v[4 * c + 2] = __float_as_uint(x.z);
                v[4 * c + 3] = __float_as_uint(x.w);
            }
    }
    tmem_st16(taddr, v);
}

// Final drain after a failed wait: wait (bounded) for loads still in flight
// into a full barrier of parity `par`.
__device__ __forceinline__ void drain_full(uint64_t* bar, uint32_t par) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, par) && globaltimer() - t0 < kTimeoutNs) {
    }
}

// ---------------------------------------------------------------------------------
// dK, dV.  m[2] Q (K-major, box 64 rows), m[3] Q (MN-major, 64), m[4] dO
// (K-major, 64), m[5] dO (MN-major, 64); K, V rows are read from `kv0`, `kv1`.
constexpr int QST = 3;  // query-block ring stages
constexpr int DKV_OFF_RING = 0;
// a stage: Qk | Qm | dOk | dOm | L2 (64 floats) | D (64 floats), padded to 1 KB so every
// stage's swizzled tiles start on a 1 KB boundary
constexpr int DKV_STAGE = 4 * TILE64 + 1024;
static_assert(DKV_STAGE % 1024 == 0 && 2 * TB * 4 <= 1024, "stage layout");
constexpr int DKV_OFF_BAR = DKV_OFF_RING + QST * DKV_STAGE;
constexpr int DKV_SMEM = DKV_OFF_BAR + 256 + 1024;
static_assert(DKV_SMEM <= 232448, "shared memory per CTA");
static_assert(8 * (1 + 2 * QST + 3 * NB + 2) + 8 <= 256, "barrier area");
// TMEM (both kernels): fixed A tiles at 0 and 64; score buffer b at 128 + b * 64,
// dP buffer b at 256 + b * 64; accumulators at 384 (and 448)
constexpr int TMEM_COLS = 512;
constexpr int A0_COL = 0, A1_COL = BD, S_COL = 2 * BD, DP_COL = S_COL + NB * TB, ACC0_COL = DP_COL + NB * TB,
              ACC1_COL = ACC0_COL + BD;
static_assert(ACC1_COL + BD <= TMEM_COLS, "TMEM columns");

__global__ void __launch_bounds__(DKV_THREADS, 1) flash_bwd_dkdv_kernel(const __grid_constant__ BwdParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DKV_OFF_BAR);
    uint64_t* a_full = bars;               // [1]  K, V rows in TMEM
    uint64_t* q_full = a_full + 1;         // [QST]
    uint64_t* q_empty = q_full + QST;      // [QST]
    uint64_t* s_full = q_empty + QST;      // [NB]  S^T and dP^T of a block computed
    uint64_t* s_empty = s_full + NB;       // [NB]  dV / dK of that buffer done
    uint64_t* e_full = s_empty + NB;       // [NB]  P^T, dS^T written (per buffer)
    uint64_t* acc_full = e_full + NB;      // [1]  every dV, dK product done
    uint64_t* drain = acc_full + 1;        // [4]  per MMA-issuing warp
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x / p.tiles;
    const int k0 = (blockIdx.x - head * p.tiles) * TR;

    if (threadIdx.x == 0) {
        mbar_init(a_full, EW_WARPS);
        for (int s = 0; s < QST; ++s) {
            mbar_init(&q_full[s], 1);
            mbar_init(&q_empty[s], 2);  // commits of the dV and dK streams
        }
        for (int b = 0; b < NB; ++b) {
            mbar_init(&s_full[b], 2);   // commits of the S^T and dP^T streams
            mbar_init(&s_empty[b], 2);  // commits of the dV and dK streams
            mbar_init(&e_full[b], EW_WARPS);
        }
        mbar_init(acc_full, 2);
        for (int r = 0; r < 4; ++r) mbar_init(&drain[r], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0 && lane == 0)
        for (int i = 2; i < 6; ++i) prefetch_map(&p.m[i]);
    if (warp == 1) {
        __syncwarp();
        tmem_alloc<1>(tmem_slot, TMEM_COLS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        // the warp waits together; one elected lane issues the copies
        {
            uint32_t pend = 0, par = 0;
            bool ok = true;
            for (int i = 0; i < p.nblk; ++i) {
                const int st = i % QST;
                const uint32_t ph = (uint32_t)(i / QST) & 1u;
                if (!warp_wait_b(&q_empty[st], ph ^ 1u, abort_flag, p, 41)) {
                    ok = false;
                    break;
                }
                pend &= ~(1u << st);
                uint8_t* sb = smem + DKV_OFF_RING + st * DKV_STAGE;
                if (elect_one()) {
                    mbar_expect_tx(&q_full[st], 4 * TILE64 + 2 * TB * 4);
                    const uint32_t fb = smem_u32(&q_full[st]);
                    for (int c = 0; c < 2; ++c) {
                        tma_load_5d<1>(sb + c * (TILE64 / 2), &p.m[2], fb, 32 * c, i * TB, head, 0, 0);
                        tma_load_5d<1>(sb + TILE64 + c * (TILE64 / 2), &p.m[3], fb, 32 * c, i * TB, head, 0, 0);
                        tma_load_5d<1>(sb + 2 * TILE64 + c * (TILE64 / 2), &p.m[4], fb, 32 * c, i * TB, head, 0, 0);
                        tma_load_5d<1>(sb + 3 * TILE64 + c * (TILE64 / 2), &p.m[5], fb, 32 * c, i * TB, head, 0, 0);
                    }
                    const int64_t lo = (int64_t)head * p.S_pad + (int64_t)i * TB;
                    bulk_load(sb + 4 * TILE64, p.L2 + lo, TB * 4, &q_full[st]);
                    bulk_load(sb + 4 * TILE64 + TB * 4, p.D + lo, TB * 4, &q_full[st]);
                }
                pend |= 1u << st;
                par = (par & ~(1u << st)) | (ph << st);
            }
            if (!ok && lane == 0)
                for (int s = 0; s < QST; ++s)
                    if (pend & (1u << s)) drain_full(&q_full[s], (par >> s) & 1u);
        }
    } else if (warp == 1 || warp >= MMA2_WARP) {
        // ---------------- MMA issuers ----------------
        // Four streams, one warp each: S^T (warp 1), dP^T, dV, dK.  One
        // thread's tcgen05.mma stream turns over about one N = 64 instruction
        // per 130 cycles, and separate streams overlap (measured); each
        // commit covers its own warp's MMAs, so the barriers a pair of
        // streams releases together count two arrivals.  Every lane polls the
        // barriers; one elected lane issues.
        {
            const int role = warp == 1 ? 0 : warp - MMA2_WARP + 1;  // 0 S^T, 1 dP^T, 2 dV, 3 dK
            const uint64_t r_kdesc = smem_desc(smem_u32(smem + DKV_OFF_RING), 16, 1024, kSw128);
            const uint64_t r_mdesc = smem_desc(smem_u32(smem + DKV_OFF_RING), TILE64 / 2, 512, kSw128Atom32);
            bool ok = warp_wait_b(a_full, 0, abort_flag, p, 42);
            bool issued = false;
            if (ok) tc_fence_after();
            if (role < 2) {
                // S^T = K . Q_i^T (A = K in TMEM) or dP^T = V . dO_i^T (A = V) into buffer i % NB
                for (int i = 0; ok && i < p.nblk; ++i) {
                    const int b = i % NB, st = i % QST;
                    ok = warp_wait_b(&q_full[st], (uint32_t)(i / QST) & 1u, abort_flag, p, 43);
                    if (ok) ok = warp_wait_b(&s_empty[b], ((uint32_t)(i / NB) & 1u) ^ 1u, abort_flag, p, 44);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t soff = (uint32_t)((st * DKV_STAGE) >> 4);
                    const uint32_t dst = tmem_base + (uint32_t)((role == 0 ? S_COL : DP_COL) + b * TB);
                    const uint32_t acol = role == 0 ? A0_COL : A1_COL;
                    const uint64_t bdesc = r_kdesc + soff + (role == 0 ? 0u : (uint32_t)((2 * TILE64) >> 4));
#pragma unroll
                    for (int s = 0; s < BD / 8; ++s)
                        if (elect_one())
                            umma_tf32_tmem_a(dst, tmem_base + (uint32_t)(acol + 8 * s),
                                             kmajor_step(bdesc, TILE64 / 2, s), kIdescKK, s > 0 ? 1u : 0u);
                    issued = true;
                    if (elect_one()) umma_commit<1>(smem_u32(&s_full[b]));
                }
            } else {
                // dV += P^T . dO_i (B = dO MN-major) or dK += dS^T . Q_i (B = Q MN-major)
                for (int i = 0; ok && i < p.nblk; ++i) {
                    const int b = i % NB, st = i % QST;
                    ok = warp_wait_b(&e_full[b], (uint32_t)(i / NB) & 1u, abort_flag, p, 45);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t soff = (uint32_t)((st * DKV_STAGE) >> 4);
                    const uint32_t acc = tmem_base + (uint32_t)(role == 2 ? ACC0_COL : ACC1_COL);
                    const uint32_t asrc = tmem_base + (uint32_t)((role == 2 ? S_COL : DP_COL) + b * TB);
                    const uint64_t bdesc = r_mdesc + soff + (uint32_t)(((role == 2 ? 3 : 1) * TILE64) >> 4);
#pragma unroll
                    for (int s = 0; s < TB / 8; ++s)
                        if (elect_one())
                            umma_tf32_tmem_a(acc, asrc + 8 * s, mnmajor_step(bdesc, s), kIdescKM,
                                             (i > 0 || s > 0) ? 1u : 0u);
                    issued = true;
                    if (elect_one()) umma_commit<1>(smem_u32(&s_empty[b]));
                    if (elect_one()) umma_commit<1>(smem_u32(&q_empty[st]));
                }
                if (ok && elect_one()) umma_commit<1>(smem_u32(acc_full));
            }
            if (!ok && issued && elect_one()) {
                umma_commit<1>(smem_u32(&drain[role]));
                drain_full(&drain[role], 0);
            }
            __syncwarp();
        }
    } else {
        // ---------------- elementwise (warps 2-17) ----------------
        const int part = (warp - 2) >> 2;  // quarter of the block's 64 queries / of the 64 columns
        const int c0 = EW_COLS * part;
        const int quarter = warp & 3;      // the TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const float sl2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
        // this CTA's K and V rows into TMEM: the A operands of S^T and dP^T
        const int64_t hoff = (int64_t)head * p.S * p.d;
        rows_to_tmem(p.kv0 + hoff, k0 + r, p.S, p.d, c0, lane_base + (uint32_t)(A0_COL + c0));
        rows_to_tmem(p.kv1 + hoff, k0 + r, p.S, p.d, c0, lane_base + (uint32_t)(A1_COL + c0));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full);
        bool ok = true;
        for (int i = 0; i < p.nblk && ok; ++i) {
            const int b = i % NB, st = i % QST;
            ok = warp_wait_b(&s_full[b], (uint32_t)(i / NB) & 1u, abort_flag, p, 46);
            // this block's L2, D landed in the stage (the stage is refilled only
            // after this block's dK product, which waits for this warp)
            if (ok) ok = warp_wait_b(&q_full[st], (uint32_t)(i / QST) & 1u, abort_flag, p, 48);
            if (!ok) break;
            tc_fence_after();
            uint32_t sv[EW_COLS], dv[EW_COLS];
            const uint32_t sa = lane_base + (uint32_t)(S_COL + b * TB + c0);
            const uint32_t pa = lane_base + (uint32_t)(DP_COL + b * TB + c0);
            tmem_ld16(sa, sv);
            tmem_ld16(pa, dv);
            const float4* lt4 = reinterpret_cast<const float4*>(smem + DKV_OFF_RING + st * DKV_STAGE + 4 * TILE64) + c0 / 4;
            float lt[EW_COLS], dt[EW_COLS];
#pragma unroll
            for (int c = 0; c < EW_COLS / 4; ++c) {
                const float4 x = lt4[c], y = lt4[TB / 4 + c];
                lt[4 * c] = x.x; lt[4 * c + 1] = x.y; lt[4 * c + 2] = x.z; lt[4 * c + 3] = x.w;
                dt[4 * c] = y.x; dt[4 * c + 1] = y.y; dt[4 * c + 2] = y.z; dt[4 * c + 3] = y.w;
            }
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < EW_COLS; ++c) {
                const float pr = ex2(fmaf(__uint_as_float(sv[c]), sl2, -lt[c]));
                const float g = __fmul_rn(__fmul_rn(pr, __fsub_rn(__uint_as_float(dv[c]), dt[c])), p.scale);
                sv[c] = __float_as_uint(pr);
                dv[c] = __float_as_uint(g);
            }
            tmem_st16(sa, sv);
            tmem_st16(pa, dv);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&e_full[b]);
        }
        // dK, dV rows of this CTA's keys: this thread's 16 columns of each
        if (ok) ok = warp_wait_b(acc_full, 0, abort_flag, p, 47);
        const int key = k0 + r;
        if (ok) {
            tc_fence_after();
            uint32_t vv[EW_COLS], kk[EW_COLS];
            tmem_ld16(lane_base + (uint32_t)(ACC0_COL + c0), vv);
            tmem_ld16(lane_base + (uint32_t)(ACC1_COL + c0), kk);
            tmem_wait_ld();
            if (key < p.S) {
                const int dc = p.d - c0;
                float* dvrow = p.out1 + ((int64_t)head * p.S + key) * p.d + c0;
                float* dkrow = p.out0 + ((int64_t)head * p.S + key) * p.d + c0;
                // d % 4 == 0 and 16-byte aligned rows (the kernel's preconditions):
                // float4 stores wherever 4 columns are inside d
#pragma unroll
                for (int c = 0; c < EW_COLS; c += 4)
                    if (c < dc) {
                        *reinterpret_cast<float4*>(dvrow + c) =
                            make_float4(__uint_as_float(vv[c]), __uint_as_float(vv[c + 1]),
                                        __uint_as_float(vv[c + 2]), __uint_as_float(vv[c + 3]));
                        *reinterpret_cast<float4*>(dkrow + c) =
                            make_float4(__uint_as_float(kk[c]), __uint_as_float(kk[c + 1]),
                                        __uint_as_float(kk[c + 2]), __uint_as_float(kk[c + 3]));
                    }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc<1>(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------
// dQ.  m[2] K (K-major, box 64 rows), m[3] V (K-major, 64), m[4] K (MN-major,
// 64); Q, dO rows are read from `kv0`, `kv1`.
constexpr int KST = 4;  // key-block ring stages
constexpr int DQ_OFF_RING = 0;
constexpr int DQ_STAGE = 3 * TILE64;  // Kk | Vk | Km
constexpr int DQ_OFF_BAR = DQ_OFF_RING + KST * DQ_STAGE;
constexpr int DQ_SMEM = DQ_OFF_BAR + 256 + 1024;
// Only the score buffer is read again by an MMA (dS over S feeds dQ += dS . K);
// a dP buffer is free once the elementwise warps loaded it.  So three score
// buffers and two dP buffers: TMEM Q at 0, dO at 64, S at 128 + b * 64,
// dP at 320 + b * 64, dQ at 448.
constexpr int DQ_NS = 3, DQ_NDP = 2;
constexpr int DQ_S_COL = 2 * BD, DQ_DP_COL = DQ_S_COL + DQ_NS * TB, DQ_ACC_COL = DQ_DP_COL + DQ_NDP * TB;
static_assert(DQ_ACC_COL + BD <= 512, "TMEM columns");
static_assert(DQ_SMEM <= 232448, "shared memory per CTA");
static_assert(8 * (1 + 2 * KST + 3 * DQ_NS + DQ_NDP + 2) + 8 <= 256, "barrier area");

__global__ void __launch_bounds__(DQ_THREADS, 1) flash_bwd_dq_kernel(const __grid_constant__ BwdParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DQ_OFF_BAR);
    uint64_t* a_full = bars;               // [1]  Q, dO rows in TMEM
    uint64_t* k_full = a_full + 1;         // [KST]
    uint64_t* k_empty = k_full + KST;      // [KST]
    uint64_t* s_full = k_empty + KST;      // [DQ_NS]  S and dP of a block computed
    uint64_t* s_empty = s_full + DQ_NS;    // [DQ_NS]  dQ product of that score buffer done
    uint64_t* e_full = s_empty + DQ_NS;    // [DQ_NS]  dS written (per score buffer)
    uint64_t* dp_empty = e_full + DQ_NS;   // [DQ_NDP] dP buffer loaded by the elementwise warps
    uint64_t* acc_full = dp_empty + DQ_NDP; // [1]
    uint64_t* drain = acc_full + 1;        // [4]  per MMA-issuing warp
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x / p.tiles;
    const int q0 = (blockIdx.x - head * p.tiles) * TR;

    if (threadIdx.x == 0) {
        mbar_init(a_full, EW_WARPS);
        for (int s = 0; s < KST; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int b = 0; b < DQ_NS; ++b) {
            mbar_init(&s_full[b], 2);   // commits of the S and dP streams
            mbar_init(&s_empty[b], 1);
            mbar_init(&e_full[b], EW_WARPS);
        }
        for (int b = 0; b < DQ_NDP; ++b) mbar_init(&dp_empty[b], EW_WARPS);
        mbar_init(acc_full, 1);
        for (int r = 0; r < 4; ++r) mbar_init(&drain[r], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0 && lane == 0)
        for (int i = 2; i < 5; ++i) prefetch_map(&p.m[i]);
    if (warp == 1) {
        __syncwarp();
        tmem_alloc<1>(tmem_slot, TMEM_COLS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        // the warp waits together; one elected lane issues the copies
        {
            uint32_t pend = 0, par = 0;
            bool ok = true;
            for (int j = 0; j < p.nblk; ++j) {
                const int st = j % KST;
                const uint32_t ph = (uint32_t)(j / KST) & 1u;
                if (!warp_wait_b(&k_empty[st], ph ^ 1u, abort_flag, p, 51)) {
                    ok = false;
                    break;
                }
                pend &= ~(1u << st);
                uint8_t* sb = smem + DQ_OFF_RING + st * DQ_STAGE;
                if (elect_one()) {
                    mbar_expect_tx(&k_full[st], DQ_STAGE);
                    const uint32_t fb = smem_u32(&k_full[st]);
                    for (int c = 0; c < 2; ++c) {
                        tma_load_5d<1>(sb + c * (TILE64 / 2), &p.m[2], fb, 32 * c, j * TB, head, 0, 0);
                        tma_load_5d<1>(sb + TILE64 + c * (TILE64 / 2), &p.m[3], fb, 32 * c, j * TB, head, 0, 0);
                        tma_load_5d<1>(sb + 2 * TILE64 + c * (TILE64 / 2), &p.m[4], fb, 32 * c, j * TB, head, 0, 0);
                    }
                }
                pend |= 1u << st;
                par = (par & ~(1u << st)) | (ph << st);
            }
            if (!ok && lane == 0)
                for (int s = 0; s < KST; ++s)
                    if (pend & (1u << s)) drain_full(&k_full[s], (par >> s) & 1u);
        }
    } else if (warp == 1 || warp >= MMA2_WARP) {
        // ---------------- MMA issuers ----------------
        // Three streams, one warp each: S (warp 1), dP, dQ (as in the dK/dV
        // kernel); s_full counts the S and dP streams' commits.
        {
            const int role = warp == 1 ? 0 : warp - MMA2_WARP + 1;  // 0 S, 1 dP, 2 dQ
            const uint64_t r_kdesc = smem_desc(smem_u32(smem + DQ_OFF_RING), 16, 1024, kSw128);
            const uint64_t r_mdesc = smem_desc(smem_u32(smem + DQ_OFF_RING), TILE64 / 2, 512, kSw128Atom32);
            bool ok = warp_wait_b(a_full, 0, abort_flag, p, 52);
            bool issued = false;
            if (ok) tc_fence_after();
            if (role < 2) {
                // S = Q . K_j^T (A = Q in TMEM) into score buffer j % DQ_NS, or
                // dP = dO . V_j^T (A = dO) into dP buffer j % DQ_NDP
                for (int j = 0; ok && j < p.nblk; ++j) {
                    const int b = j % DQ_NS, pb = j % DQ_NDP, st = j % KST;
                    ok = warp_wait_b(&k_full[st], (uint32_t)(j / KST) & 1u, abort_flag, p, 53);
                    if (ok) {
                        ok = role == 0
                                 ? warp_wait_b(&s_empty[b], ((uint32_t)(j / DQ_NS) & 1u) ^ 1u, abort_flag, p, 54)
                                 : warp_wait_b(&dp_empty[pb], ((uint32_t)(j / DQ_NDP) & 1u) ^ 1u, abort_flag, p, 58);
                    }
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t soff = (uint32_t)((st * DQ_STAGE) >> 4);
                    const uint32_t dst = tmem_base + (uint32_t)(role == 0 ? DQ_S_COL + b * TB : DQ_DP_COL + pb * TB);
                    const uint32_t acol = role == 0 ? A0_COL : A1_COL;
                    const uint64_t bdesc = r_kdesc + soff + (role == 0 ? 0u : (uint32_t)(TILE64 >> 4));
#pragma unroll
                    for (int s = 0; s < BD / 8; ++s)
                        if (elect_one())
                            umma_tf32_tmem_a(dst, tmem_base + (uint32_t)(acol + 8 * s),
                                             kmajor_step(bdesc, TILE64 / 2, s), kIdescKK, s > 0 ? 1u : 0u);
                    issued = true;
                    if (elect_one()) umma_commit<1>(smem_u32(&s_full[b]));
                }
            } else {
                for (int j = 0; ok && j < p.nblk; ++j) {
                    const int b = j % DQ_NS, st = j % KST;
                    ok = warp_wait_b(&e_full[b], (uint32_t)(j / DQ_NS) & 1u, abort_flag, p, 55);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t soff = (uint32_t)((st * DQ_STAGE) >> 4);
                    const uint32_t dsa = tmem_base + (uint32_t)(DQ_S_COL + b * TB);
                    // dQ += dS . K_j (A = dS in TMEM, B = K MN-major)
#pragma unroll
                    for (int s = 0; s < TB / 8; ++s)
                        if (elect_one())
                            umma_tf32_tmem_a(tmem_base + (uint32_t)DQ_ACC_COL, dsa + 8 * s,
                                             mnmajor_step(r_mdesc + soff + (uint32_t)((2 * TILE64) >> 4), s),
                                             kIdescKM, (j > 0 || s > 0) ? 1u : 0u);
                    issued = true;
                    if (elect_one()) umma_commit<1>(smem_u32(&s_empty[b]));
                    if (elect_one()) umma_commit<1>(smem_u32(&k_empty[st]));
                }
                if (ok && elect_one()) umma_commit<1>(smem_u32(acc_full));
            }
            if (!ok && issued && elect_one()) {
                umma_commit<1>(smem_u32(&drain[role]));
                drain_full(&drain[role], 0);
            }
            __syncwarp();
        }
    } else {
        // ---------------- elementwise (warps 2-17) ----------------
        const int part = (warp - 2) >> 2;  // quarter of the block's 64 keys / of the 64 columns
        const int c0 = EW_COLS * part;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int row = q0 + r;            // < S_pad: tiles * 128 <= S_pad
        const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const float sl2 = p.scale * 1.4426950408889634f;
        // this CTA's Q and dO rows into TMEM: the A operands of S and dP
        const int64_t hoff = (int64_t)head * p.S * p.d;
        rows_to_tmem(p.kv0 + hoff, row, p.S, p.d, c0, lane_base + (uint32_t)(A0_COL + c0));
        rows_to_tmem(p.kv1 + hoff, row, p.S, p.d, c0, lane_base + (uint32_t)(A1_COL + c0));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full);
        const float l2 = p.L2[(int64_t)head * p.S_pad + row];
        const float dr = p.D[(int64_t)head * p.S_pad + row];
        bool ok = true;
        for (int j = 0; j < p.nblk && ok; ++j) {
            const int b = j % DQ_NS, pb = j % DQ_NDP;
            ok = warp_wait_b(&s_full[b], (uint32_t)(j / DQ_NS) & 1u, abort_flag, p, 56);
            if (!ok) break;
            tc_fence_after();
            uint32_t sv[EW_COLS], dv[EW_COLS];
            const uint32_t sa = lane_base + (uint32_t)(DQ_S_COL + b * TB + c0);
            tmem_ld16(sa, sv);
            tmem_ld16(lane_base + (uint32_t)(DQ_DP_COL + pb * TB + c0), dv);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&dp_empty[pb]);  // the dP buffer may be refilled
#pragma unroll
            for (int c = 0; c < EW_COLS; ++c) {
                const float pr = ex2(fmaf(__uint_as_float(sv[c]), sl2, -l2));
                sv[c] = __float_as_uint(__fmul_rn(__fmul_rn(pr, __fsub_rn(__uint_as_float(dv[c]), dr)), p.scale));
            }
            // keys past S: K, V rows there are zero, but exp(-L) may overflow for a
            // row whose scores are all far below zero; their dS is zero outright
            const int valid = p.S - j * TB - c0;
            if (valid < EW_COLS) {
#pragma unroll
                for (int c = 0; c < EW_COLS; ++c)
                    if (c >= valid) sv[c] = 0u;
            }
            tmem_st16(sa, sv);  // dS over S: the A operand of dQ += dS . K
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&e_full[b]);
        }
        if (ok) ok = warp_wait_b(acc_full, 0, abort_flag, p, 57);
        if (ok) {
            tc_fence_after();
            uint32_t qv[EW_COLS];
            tmem_ld16(lane_base + (uint32_t)(DQ_ACC_COL + c0), qv);
            tmem_wait_ld();
            if (row < p.S) {
                const int dc = p.d - c0;
                float* qrow = p.out0 + ((int64_t)head * p.S + row) * p.d + c0;
#pragma unroll
                for (int c = 0; c < EW_COLS; c += 4)
                    if (c < dc)
                        *reinterpret_cast<float4*>(qrow + c) =
                            make_float4(__uint_as_float(qv[c]), __uint_as_float(qv[c + 1]),
                                        __uint_as_float(qv[c + 2]), __uint_as_float(qv[c + 3]));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc<1>(tmem_base, TMEM_COLS);
    }
}

// D = rowsum(dO * O) and L2 = L * log2(e) per row into [heads, S_pad], zero
// past S.  Half a warp per row: float4 loads (d % 4 == 0, 16-byte aligned
// rows), a shuffle sum over the 16 lanes.
__global__ void fa_bwd_prep_kernel(const float* __restrict__ dO, const float* __restrict__ O,
                                   const float* __restrict__ L, float* __restrict__ D,
                                   float* __restrict__ L2, int64_t heads, int S, int S_pad, int d) {
    const int64_t n = heads * S_pad;
    const int sub = threadIdx.x & 15, half = (threadIdx.x >> 4) & 1;
    const int64_t warp_id = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    // a warp takes rows 2 * pair and 2 * pair + 1; the loop bound is the same for
    // the whole warp, so every lane reaches every shuffle
    for (int64_t pair = warp_id; 2 * pair < n; pair += warps) {
        const int64_t i = 2 * pair + half;
        const bool live = i < n;
        const int64_t hd = live ? i / S_pad : 0;
        const int row = live ? (int)(i - hd * S_pad) : S;
        float acc = 0.0f;
        if (row < S) {
            const float4* g4 = reinterpret_cast<const float4*>(dO + (hd * S + row) * (int64_t)d);
            const float4* o4 = reinterpret_cast<const float4*>(O + (hd * S + row) * (int64_t)d);
            for (int c = sub; c < d / 4; c += 16) {
                const float4 x = __ldg(g4 + c), y = __ldg(o4 + c);
                acc = fmaf(x.x, y.x, acc);
                acc = fmaf(x.y, y.y, acc);
                acc = fmaf(x.z, y.z, acc);
                acc = fmaf(x.w, y.w, acc);
            }
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off, 16);
        if (live && sub == 0) {
            D[i] = acc;
            L2[i] = row < S ? __fmul_rn(L[hd * S + row], 1.4426950408889634f) : 0.0f;
        }
    }
}

}  // namespace

bool flash_bwd_tc_supported(int d, const float* const* ptrs, int n) {
    if (d < 32 || d > BD || d % 4 != 0) return false;
    for (int i = 0; i < n; ++i)
        if (!al16(ptrs[i])) return false;
    return true;
}

int flash_backward_tc(const float* dout, const float* q, const float* k, const float* v,
                      const float* o, const float* lse, float* dq, float* dk, float* dv,
                      int64_t heads, int S, int d, float scale, cudaStream_t s) {
    static DeviceOnce cfg_dkdv, cfg_dq;
    TLC_TRY(smem_limit_once(cfg_dkdv, flash_bwd_dkdv_kernel, DKV_SMEM));
    TLC_TRY(smem_limit_once(cfg_dq, flash_bwd_dq_kernel, DQ_SMEM));
    if (heads > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "flash_attention_backward: too many heads");
    const int tiles = (S + TR - 1) / TR;
    const int S_pad = tiles * TR;
    const int64_t grid = (int64_t)tiles * heads;
    if (grid > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "flash_attention_backward: too many tiles");
    void* scratch = nullptr;
    TLC_TRY(scratch_alloc(&scratch, sizeof(float) * 2 * (size_t)(heads * S_pad), s));
    float* Dp = static_cast<float*>(scratch);
    float* L2p = Dp + heads * S_pad;
    int rc = TLC_OK;
    do {
        const int64_t n = heads * S_pad;
        const int pg = (int)std::max<int64_t>(1, std::min<int64_t>((16 * n + 255) / 256, 148 * 32));
        fa_bwd_prep_kernel<<<pg, 256, 0, s>>>(dout, o, lse, Dp, L2p, heads, S, S_pad, d);
        count_launch();
        if ((rc = check_launch("flash_attention_backward")) != TLC_OK) break;

        const int64_t bsz[kMaxBatchDims] = {heads, 1, 1};
        const int64_t bstr[kMaxBatchDims] = {(int64_t)S * d, 0, 0};
        BwdParams p;
        memset(&p, 0, sizeof(p));
        p.L2 = L2p;
        p.D = Dp;
        p.S = S;
        p.S_pad = S_pad;
        p.d = d;
        p.tiles = tiles;
        p.nblk = S_pad / TB;
        p.scale = scale;
        if ((rc = tc_error_word(&p.err)) != TLC_OK) break;
        const CUtensorMapSwizzle K_SW = CU_TENSOR_MAP_SWIZZLE_128B, M_SW = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
        // dK, dV
        if ((rc = encode_tiled(&p.m[2], q, d, S, d, bsz, bstr, 32, TB, K_SW)) != TLC_OK) break;
        if ((rc = encode_tiled(&p.m[3], q, d, S, d, bsz, bstr, 32, TB, M_SW)) != TLC_OK) break;
        if ((rc = encode_tiled(&p.m[4], dout, d, S, d, bsz, bstr, 32, TB, K_SW)) != TLC_OK) break;
        if ((rc = encode_tiled(&p.m[5], dout, d, S, d, bsz, bstr, 32, TB, M_SW)) != TLC_OK) break;
        p.kv0 = k;
        p.kv1 = v;
        p.out0 = dk;
        p.out1 = dv;
        flash_bwd_dkdv_kernel<<<(unsigned)grid, DKV_THREADS, DKV_SMEM, s>>>(p);
        count_launch();
        if ((rc = check_launch("flash_attention_backward (dK, dV)")) != TLC_OK) break;
        // dQ
        if ((rc = encode_tiled(&p.m[2], k, d, S, d, bsz, bstr, 32, TB, K_SW)) != TLC_OK) break;
        if ((rc = encode_tiled(&p.m[3], v, d, S, d, bsz, bstr, 32, TB, K_SW)) != TLC_OK) break;
        if ((rc = encode_tiled(&p.m[4], k, d, S, d, bsz, bstr, 32, TB, M_SW)) != TLC_OK) break;
        p.kv0 = q;
        p.kv1 = dout;
        p.out0 = dq;
        p.out1 = nullptr;
        flash_bwd_dq_kernel<<<(unsigned)grid, DQ_THREADS, DQ_SMEM, s>>>(p);
        count_launch();
        rc = check_launch("flash_attention_backward (dQ)");
    } while (false);
    scratch_free(scratch, s);
    return rc;
}

}  // namespace tlc
