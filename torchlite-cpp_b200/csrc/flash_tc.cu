// flash_attention forward (src/ops.cpp:1040-1137 of torchlite-cpp) on the
// tensor cores: TLC_MODE_TF32, head dim 32 <= d <= 64 with d % 4 == 0 and
// 16-byte aligned operands (the TMA tiles' requirements).
//
// One CTA per SM owns two 128-row query tiles of one head and walks the
// head's keys in blocks of 64, as the reference's tiles do (its 64 x 64
// query tiles become 128-row tiles; the per-row arithmetic is the same online
// softmax).  21 warps:
//   warp 0      TMA producer: the two tiles' Q rows once (128-byte swizzle,
//               the score MMAs' A operand), then K and V blocks into two
//               rings (4 K stages, 3 V stages); V is loaded key-major with
//               32-byte swizzle granules (the MN-major operand of P.V).
//   warp 1      TMEM owner; score issuer of query tile 0, warp 18 of tile 1:
//               S_t = Q_t . K_j^T (M = 128, N = 64, K = d) into one of three
//               TMEM score buffers per tile, as far ahead as the K ring and
//               the buffers allow.
//   warps 19-20 P.V issuers of tiles 0 and 1: O_t += P_t . V_j (M = 128,
//               N = 64, K = 64 keys) into a TMEM accumulator, with A = P read
//               from tensor memory.  One issuing thread turns over an N = 64
//               MMA only about once per 130 cycles; separate score and P.V
//               streams per tile overlap.
//   warps 2-9   softmax for query tile 0, warps 10-17 for query tile 1: two
//               warps per TMEM lane quarter, thread = (query row, half of the
//               keys).  Per key block: tcgen05.ld the half row of scores,
//               t = s * scale (masked to -inf past S) in log2 units; the two
//               halves exchange their maxima (shared memory, 64-thread named
//               barrier); p = exp(t - m), l = l * corr + sum p (partial per
//               half); p is stored over the scores in TMEM (tcgen05.st), where
//               P.V reads it, and P.V accumulates O in TMEM: no shared-memory
//               round trip for P and no per-block wait on P.V.  The running
//               maximum m moves only when a block's maximum exceeds it by more
//               than a factor 2^8 (conditional rescaling, as FlashAttention-4
//               does); then O and l are rescaled by exp(m_old - m_new) in
//               place.  At the end O = o * (1 / l), L = m + log(l).
// TMEM per query tile (256 of the 512 columns): three score / probability
// buffers of 64, O 64.  A buffer is reused three blocks later, after the P.V
// issuer's commit for the P.V that read it (measured: three buffers with
// separate score and P.V issuers 0.467 ms against 0.478 for two buffers and
// one issuer per tile on 192 heads x 2048 x 64; either change alone gained
// nothing).  Every mbarrier wait is bounded (a %globaltimer deadline, an
// abort flag, the device error word), as in the GEMM kernel, and the
// named-barrier syncs are taken the same number of times by both warps of a
// pair on every path.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace tlc {
namespace {

constexpr int FQ = 128;      // query rows per tile (TMEM lanes)
constexpr int FK = 64;       // keys per block
constexpr int FD = 64;       // head dim of the tiles (d <= 64, zero-filled)
constexpr int NQ = 2;        // query tiles per CTA
constexpr int KST = 4;       // K ring stages
constexpr int VST = 3;       // V ring stages
constexpr int SPB = 3;       // score / probability buffers per query tile in TMEM
constexpr int K_BYTES = FK * FD * 4;   // 2 boxes [64 keys x 32 dims] of 8 KB
constexpr int V_BYTES = FK * FD * 4;   // 2 chunks [64 keys x 32 dims] of 8 KB (MN-major)
constexpr int Q_BYTES = FQ * FD * 4;  // a tile's Q rows: 2 boxes [128 rows x 32 dims] of 16 KB
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + NQ * Q_BYTES;
constexpr int OFF_V = OFF_K + KST * K_BYTES;
constexpr int OFF_X = OFF_V + VST * V_BYTES;  // row-max exchange: [2 parities][NQ][2 halves][128]
constexpr int X_BYTES = 2 * NQ * 2 * FQ * 4;
constexpr int OFF_BAR = OFF_X + X_BYTES;
constexpr int BAR_BYTES = 8 * (NQ + 2 * KST + 2 * VST + 3 * SPB * NQ + 3 * NQ) + 8;  // + TMEM slot, abort flag
constexpr int SMEM = OFF_BAR + 512 + 1024;  // barriers + 1 KB alignment slack
static_assert(BAR_BYTES <= 512, "barrier area");
constexpr int SM_WARPS = 8;                 // softmax warps per query tile: 2 per TMEM lane quarter
constexpr int MMA2_WARP = 2 + NQ * SM_WARPS;  // the MMA warp of query tile 1 (tile 0: warp 1)
constexpr int THREADS = 32 * (MMA2_WARP + 3);  // + the P.V issuers of tiles 0, 1
// TMEM: tile t owns columns t*256 ..: S/P buffer b at t*256 + b*64, O at t*256 + 192
constexpr int TMEM_COLS = 512;
constexpr int TILE_COLS = 256, SP_COL = 0, O_COL = SP_COL + SPB * FK;
static_assert(O_COL + FD <= TILE_COLS, "TMEM columns of a query tile");
// The running row maximum (log2 units) moves only when a block's maximum
// exceeds it by more than this; probabilities stay <= 2^8 in between.
constexpr float kRescaleLog2 = 8.0f;
// How long a waiting thread may sleep per poll (it wakes when the phase
// completes): producer, MMA issuers, softmax warps.
constexpr uint32_t kSleepNs = 100000, kSleepMma = 100000, kSleepSm = 100000;
static_assert(SMEM <= 232448, "shared memory per CTA");

struct FtParams {
    CUtensorMap tmK, tmV, tmQ;
    float* O;
    float* L;
    int S, d;
    int tiles;  // query tile pairs per head
    int nk;     // key blocks
    float scale;
    int vec_o;  // float4 stores of O
    uint64_t timeout_ns;
    int* err;
};

__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Waits like wait_bounded, for a whole warp: every lane polls (measured
// faster than lane 0 polling and sharing its result with a shuffle).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          const FtParams& p, int site) {
    return warp_wait_bounded(bar, parity, abort_flag, p.timeout_ns, p.err, site, kSleepSm);
}

__global__ void __launch_bounds__(THREADS, 1) flash_tc_kernel(const __grid_constant__ FtParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* a_full = bars;                  // [NQ]  the tile's Q rows in shared memory
    uint64_t* k_full = a_full + NQ;           // [KST]
    uint64_t* k_empty = k_full + KST;         // [KST]
    uint64_t* v_full = k_empty + KST;         // [VST]
    uint64_t* v_empty = v_full + VST;         // [VST]
    uint64_t* s_full = v_empty + VST;         // [NQ][SPB]
    uint64_t* s_empty = s_full + SPB * NQ;    // [NQ][SPB]
    // p_full is per buffer: a softmax warp may finish block j + 1 before the
    // MMA thread has looked at block j, and a parity wait tells apart only
    // two consecutive phases of one barrier
    uint64_t* p_full = s_empty + SPB * NQ;    // [NQ][SPB]
    // o_last completes once, after the tile's last P.V, so the softmax's
    // final wait needs no parity reasoning.  (Waiting for the last phases of a
    // per-block barrier by parity is ambiguous once the last P.V has finished
    // before the wait starts: a parity wait tells apart only the current and
    // the previous phase.)
    uint64_t* o_last = p_full + SPB * NQ;     // [NQ]
    uint64_t* drain = o_last + NQ;            // [2][NQ]: S, P.V issuers
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2 * NQ);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x / p.tiles;
    const int q0 = (blockIdx.x - head * p.tiles) * (NQ * FQ);

    if (threadIdx.x == 0) {
        for (int t = 0; t < NQ; ++t) mbar_init(&a_full[t], 1);
        for (int s = 0; s < KST; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], NQ);  // a commit from each tile's score issuer
        }
        for (int s = 0; s < VST; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], NQ);
        }
        for (int t = 0; t < NQ; ++t) {
            for (int b = 0; b < SPB; ++b) {
                mbar_init(&s_full[SPB * t + b], 1);
                mbar_init(&s_empty[SPB * t + b], 1);  // committed after the P.V that read it
                mbar_init(&p_full[SPB * t + b], SM_WARPS);
            }
            mbar_init(&o_last[t], 1);
        }
        for (int t = 0; t < 2 * NQ; ++t) mbar_init(&drain[t], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 0 && lane == 0) {
        prefetch_map(&p.tmK);
        prefetch_map(&p.tmQ);
        prefetch_map(&p.tmV);
    }
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
        // The warp waits together; one elected lane issues (as in the GEMM).
        {
            uint32_t pend_k = 0, par_k = 0, pend_v = 0, par_v = 0;
            bool ok = true;
            if (elect_one()) {
                for (int t = 0; t < NQ; ++t) {
                    mbar_expect_tx(&a_full[t], Q_BYTES);
                    for (int c = 0; c < FD / 32; ++c)
                        tma_load_5d<1>(smem + OFF_Q + t * Q_BYTES + c * (Q_BYTES / 2), &p.tmQ,
                                       smem_u32(&a_full[t]), 32 * c, q0 + t * FQ, head, 0, 0);
                }
            }
            __syncwarp();
            for (int j = 0; ok && j < p.nk; ++j) {
                const int ks = j % KST, vs = j % VST;
                const uint32_t kph = (uint32_t)(j / KST) & 1u, vph = (uint32_t)(j / VST) & 1u;
                if (!warp_wait_bounded(&k_empty[ks], kph ^ 1u, abort_flag, p.timeout_ns, p.err, 21, kSleepNs)) {
                    ok = false;
                    break;
                }
                pend_k &= ~(1u << ks);
                if (elect_one()) {
                    mbar_expect_tx(&k_full[ks], K_BYTES);
                    for (int c = 0; c < FD / 32; ++c)
                        tma_load_5d<1>(smem + OFF_K + ks * K_BYTES + c * (K_BYTES / 2), &p.tmK,
                                       smem_u32(&k_full[ks]), 32 * c, j * FK, head, 0, 0);
                }
                pend_k |= 1u << ks;
                par_k = (par_k & ~(1u << ks)) | (kph << ks);
                if (!warp_wait_bounded(&v_empty[vs], vph ^ 1u, abort_flag, p.timeout_ns, p.err, 22, kSleepNs)) {
                    ok = false;
                    break;
                }
                pend_v &= ~(1u << vs);
                if (elect_one()) {
                    mbar_expect_tx(&v_full[vs], V_BYTES);
                    for (int c = 0; c < FD / 32; ++c)
                        tma_load_5d<1>(smem + OFF_V + vs * V_BYTES + c * (V_BYTES / 2), &p.tmV,
                                       smem_u32(&v_full[vs]), 32 * c, j * FK, head, 0, 0);
                }
                pend_v |= 1u << vs;
                par_v = (par_v & ~(1u << vs)) | (vph << vs);
            }
            if (!ok && lane == 0) {
                // loads still in flight land before the CTA frees anything
                for (int t = 0; t < NQ; ++t) {
                    const uint64_t t1 = globaltimer();
                    while (!mbar_try_wait(&a_full[t], 0) && globaltimer() - t1 < p.timeout_ns) {
                    }
                }
                for (int s = 0; s < KST; ++s)
                    if (pend_k & (1u << s)) {
                        const uint64_t t1 = globaltimer();
                        while (!mbar_try_wait(&k_full[s], (par_k >> s) & 1u) &&
                               globaltimer() - t1 < p.timeout_ns) {
                        }
                    }
                for (int s = 0; s < VST; ++s)
                    if (pend_v & (1u << s)) {
                        const uint64_t t1 = globaltimer();
                        while (!mbar_try_wait(&v_full[s], (par_v >> s) & 1u) &&
                               globaltimer() - t1 < p.timeout_ns) {
                        }
                    }
            }
        }
    } else if (warp == 1 || warp >= MMA2_WARP) {
        // ---------------- MMA issuers: scores and P.V, one warp each per tile ----------------
        // Each tile's chain (S, softmax, P, P.V) runs at its own pace;
        // the tiles share only the K and V rings, whose empty barriers take a
        // commit from both tiles' issuers.
        const int mt = (warp == 1 || warp == MMA2_WARP + 1) ? 0 : 1;
        const bool pv_role = warp > MMA2_WARP;
        // The whole warp runs the chain, every lane polling the barriers; one
        // elected lane issues each MMA and commit (a lone lane in a divergent
        // branch leaves the tensor pipe idle after each commit: measured).
        {
            // kind::tf32, fp32 D; N = 64 (bits 17-22, >> 3), M = 128 (bits 24-28, >> 4);
            // S: A (Q) and B (K) K-major; P.V: A (P, in TMEM) K-major, B (V) MN-major (bit 16).
            const uint32_t idesc_s = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(FK >> 3) << 17) |
                                     ((uint32_t)(FQ >> 4) << 24);
            const uint32_t idesc_pv = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) |
                                      ((uint32_t)(FD >> 3) << 17) | ((uint32_t)(FQ >> 4) << 24);
            // descriptors of K stage 0, V stage 0; any other stage or k-step only
            // moves the start-address field (address >> 4)
            const uint64_t k_desc = smem_desc(smem_u32(smem + OFF_K), 16, 1024, kSw128);
            const uint64_t q_desc = smem_desc(smem_u32(smem + OFF_Q), 16, 1024, kSw128);
            const uint64_t v_desc = smem_desc(smem_u32(smem + OFF_V), V_BYTES / 2, 512, kSw128Atom32);
            // the score issuers need the tile's Q rows
            bool ok =
                pv_role || warp_wait_bounded(&a_full[mt], 0, abort_flag, p.timeout_ns, p.err, 23, kSleepMma);
            bool issued = false;
            tc_fence_after();
            // S_t(j) = Q_t . K_j^T into buffer (t, j % SPB): 8 MMAs of K = 8 over d = 64,
            // once the P.V that last read that buffer is done
            auto issue_s = [&](int t, int j) -> bool {
                const int b = j % SPB;
                if (!warp_wait_bounded(&s_empty[SPB * t + b], ((uint32_t)(j / SPB) & 1u) ^ 1u, abort_flag,
                                       p.timeout_ns, p.err, 24, kSleepMma))
                    return false;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(t * TILE_COLS + SP_COL + b * FK);
                const uint64_t qd = q_desc + (uint32_t)((t * Q_BYTES) >> 4);
                const uint64_t kd = k_desc + (uint32_t)(((j % KST) * K_BYTES) >> 4);
                // A = Q from shared memory (K-major, two 16 KB boxes of 32 dims)
#pragma unroll
                for (int s = 0; s < FD / 8; ++s)
                    if (elect_one())
                    umma_tf32<1>(d, qd + (uint32_t)(((s >> 2) * (Q_BYTES / 2) + (s & 3) * 32) >> 4),
                                 kd + (uint32_t)(((s >> 2) * (K_BYTES / 2) + (s & 3) * 32) >> 4), idesc_s,
                                 s > 0 ? 1u : 0u);
                if (elect_one()) umma_commit<1>(smem_u32(&s_full[SPB * t + b]));
                issued = true;
                return true;
            };
            // O_t += P_t . V_j: A = the probabilities the softmax wrote over the
            // scores in TMEM, B = V from shared memory; 8 MMAs of K = 8 keys
            // (the first block's first MMA starts O from zero)
            auto issue_pv = [&](int t, int j) -> bool {
                const int b = j % SPB;
                if (!warp_wait_bounded(&p_full[SPB * t + b], (uint32_t)(j / SPB) & 1u, abort_flag,
                                       p.timeout_ns, p.err, 25, kSleepMma))
                    return false;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(t * TILE_COLS + O_COL);
                const uint32_t pa = tmem_base + (uint32_t)(t * TILE_COLS + SP_COL + b * FK);
                const uint64_t vd = v_desc + (uint32_t)(((j % VST) * V_BYTES) >> 4);
#pragma unroll
                for (int s = 0; s < FK / 8; ++s)
                    if (elect_one())
                    umma_tf32_tmem_a(d, pa + 8 * s, vd + (uint32_t)((s * 1024) >> 4), idesc_pv,
                                     (j > 0 || s > 0) ? 1u : 0u);
                if (elect_one()) umma_commit<1>(smem_u32(&s_empty[SPB * t + b]));
                issued = true;
                return true;
            };
            if (!pv_role) {
                // scores, as far ahead as the K ring and the three buffers allow
                for (int j = 0; ok && j < p.nk; ++j) {
                    const int ks = j % KST;
                    ok = warp_wait_bounded(&k_full[ks], (uint32_t)(j / KST) & 1u, abort_flag, p.timeout_ns,
                                           p.err, 28, kSleepMma);
                    if (ok) ok = issue_s(mt, j);
                    if (ok && elect_one()) umma_commit<1>(smem_u32(&k_empty[ks]));
                }
            } else {
                for (int j = 0; ok && j < p.nk; ++j) {
                    ok = warp_wait_bounded(&v_full[j % VST], (uint32_t)(j / VST) & 1u, abort_flag,
                                           p.timeout_ns, p.err, 29, kSleepMma);
                    if (ok) ok = issue_pv(mt, j);
                    if (ok && elect_one()) umma_commit<1>(smem_u32(&v_empty[j % VST]));
                }
                if (ok && elect_one()) umma_commit<1>(smem_u32(&o_last[mt]));
            }
            if (!ok && issued && elect_one()) {
                uint64_t* dr = &drain[mt + (pv_role ? NQ : 0)];
                umma_commit<1>(smem_u32(dr));
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(dr, 0) && globaltimer() - t0 < p.timeout_ns) {
                }
            }
            __syncwarp();
        }
    } else {
        // ---------------- softmax (warps 2-9: tile 0, 10-17: tile 1) ----------------
        // Two warps per TMEM lane quarter: thread (row r, half h) owns keys
        // 32h .. 32h + 31 of each score block and O columns 32h .. 32h + 31.
        // The halves of a row exchange their block maxima through shared
        // memory (a 64-thread named barrier per lane quarter); each keeps its
        // own partial row sum, added at the end.  Scores are kept in log2
        // units (u = s * scale * log2 e, so exp(t - m) = 2^(u - m2)).
        // O accumulates in TMEM across blocks.  The reference maximum m2
        // moves only when a block's maximum exceeds it by more than
        // kRescaleLog2; then (rarely, after the first blocks) this thread
        // waits for the previous P.V and rescales its O columns and l by
        // 2^(m2_old - m2_new) in place.  The sums are the reference's up to
        // that common factor, which the final O / l and L = m + log(l) cancel.
        const int wt = warp - 2;
        const int t = wt / SM_WARPS;
        const int h = (wt % SM_WARPS) >> 2;  // key / column half
        const int quarter = warp & 3;        // the TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane;
        const int row = q0 + t * FQ + r;
        const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const uint32_t o_addr = lane_base + (uint32_t)(t * TILE_COLS + O_COL + 32 * h);
        float* xchg = reinterpret_cast<float*>(smem + OFF_X);  // [par][t][h][row]
        const int bar_id = 1 + t * 4 + quarter;              // named barrier of the two halves
        const float sl2 = p.scale * 1.4426950408889634f;      // scale * log2(e)
        const bool fast = sl2 > 0.0f;  // max(s) * sl2 == max(s * sl2): one FFMA per probability
        float m2 = -INFINITY, l = 0.0f;
        bool ok = true;
        auto ex2 = [](float x) {
            float y;
            asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
            return y;
        };
        // Both warps of a row pair execute the same number of named-barrier
        // syncs whatever happens (a bar.sync has no time limit): after a
        // failed wait a warp stops waiting and computing but still takes
        // every sync, and each of its waits is bounded.
        for (int j = 0; j < p.nk; ++j) {
            const int b = j % SPB;
            const uint32_t sp_addr = lane_base + (uint32_t)(t * TILE_COLS + SP_COL + b * FK + 32 * h);
            if (ok) ok = warp_wait(&s_full[SPB * t + b], (uint32_t)(j / SPB) & 1u, abort_flag, p, 30);
            float u[32];
            if (ok) {
                tc_fence_after();
                uint32_t sv[32];
                tmem_ld32(sp_addr, sv);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c) u[c] = __uint_as_float(sv[c]);
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) u[c] = 0.0f;
            }
            const int valid = p.S - j * FK - 32 * h;  // keys of this half inside S
            const bool plain = fast && valid >= 32;
            if (!plain) {
                // general form: u = s * sl2, keys past S at -inf
#pragma unroll
                for (int c = 0; c < 32; ++c) u[c] = c < valid ? __fmul_rn(u[c], sl2) : -INFINITY;
            }
            float mx[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) mx[c] = fmaxf(fmaxf(u[c], u[c + 8]), fmaxf(u[c + 16], u[c + 24]));
#pragma unroll
            for (int w = 4; w > 0; w >>= 1)
#pragma unroll
                for (int c = 0; c < w; ++c) mx[c] = fmaxf(mx[c], mx[c + w]);
            const float mine = plain ? __fmul_rn(mx[0], sl2) : mx[0];
            // exchange buffers alternate by block parity: a half can write block
            // j + 1's maximum while the other still reads block j's
            float* xb = xchg + (((j & 1) * NQ + t) * 2) * FQ;
            xb[h * FQ + r] = mine;
            asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
            const float m_blk = fmaxf(mine, xb[(h ^ 1) * FQ + r]);
            // both halves of the row take the same decision from the same values
            const bool move = m_blk > m2 + kRescaleLog2;
            const float m_new = move ? m_blk : m2;
            const float corr = move ? ex2(m2 - m_new) : 1.0f;
            if (plain) {
#pragma unroll
                for (int c = 0; c < 32; ++c) u[c] = ex2(fmaf(u[c], sl2, -m_new));
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) u[c] = ex2(u[c] - m_new);
            }
            float sm[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) sm[c] = (u[c] + u[c + 8]) + (u[c + 16] + u[c + 24]);
#pragma unroll
            for (int w = 4; w > 0; w >>= 1)
#pragma unroll
                for (int c = 0; c < w; ++c) sm[c] += sm[c + w];
            l = fmaf(l, corr, sm[0]);
            m2 = m_new;
            // rescale O in TMEM where the maximum moved (not before the first
            // P.V, which starts O from zero): after the previous P.V is done
            // (the commit that frees its buffer), before this block's P.V is
            // issued (that waits for p_full)
            if (ok && j > 0 && __any_sync(0xffffffffu, move)) {
                ok = warp_wait(&s_empty[SPB * t + (j - 1) % SPB], (uint32_t)((j - 1) / SPB) & 1u, abort_flag,
                               p, 31);
                if (ok) {
                    tc_fence_after();
                    uint32_t ov[32];
                    tmem_ld32(o_addr, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__fmul_rn(__uint_as_float(ov[c]), corr));
                    tmem_st32(o_addr, ov);
                }
            }
            if (ok) {
                // the probabilities over this half's scores, in place in TMEM: the
                // A operand (lane = row, column = key) of P.V
                uint32_t pv[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) pv[c] = __float_as_uint(u[c]);
                tmem_st32(sp_addr, pv);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[SPB * t + b]);
            }
        }
        // O after the last P.V: o_last's only phase.  (In the loop, the
        // rescale's wait for block j - 1 on its buffer's s_empty is
        // unambiguous: block j's scores imply P.V of block j - 3 is done, so
        // that barrier is in the phase of P.V j - 1, and P.V j + 2 on the same
        // buffer cannot start before this warp's p_full arrival.)
        float o[32];
        if (ok) ok = warp_wait(&o_last[t], 0u, abort_flag, p, 32);
        if (ok) {
            tc_fence_after();
            uint32_t ov[32];
            tmem_ld32(o_addr, ov);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __uint_as_float(ov[c]);
        }
        // the row sum: this half's partial plus the other's
        float* xl = xchg + (t * 2) * FQ;  // parity-0 buffer; every max read is done
        asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
        xl[h * FQ + r] = l;
        asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
        const float lsum = l + xl[(h ^ 1) * FQ + r];
        if (ok && row < p.S) {
            const float inv = __fdiv_rn(1.0f, lsum);
            float* orow = p.O + ((int64_t)head * p.S + row) * p.d + 32 * h;
            const int dc = p.d - 32 * h;  // this half's columns inside d
            if (p.vec_o) {
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                    if (c < dc)
                        *reinterpret_cast<float4*>(orow + c) =
                            make_float4(__fmul_rn(o[c], inv), __fmul_rn(o[c + 1], inv),
                                        __fmul_rn(o[c + 2], inv), __fmul_rn(o[c + 3], inv));
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    if (c < dc) orow[c] = __fmul_rn(o[c], inv);
            }
            // L = m + log(l) with m = m2 * ln 2 back in the scores' units
            if (p.L && h == 0)
                p.L[(int64_t)head * p.S + row] = __fadd_rn(__fmul_rn(m2, 0.6931471805599453f), logf(lsum));
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

}  // namespace

bool flash_tc_supported(int d, const float* q, const float* k, const float* v) {
    return d >= 32 && d <= FD && d % 4 == 0 && al16(q) && al16(k) && al16(v);
}

int flash_forward_tc(const float* q, const float* k, const float* v, float* o, float* lse,
                     int64_t heads, int S, int d, float scale, cudaStream_t s) {
    static DeviceOnce once;
    TLC_TRY(smem_limit_once(once, flash_tc_kernel, SMEM));
    if (heads > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "flash_attention: too many heads");
    FtParams p;
    memset(&p, 0, sizeof(p));
    const int64_t bsz[kMaxBatchDims] = {heads, 1, 1};
    const int64_t bstr[kMaxBatchDims] = {(int64_t)S * d, 0, 0};
    TLC_TRY(encode_tiled(&p.tmK, k, d, S, d, bsz, bstr, 32, FK, CU_TENSOR_MAP_SWIZZLE_128B));
    TLC_TRY(encode_tiled(&p.tmQ, q, d, S, d, bsz, bstr, 32, FQ, CU_TENSOR_MAP_SWIZZLE_128B));
    TLC_TRY(encode_tiled(&p.tmV, v, d, S, d, bsz, bstr, 32, FK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    p.O = o;
    p.L = lse;
    p.S = S;
    p.d = d;
    p.tiles = (S + NQ * FQ - 1) / (NQ * FQ);
    p.nk = (S + FK - 1) / FK;
    p.scale = scale;
    p.vec_o = al16(o) ? 1 : 0;
    p.timeout_ns = 2000000000ull;
    TLC_TRY(tc_error_word(&p.err));
    const int64_t grid = (int64_t)p.tiles * heads;
    if (grid > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "flash_attention: too many tiles");
    flash_tc_kernel<<<(unsigned)grid, THREADS, SMEM, s>>>(p);
    count_launch();
    return check_launch("flash_attention (tensor cores)");
}

}  // namespace tlc
