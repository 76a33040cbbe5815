// flash_attention forward (src/ops.cpp:1040-1137 of torchlite-cpp) on the
// tensor cores: TLC_MODE_TF32, head dim 32 <= d <= 64 with d % 4 == 0 and
// 16-byte aligned operands (the TMA tiles' requirements).
//
// One CTA per SM-resident block owns two 128-row query tiles of one head and
// walks the head's keys in blocks of 64, as the reference's tiles do (its
// 64 x 64 query tiles become 128-row tiles; the per-row arithmetic is the
// same online softmax).  10 warps:
//   warp 0      TMA producer: Q tiles once, then K and V blocks into two
//               rings (3 K stages, 2 V stages), 128-byte swizzle; V is loaded
//               key-major with 32-byte swizzle granules (the MN-major operand
//               of P.V).
//   warp 1      TMEM owner and MMA issuer (one thread): S_t = Q_t . K_j^T
//               (M = 128, N = 64, K = d) into a double-buffered TMEM score
//               tile per query tile, issued one key block ahead;
//               O_t,blk = P_t . V_j (M = 128, N = 64, K = 64 keys) into a TMEM
//               block accumulator per query tile.
//   warps 2-5   softmax for query tile 0, warps 6-9 for query tile 1; thread
//               = one query row (TMEM lane).  Per key block: tcgen05.ld the
//               score row, t = s * scale (masked to -inf past S), in log2
//               units; m_new = max(m, max t), corr = exp(m - m_new),
//               p = exp(t - m_new), l = l * corr + sum p (max and sum as
//               trees); p is written into the P tile in shared memory (the
//               K-major A operand of P.V, same swizzle as a TMA tile) after
//               the previous block's O_blk has been folded into registers
//               (o = o * corr + O_blk), so each P.V runs under the next
//               block's softmax.  At the end O = o * (1 / l), L = m + log(l).
// The two query tiles' softmax warps share the SM's exp units and alternate
// with each other's tensor-core work.  Every mbarrier wait is bounded (a
// %globaltimer deadline, an abort flag, the device error word), as in the
// GEMM kernel.
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
constexpr int KST = 3;       // K ring stages
constexpr int VST = 2;       // V ring stages
constexpr int Q_BYTES = FQ * FD * 4;   // 2 boxes [128 rows x 32 dims] of 16 KB
constexpr int K_BYTES = FK * FD * 4;   // 2 boxes [64 keys x 32 dims] of 8 KB
constexpr int V_BYTES = FK * FD * 4;   // 2 chunks [64 keys x 32 dims] of 8 KB (MN-major)
constexpr int P_BYTES = FQ * FK * 4;   // 2 blocks [128 rows x 32 keys] of 16 KB
constexpr int OFF_K = NQ * Q_BYTES;
constexpr int OFF_V = OFF_K + KST * K_BYTES;
constexpr int OFF_P = OFF_V + VST * V_BYTES;
constexpr int OFF_BAR = OFF_P + NQ * P_BYTES;
constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers + 1 KB alignment slack
constexpr int THREADS = 64 + NQ * 128;
constexpr int TMEM_COLS = 512;  // S[t][2] at t*128 + b*64, O_blk[t] at 256 + t*64
static_assert(SMEM <= 232448, "shared memory per CTA");

struct FtParams {
    CUtensorMap tmQ, tmK, tmV;
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

// Waits like wait_bounded, for a whole warp: lane 0 polls, the warp follows.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          const FtParams& p, int site) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = wait_bounded(bar, parity, abort_flag, p.timeout_ns, p.err, site);
    return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

__global__ void __launch_bounds__(THREADS, 1) flash_tc_kernel(const __grid_constant__ FtParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* q_full = bars;                  // [1]
    uint64_t* k_full = q_full + 1;            // [KST]
    uint64_t* k_empty = k_full + KST;         // [KST]
    uint64_t* v_full = k_empty + KST;         // [VST]
    uint64_t* v_empty = v_full + VST;         // [VST]
    uint64_t* s_full = v_empty + VST;         // [NQ][2]
    uint64_t* s_empty = s_full + 2 * NQ;      // [NQ][2]
    uint64_t* p_full = s_empty + 2 * NQ;      // [NQ]
    uint64_t* o_full = p_full + NQ;           // [NQ]
    uint64_t* o_empty = o_full + NQ;          // [NQ]
    uint64_t* drain = o_empty + NQ;           // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x / p.tiles;
    const int q0 = (blockIdx.x - head * p.tiles) * (NQ * FQ);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < KST; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VST; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int t = 0; t < NQ; ++t) {
            for (int b = 0; b < 2; ++b) {
                mbar_init(&s_full[2 * t + b], 1);
                mbar_init(&s_empty[2 * t + b], 4);  // one arrival per softmax warp
            }
            mbar_init(&p_full[t], 4);
            mbar_init(&o_full[t], 1);
            mbar_init(&o_empty[t], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 0 && lane == 0) {
        prefetch_map(&p.tmQ);
        prefetch_map(&p.tmK);
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
        if (lane == 0) {
            const uint32_t qb = smem_u32(q_full);
            mbar_expect_tx(q_full, NQ * Q_BYTES);
            for (int t = 0; t < NQ; ++t)
                for (int c = 0; c < FD / 32; ++c)
                    tma_load_5d<1>(smem + t * Q_BYTES + c * (Q_BYTES / 2), &p.tmQ, qb, 32 * c,
                                   q0 + t * FQ, head, 0, 0);
            uint32_t pend_k = 0, par_k = 0, pend_v = 0, par_v = 0;
            bool ok = true;
            for (int j = 0; ok && j < p.nk; ++j) {
                const int ks = j % KST, vs = j % VST;
                const uint32_t kph = (uint32_t)(j / KST) & 1u, vph = (uint32_t)(j / VST) & 1u;
                if (!wait_bounded(&k_empty[ks], kph ^ 1u, abort_flag, p.timeout_ns, p.err, 21)) {
                    ok = false;
                    break;
                }
                pend_k &= ~(1u << ks);
                mbar_expect_tx(&k_full[ks], K_BYTES);
                for (int c = 0; c < FD / 32; ++c)
                    tma_load_5d<1>(smem + OFF_K + ks * K_BYTES + c * (K_BYTES / 2), &p.tmK,
                                   smem_u32(&k_full[ks]), 32 * c, j * FK, head, 0, 0);
                pend_k |= 1u << ks;
                par_k = (par_k & ~(1u << ks)) | (kph << ks);
                if (!wait_bounded(&v_empty[vs], vph ^ 1u, abort_flag, p.timeout_ns, p.err, 22)) {
                    ok = false;
                    break;
                }
                pend_v &= ~(1u << vs);
                mbar_expect_tx(&v_full[vs], V_BYTES);
                for (int c = 0; c < FD / 32; ++c)
                    tma_load_5d<1>(smem + OFF_V + vs * V_BYTES + c * (V_BYTES / 2), &p.tmV,
                                   smem_u32(&v_full[vs]), 32 * c, j * FK, head, 0, 0);
                pend_v |= 1u << vs;
                par_v = (par_v & ~(1u << vs)) | (vph << vs);
            }
            if (!ok) {
                // loads still in flight land before the CTA frees anything
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(q_full, 0) && globaltimer() - t0 < p.timeout_ns) {
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
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // kind::tf32, fp32 D; N = 64 (bits 17-22, >> 3), M = 128 (bits 24-28, >> 4);
            // S: A (Q) and B (K) K-major; P.V: A (P) K-major, B (V) MN-major (bit 16).
            const uint32_t idesc_s = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(FK >> 3) << 17) |
                                     ((uint32_t)(FQ >> 4) << 24);
            const uint32_t idesc_pv = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) |
                                      ((uint32_t)(FD >> 3) << 17) | ((uint32_t)(FQ >> 4) << 24);
            const uint32_t sq = smem_u32(smem), sk = smem_u32(smem + OFF_K),
                           sv = smem_u32(smem + OFF_V), sp = smem_u32(smem + OFF_P);
            bool ok = wait_bounded(q_full, 0, abort_flag, p.timeout_ns, p.err, 23);
            bool issued = false;
            tc_fence_after();
            // S_t(j) = Q_t . K_j^T into S buffer (t, j & 1): 8 MMAs of K = 8 over d = 64
            auto issue_s = [&](int t, int j) -> bool {
                const int b = j & 1;
                if (!wait_bounded(&s_empty[2 * t + b], ((uint32_t)(j >> 1) & 1u) ^ 1u, abort_flag,
                                  p.timeout_ns, p.err, 24))
                    return false;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(t * 128 + b * 64);
                const uint32_t qa = sq + t * Q_BYTES, ka = sk + (j % KST) * K_BYTES;
#pragma unroll
                for (int s = 0; s < FD / 8; ++s) {
                    const uint64_t ad = smem_desc(qa + (s >> 2) * (Q_BYTES / 2) + (s & 3) * 32, 16, 1024, kSw128);
                    const uint64_t bd = smem_desc(ka + (s >> 2) * (K_BYTES / 2) + (s & 3) * 32, 16, 1024, kSw128);
                    umma_tf32<1>(d, ad, bd, idesc_s, s > 0 ? 1u : 0u);
                }
                umma_commit<1>(smem_u32(&s_full[2 * t + b]));
                issued = true;
                return true;
            };
            // O_blk_t = P_t . V_j: 8 MMAs of K = 8 over the 64 keys
            auto issue_pv = [&](int t, int j) -> bool {
                if (!wait_bounded(&p_full[t], (uint32_t)j & 1u, abort_flag, p.timeout_ns, p.err, 25))
                    return false;
                if (!wait_bounded(&o_empty[t], ((uint32_t)j & 1u) ^ 1u, abort_flag, p.timeout_ns, p.err, 26))
                    return false;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(256 + t * 64);
                const uint32_t pa = sp + t * P_BYTES, va = sv + (j % VST) * V_BYTES;
#pragma unroll
                for (int s = 0; s < FK / 8; ++s) {
                    const uint64_t ad = smem_desc(pa + (s >> 2) * (P_BYTES / 2) + (s & 3) * 32, 16, 1024, kSw128);
                    const uint64_t bd = smem_desc(va + s * 1024, V_BYTES / 2, 512, kSw128Atom32);
                    umma_tf32<1>(d, ad, bd, idesc_pv, s > 0 ? 1u : 0u);
                }
                umma_commit<1>(smem_u32(&o_full[t]));
                issued = true;
                return true;
            };
            if (ok) ok = wait_bounded(&k_full[0], 0, abort_flag, p.timeout_ns, p.err, 27);
            if (ok) tc_fence_after();
            for (int t = 0; ok && t < NQ; ++t) ok = issue_s(t, 0);
            if (ok) umma_commit<1>(smem_u32(&k_empty[0]));
            for (int j = 0; ok && j < p.nk; ++j) {
                const bool more = j + 1 < p.nk;
                if (more) {
                    const int ks = (j + 1) % KST;
                    ok = wait_bounded(&k_full[ks], (uint32_t)((j + 1) / KST) & 1u, abort_flag,
                                      p.timeout_ns, p.err, 28);
                    if (ok) ok = issue_s(0, j + 1);
                }
                if (ok) ok = wait_bounded(&v_full[j % VST], (uint32_t)(j / VST) & 1u, abort_flag,
                                          p.timeout_ns, p.err, 29);
                if (ok) ok = issue_pv(0, j);
                if (ok && more) {
                    ok = issue_s(1, j + 1);
                    if (ok) umma_commit<1>(smem_u32(&k_empty[(j + 1) % KST]));
                }
                if (ok) ok = issue_pv(1, j);
                if (ok) umma_commit<1>(smem_u32(&v_empty[j % VST]));
            }
            if (!ok && issued) {
                umma_commit<1>(smem_u32(drain));
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < p.timeout_ns) {
                }
            }
        }
    } else {
        // ---------------- softmax (warps 2-5: tile 0, 6-9: tile 1) ----------------
        // Scores are kept in log2 units (u = s * scale * log2 e, so exp(t - m) =
        // exp2(u - m2)).  O_blk of block j is folded into o while block j + 1's
        // probabilities are computed, so P.V(j) runs under softmax(j + 1).
        const int t = (warp - 2) >> 2;
        const int quarter = warp & 3;  // the TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane;
        const int row = q0 + t * FQ + r;
        const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
        uint8_t* prow = smem + OFF_P + t * P_BYTES + r * 128;
        const int sw = r & 7;
        const float sl2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
        float o[FD];
#pragma unroll
        for (int c = 0; c < FD; ++c) o[c] = 0.0f;
        float m2 = -INFINITY, l = 0.0f, corr_prev = 0.0f;
        bool ok = true;
        // o = o * corr + O_blk of the block whose P.V completes with parity `par`
        auto fold_block = [&](uint32_t par, bool release) -> bool {
            if (!warp_wait(&o_full[t], par, abort_flag, p, 31)) return false;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < FD / 16; ++h) {
                uint32_t ob[16];
                tmem_ld16(lane_base + (uint32_t)(256 + t * 64 + 16 * h), ob);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    o[16 * h + c] = fmaf(o[16 * h + c], corr_prev, __uint_as_float(ob[c]));
            }
            if (release) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_empty[t]);
            }
            return true;
        };
        for (int j = 0; j < p.nk; ++j) {
            const int b = j & 1;
            ok = warp_wait(&s_full[2 * t + b], (uint32_t)(j >> 1) & 1u, abort_flag, p, 30);
            if (!ok) break;
            tc_fence_after();
            float u[FK];
            {
                uint32_t s0[32], s1[32];
                tmem_ld32(lane_base + (uint32_t)(t * 128 + b * 64), s0);
                tmem_ld32(lane_base + (uint32_t)(t * 128 + b * 64 + 32), s1);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    u[c] = __fmul_rn(__uint_as_float(s0[c]), sl2);
                    u[32 + c] = __fmul_rn(__uint_as_float(s1[c]), sl2);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[2 * t + b]);
            const int valid = p.S - j * FK;
            if (valid < FK) {  // the tail block: keys past S take no weight
#pragma unroll
                for (int c = 0; c < FK; ++c)
                    if (c >= valid) u[c] = -INFINITY;
            }
            // row max and sum as trees (max is exact in any order)
            float mx[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) mx[c] = fmaxf(fmaxf(u[c], u[c + 16]), fmaxf(u[c + 32], u[c + 48]));
#pragma unroll
            for (int w = 8; w > 0; w >>= 1)
#pragma unroll
                for (int c = 0; c < w; ++c) mx[c] = fmaxf(mx[c], mx[c + w]);
            const float m_new = fmaxf(m2, mx[0]);
            const float corr = exp2f(__fsub_rn(m2, m_new));
#pragma unroll
            for (int c = 0; c < FK; ++c) u[c] = exp2f(__fsub_rn(u[c], m_new));
            float sm[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) sm[c] = (u[c] + u[c + 16]) + (u[c + 32] + u[c + 48]);
#pragma unroll
            for (int w = 8; w > 0; w >>= 1)
#pragma unroll
                for (int c = 0; c < w; ++c) sm[c] += sm[c + w];
            // fold the previous block (its P.V ran during this block's softmax);
            // that also frees the P tile for this block's probabilities
            if (j > 0) {
                ok = fold_block((uint32_t)(j - 1) & 1u, true);
                if (!ok) break;
            }
            l = fmaf(l, corr, sm[0]);
            m2 = m_new;
            corr_prev = corr;
            // P row into the swizzled K-major tile: keys c..c+3 are 16-byte granule
            // (c % 32) / 4 of the row's 128-byte line in block c / 32
#pragma unroll
            for (int c = 0; c < FK; c += 4) {
                uint8_t* dst = prow + (c >> 5) * (P_BYTES / 2) + ((((c & 31) >> 2) ^ sw) << 4);
                *reinterpret_cast<float4*>(dst) = make_float4(u[c], u[c + 1], u[c + 2], u[c + 3]);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        if (ok) ok = fold_block((uint32_t)(p.nk - 1) & 1u, false);
        if (ok && row < p.S) {
            const float inv = __fdiv_rn(1.0f, l);
            float* orow = p.O + ((int64_t)head * p.S + row) * p.d;
            if (p.vec_o) {
#pragma unroll
                for (int c = 0; c < FD; c += 4)
                    if (c < p.d)
                        *reinterpret_cast<float4*>(orow + c) =
                            make_float4(__fmul_rn(o[c], inv), __fmul_rn(o[c + 1], inv),
                                        __fmul_rn(o[c + 2], inv), __fmul_rn(o[c + 3], inv));
            } else {
#pragma unroll
                for (int c = 0; c < FD; ++c)
                    if (c < p.d) orow[c] = __fmul_rn(o[c], inv);
            }
            // L = m + log(l) with m = m2 * ln 2 back in the scores' units
            if (p.L) p.L[(int64_t)head * p.S + row] = __fadd_rn(__fmul_rn(m2, 0.6931471805599453f), logf(l));
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
    static bool configured[64] = {};
    int dev = 0;
    TLC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(TLC_ERR_UNSUPPORTED, "device index above 63");
    if (!configured[dev]) {
        TLC_CUDA_TRY(cudaFuncSetAttribute(flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        configured[dev] = true;
    }
    if (heads > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "flash_attention: too many heads");
    FtParams p;
    memset(&p, 0, sizeof(p));
    const int64_t bsz[kMaxBatchDims] = {heads, 1, 1};
    const int64_t bstr[kMaxBatchDims] = {(int64_t)S * d, 0, 0};
    TLC_TRY(encode_tiled(&p.tmQ, q, d, S, d, bsz, bstr, 32, FQ, CU_TENSOR_MAP_SWIZZLE_128B));
    TLC_TRY(encode_tiled(&p.tmK, k, d, S, d, bsz, bstr, 32, FK, CU_TENSOR_MAP_SWIZZLE_128B));
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
