// Tensor-core GEMM for TLC_MODE_TF32 and TLC_MODE_3XTF32 on sm_100a (tcgen05).
//
// Persistent, warp-specialised kernel; 10 warps per CTA:
//   warp 0      TMA producer: the warp waits for free stages together and one
//               elected lane streams A and B k-blocks (32 fp32 = 128 bytes of
//               k) into a ring of shared-memory stages with
//               cp.async.bulk.tensor (128-byte swizzle), completion tracked by
//               an mbarrier per stage (expect_tx bytes).
//   warp 1      TMEM allocation; in the leader CTA the whole warp runs the MMA
//               loop, every lane polling the stage barriers, and one elected
//               lane issues tcgen05.mma.kind::tf32 (K = 8 per instruction, 4
//               per k-block and product) into an fp32 accumulator in tensor
//               memory; tcgen05.commit from the same lane frees each stage and
//               publishes each finished accumulator.  (Issued by lane 0 alone
//               in a divergent branch, the same loop loses ~100-300 cycles of
//               tensor-pipe time at every commit: measured.)
//   warps 2-9   epilogue: tcgen05.ld the accumulator (two warps per TMEM lane
//               quarter, each thread half of one of the 128 rows), store fp32 C.
// The accumulator is double-buffered in TMEM, so the epilogue of one tile
// overlaps the main loop of the next.
//
// CTA pairs (CG = 2, the default for problems with more than 128 rows): two
// CTAs of a cluster share one M = 256 tcgen05.mma.cta_group::2.  Each CTA
// loads its own 128 rows of A and its own half of the tile's B columns, so a
// CTA moves 32 KB per k-block instead of 48 KB for the same 128 x 256 x 32 of
// work, and six stages fit instead of four.  Both CTAs' TMA loads complete on
// the leader CTA's full barrier; the leader issues the MMAs (reading both
// CTAs' shared memory, writing both CTAs' TMEM) and commits each completion
// to a barrier in each CTA with a unicast commit; each CTA's epilogue drains
// its own TMEM rows and signals the leader.  No load uses cluster multicast:
// every CTA fetches its own tiles.
//
// Operand layouts are read in place: A may be K-major (row-major [M,K]) or
// M-major (a transposed view, storage [K,M]); B may be N-major (row-major
// [K,N]) or K-major (a transposed view, storage [N,K], the X.W^T of Linear).
// The instruction descriptor's per-operand major bits select the layout; an
// MN-major tile is held as 32-element-wide column chunks with the 128-byte
// swizzle of 32-byte granules (atoms of 4 k-rows x 128 bytes), the one
// shared-memory layout MN-major TF32 operands accept.  When the MN extent is a
// multiple of 32 (and there are at most two batch dims), the tensor map has a
// chunk dimension and one TMA instruction loads all chunks of a k-block;
// otherwise each chunk is its own load.  Batch dims (up to 3,
// broadcast dims with stride 0) are extra dimensions of the 5-D tensor maps,
// so ragged M, N and K tails are zero-filled by TMA per batch entry and never
// read a neighbouring matrix.
//
// 3xTF32 (Ootomo & Yokota, "Recovering single precision accuracy from Tensor
// Cores while surpassing the FP32 theoretical peak performance", 2022): each
// operand x is split as hi + lo.  kind::tf32 reads an fp32 input truncated to
// TF32 (measured), so hi is the operand itself and a pre-pass writes only
// lo = x - trunc_tf32(x) (exact in fp32); the allocation-free entry point
// splits as hi = round_to_tf32(x), lo = x - hi into its fixed array instead.
// A stage holds hi and lo tiles of A and B for a k-block, and the
// MMA thread issues lo(A).hi(B), hi(A).lo(B) and hi(A).hi(B) from them, so
// each tile is loaded once for three products (12 MMAs per stage handshake).
// Because the tensor cores' fp32 accumulation error grows with the chain
// length, 3xTF32 accumulates each 256-wide k chunk from zero in its own
// (double-buffered) TMEM accumulator and the epilogue adds the chunk results
// in fp32 round-to-nearest registers: 8 epilogue warps, two per TMEM lane
// quarter, each holding half of a 256-column row.
//
// Every mbarrier wait is bounded by a %globaltimer deadline; on expiry the
// waiting thread raises a CTA-wide abort flag and a device error word, every
// role leaves its loop, in-flight TMA copies and MMAs are drained (again with
// a bound), the TMEM is freed, and the host reports TLC_ERR_TIMEOUT.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace tlc {

__device__ int g_tc_error = 0;  // first failing wait site of any tensor-core launch

namespace {

constexpr int BM = 128;        // rows of A (and of D) per CTA
constexpr int BK = 32;         // k per stage: 32 fp32 = one 128-byte swizzle row
constexpr int UMMA_K = 8;      // k per tcgen05.mma.kind::tf32
// A waiting thread sleeps up to this long per poll (it wakes when the phase
// completes), so idle waiters leave their schedulers' issue slots to the MMA
// and TMA threads.
constexpr uint32_t kGemmSleepNs = 20000;

struct TcParams {
    CUtensorMap tmA[2];  // [0] A (TF32) or hi(A) (3xTF32); [1] lo(A)
    CUtensorMap tmB[2];
    CUtensorMap tmC;     // C {N, M, batch...}, 32 x 32 boxes, 128-byte swizzle (if tma_c)
    float* C;
    int64_t c_rs;
    int64_t cbs[kMaxBatchDims];
    int bsz[kMaxBatchDims];
    int a_bc[kMaxBatchDims];  // 1: A indexes this batch dim, 0: broadcast (coordinate 0)
    int b_bc[kMaxBatchDims];
    int nb;
    int M, N, K;
    int m_tiles, n_tiles;
    int64_t num_tiles;
    int k_blocks;
    int chunk_kb;     // k-blocks per accumulation chunk (== k_blocks: one chunk)
    int num_chunks;
    int a_mn, b_mn;   // 1: operand is MN-major in memory
    int a_chunked, b_chunked;  // 1: MN-major map with a chunk dim: one load per k-block
    int vec_c;        // float4 stores allowed
    int tma_c;        // TF32: C written by TMA stores from the epilogue's staging squares
    int m64;          // CONV: M = 64 MMAs (A has at most 64 rows); the accumulator's row
                      // 16q + i sits in TMEM lane 32q + i (i < 16) of lane quarter q
    uint64_t timeout_ns;
    int* err;
    const float* bias;  // epilogue (see Gemm): c * scale if apply_scale, + bias[col]
    float scale;
    int apply_scale;
    // Implicit-GEMM convolution (the CONV variants: single CTA, stride 1).
    // B is the NHWC input through a 4-D tensor map {C, W, H, N} (tmB; X3:
    // tmB[1] its lo plane).  k-block kb is channels 32 * (kb % cv_cblocks) ..
    // + 31 of tap kb / cv_cblocks = kh * kW + kw; a tile is cv_rows output rows
    // of cv_W_out pixels (tile_n columns, the MMA's N), each row one TMA box
    // {32 channels, W_out columns} starting at input column kw - pad_w of input
    // row oh - pad_h + kh (out-of-range rows and columns are the padding:
    // zero-filled by TMA).  Batch dim 0 is the image, batch dim 1 the group
    // (channel offset cv_c_group per group).  The bias, if any, is one value
    // per output row: bias[b1 * bias_group + row].
    int tile_n;
    int cv_cblocks, cv_kW, cv_pad_h, cv_pad_w, cv_rows, cv_W_out, cv_c_group;
    int64_t bias_group;
    // The weight-gradient variant (CONV = 2, ConvDw): A is dO through a map
    // {W_out, H_out, C_out, N, 1} (box: 32 pixels of one row x 128 channels),
    // B the NHWC input through {C, W, H, N, 1} (box: 32 channels x 32 pixels,
    // MN-major); batch dim 0 is the split, 1 the group.  k-block kb is pixels
    // 32 * (kb % dw_wblocks) .. + 31 of output row split * dw_rows +
    // kb / dw_wblocks (flattened n * dw_H + oh); a row's last block issues
    // dw_last_ksteps k-steps of 8.  Column chunk j (32 wide) is channels
    // 32 * (j % cv_cblocks) .. of tap j / cv_cblocks; chunks of taps >=
    // dw_taps load channel dw_c_oob (past the tensor: zeros).
    int dw_rows, dw_wblocks, dw_last_ksteps, dw_H, dw_taps, dw_c_oob;
    // dw_chunked: B's map is {32, W, C / 32, H, N} (channel chunks as a dim)
    // and one box {32, 32, cv_cblocks} brings all chunks of a tap; tile_n is
    // then a multiple of 32 * cv_cblocks and dw_c_oob is a chunk coordinate.
    int dw_chunked;
    // Split K (small problems): batch dim split_dim (the last, >= 0) is the
    // split; its tiles start kps k-blocks apart (the last split's k-blocks past
    // K read zeros) and write partial products; -1: none.
    int split_dim, kps;
    // CONV variants: rows of the A box (64 when M <= 64: the MMA's rows 64..127
    // then read stale shared memory, whose products land in accumulator rows
    // that are never stored)
    int a_box_rows;
};

// The GEMM epilogue on one output value: one IEEE fp32 operation per step,
// as the reference's separate tl::scale / tl::add would round it.
__device__ __forceinline__ float tc_epilogue(const TcParams& p, float v, int col) {
    if (p.apply_scale) v = __fmul_rn(v, p.scale);
    if (p.bias) v = __fadd_rn(v, p.bias[col]);
    return v;
}
// The same with a per-row bias value (the CONV variants).
__device__ __forceinline__ float tc_epilogue_row(const TcParams& p, float v, float rb) {
    if (p.apply_scale) v = __fmul_rn(v, p.scale);
    if (p.bias) v = __fadd_rn(v, rb);
    return v;
}

// ---- tile bookkeeping ----------------------------------------------------------------

struct TileCoord {
    int b, m, n;  // batch index, tile row, tile column
};

// Tiles in batch-major order; inside a batch, groups of 16 tile rows are
// walked column by column so CTAs running together share A panels and
// B panels in L2.
__device__ __forceinline__ TileCoord tile_coord(const TcParams& p, int64_t t) {
    const int64_t per_batch = (int64_t)p.m_tiles * p.n_tiles;
    TileCoord c;
    c.b = (int)(t / per_batch);
    int r = (int)(t - (int64_t)c.b * per_batch);
    constexpr int GM = 16;
    const int group = r / (GM * p.n_tiles);
    const int first_m = group * GM;
    const int gm = min(GM, p.m_tiles - first_m);
    const int in_group = r - group * GM * p.n_tiles;
    c.m = first_m + in_group % gm;
    c.n = in_group / gm;
    return c;
}

__device__ __forceinline__ void batch_coords(const TcParams& p, int b, int (&idx)[kMaxBatchDims]) {
#pragma unroll
    for (int i = kMaxBatchDims - 1; i >= 0; --i) {
        if (i < p.nb) {
            idx[i] = b % p.bsz[i];
            b /= p.bsz[i];
        } else {
            idx[i] = 0;
        }
    }
}

// Walks the k-blocks of one tile in accumulation chunks of chunk_kb k-blocks.
// Each chunk is accumulated from zero in its own TMEM accumulator, so no
// tensor-core accumulation chain is longer than one chunk (TF32: one chunk
// per tile).  Incremental (no divisions): the MMA thread's per-k-block
// instruction count bounds the MMA issue rate.
struct KbIter {
    int in_chunk = 0, chunk_start = 0, nc = 0;
    __device__ __forceinline__ void start(const TcParams& p) {
        in_chunk = 0;
        chunk_start = 0;
        nc = min(p.chunk_kb, p.k_blocks);
    }
    __device__ __forceinline__ int kb() const { return chunk_start + in_chunk; }
    __device__ __forceinline__ bool first() const { return in_chunk == 0; }
    __device__ __forceinline__ bool last() const { return in_chunk == nc - 1; }
    // k-blocks left in the current chunk (this one included)
    __device__ __forceinline__ int left_in_chunk() const { return nc - in_chunk; }
    __device__ __forceinline__ void next(const TcParams& p) {
        if (++in_chunk == nc) {
            in_chunk = 0;
            chunk_start += p.chunk_kb;
            nc = min(p.chunk_kb, p.k_blocks - chunk_start);
        }
    }
};

// Shapes of one kernel variant.  CG: CTAs per MMA (1, or a pair); UN: the
// MMA's N (tile columns); X3: 3xTF32.  Per k-block each CTA holds 128 rows of
// A and UN / CG columns of B (X3: a hi and a lo copy of each, so the three
// products of a k-block read four tiles loaded once); it accumulates into a
// 128 x UN fp32 TMEM accumulator, double-buffered.
template <int CG, int UN, bool X3>
struct Cfg {
    static constexpr int B_COLS = UN / CG;
    static constexpr int A_BYTES = BM * BK * 4;           // 16 KB
    static constexpr int B_BYTES = B_COLS * BK * 4;       // 4 KB per 32 columns
    static constexpr int PAIR_BYTES = A_BYTES + B_BYTES;  // [A | B]
    // X3: [hi(A) | hi(B) | lo(A) | lo(B)]
    static constexpr int KB_BYTES = (X3 ? 2 : 1) * PAIR_BYTES;
    // k-blocks per stage: one full-barrier wait and one commit serve SUBS
    // k-blocks (the MMA thread's per-stage handshake costs as much as ~1 MMA)
    static constexpr int SUBS = KB_BYTES <= 32 * 1024 ? 2 : 1;
    static constexpr int STAGE_BYTES = SUBS * KB_BYTES;
    static constexpr int STAGES = (192 * 1024 / STAGE_BYTES) > 8 ? 8 : (192 * 1024 / STAGE_BYTES);
    // 8 epilogue warps, two per TMEM lane quarter, each holding half of the
    // row's columns: X3 keeps every output row's chunk sums in registers, and
    // for TF32 twice the store streams shorten the epilogue of short-K tiles
    // (measured: attention-shaped products +5 %, conv +2 %, long K unchanged).
    static constexpr int EPI_WARPS = 8;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int EPI_COLS = UN * 4 / EPI_WARPS;  // accumulator columns per epilogue warp
    static constexpr int TMEM_COLS = 2 * UN;
    static constexpr int TILE_M = BM * CG;
    static constexpr int BAR_BYTES = 256;
    // TF32: each epilogue warp turns its 32 rows x 32 columns around in shared
    // memory so that one store instruction writes four whole 128-byte rows.
    static constexpr int EPI_STAGE_BYTES = X3 ? 0 : EPI_WARPS * 32 * 32 * 4;
    static constexpr int TOTAL = STAGES * STAGE_BYTES + BAR_BYTES + EPI_STAGE_BYTES + 1024;  // + alignment slack
    static_assert(TMEM_COLS <= 512, "two accumulators must fit in TMEM");
    static_assert(B_COLS % 32 == 0 && B_COLS <= 256, "B tile columns");
    static_assert(STAGES >= 2, "at least two pipeline stages");
    static_assert(EPI_COLS % 32 == 0, "epilogue columns in 32-column TMEM loads");
    static_assert(TOTAL <= 227 * 1024, "dynamic shared memory per CTA");
};

// X3: the epilogue adds the chunk partials of each output element into
// registers in fp32 round-to-nearest and stores after the last chunk.
template <int CG, int UN, bool X3, int CONV = 0>
__global__ void __launch_bounds__(Cfg<CG, UN, X3>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ TcParams p) {
    using S = Cfg<CG, UN, X3>;
    constexpr int STAGES = S::STAGES;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte-swizzle atoms.
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    // [stages][epilogue staging (TF32)][barriers]: the staging squares start
    // 1024-byte aligned, as the 128-byte swizzle of the TMA store requires.
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES + S::EPI_STAGE_BYTES);
    uint64_t* full = bars;                 // [STAGES]  (used in the leader CTA)
    uint64_t* empty = bars + STAGES;       // [STAGES]
    uint64_t* tfull = bars + 2 * STAGES;   // [2]
    uint64_t* tempty = tfull + 2;          // [2]       (used in the leader CTA)
    uint64_t* drain = tempty + 2;          // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int64_t unit = CG == 2 ? blockIdx.x / 2 : blockIdx.x;  // tile-walking unit (pair)
    const int64_t units = CG == 2 ? gridDim.x / 2 : gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], S::EPI_WARPS * CG);  // one arrival per epilogue warp of each CTA
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        prefetch_map(&p.tmA[0]);
        prefetch_map(&p.tmB[0]);
        if constexpr (X3) {
            prefetch_map(&p.tmA[1]);
            prefetch_map(&p.tmB[1]);
        }
    }
    if (warp == 1) {
        __syncwarp();
        tmem_alloc<CG>(tmem_slot, S::TMEM_COLS);
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();  // peer barriers initialised before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        {
            int stage = 0;
            uint32_t phase = 0;
            // Bit s of pend: a load was issued into stage s and nobody has seen
            // it complete yet; bit s of pend_par: the parity it completes with.
            uint32_t pend = 0, pend_par = 0;
            const uint32_t a_chunk_bytes = 32 * BK * 4;
            bool ok = true;
            for (int64_t t = unit; ok && t < p.num_tiles; t += units) {
                const TileCoord tc = tile_coord(p, t);
                int bi[kMaxBatchDims];
                batch_coords(p, tc.b, bi);
                const int a0 = p.a_bc[0] ? bi[0] : 0, a1 = p.a_bc[1] ? bi[1] : 0,
                          a2 = p.a_bc[2] ? bi[2] : 0;
                const int b0 = p.b_bc[0] ? bi[0] : 0, b1 = p.b_bc[1] ? bi[1] : 0,
                          b2 = p.b_bc[2] ? bi[2] : 0;
                const int m0 = tc.m * S::TILE_M + (int)rank * BM;       // this CTA's A rows
                const int n0 = tc.n * UN + (int)rank * S::B_COLS;       // this CTA's B columns
                // CONV = 2: the tile's B boxes (fixed over its k-blocks) and the
                // position of its first k-block, advanced without divisions
                int dw_img = 0, dw_oh = 0, dw_wb = 0, nbox = 0;
                int bx_c[8], bx_w[8], bx_h[8];
                if constexpr (CONV == 2) {
                    const int R0 = bi[0] * p.dw_rows;
                    dw_img = R0 / p.dw_H;
                    dw_oh = R0 - dw_img * p.dw_H;
                    const int per_box = p.dw_chunked ? p.cv_cblocks : 1;  // 32-channel chunks per box
                    nbox = p.tile_n / (32 * per_box);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        bx_c[c] = p.dw_c_oob;
                        bx_w[c] = bx_h[c] = 0;
                        if (c < nbox) {
                            const int jc = (tc.n * p.tile_n >> 5) + c * per_box;  // first chunk of box c
                            const int tap = jc / p.cv_cblocks, cb = jc - tap * p.cv_cblocks;
                            const int kh = tap / p.cv_kW, kw = tap - kh * p.cv_kW;
                            if (tap < p.dw_taps)
                                bx_c[c] = p.dw_chunked ? bi[1] * p.cv_cblocks : bi[1] * p.cv_c_group + cb * 32;
                            bx_w[c] = kw - p.cv_pad_w;
                            bx_h[c] = kh - p.cv_pad_h;
                        }
                    }
                }
                // split K (constant indices keep bi in registers)
                const int kb_base = p.split_dim < 0 ? 0
                                    : (p.split_dim == 0 ? bi[0] : p.split_dim == 1 ? bi[1] : bi[2]) * p.kps;
                KbIter it;
                it.start(p);
                for (int kb = 0; kb < p.k_blocks;) {
                    if (!warp_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.timeout_ns, p.err, 1,
                                           kGemmSleepNs)) {
                        ok = false;
                        break;
                    }
                    // The stage's previous load was consumed (the MMA that read it finished).
                    pend &= ~(1u << stage);
                    // up to SUBS k-blocks of one accumulation chunk share the stage
                    const int nsub = min(S::SUBS, it.left_in_chunk());
                    const uint32_t fb = CG == 2 ? mapa(smem_u32(&full[stage]), 0)
                                                : smem_u32(&full[stage]);
                    if (leader && elect_one()) {
                        if constexpr (CONV == 1)
                            mbar_expect_tx(&full[stage], nsub * (X3 ? 2 : 1) *
                                                             (p.a_box_rows * BK * 4 + p.cv_rows * p.cv_W_out * 128));
                        else if constexpr (CONV == 2)
                            mbar_expect_tx(&full[stage], nsub * (X3 ? 2 : 1) *
                                                             (p.a_box_rows * BK * 4 + p.tile_n * BK * 4));
                        else
                            mbar_expect_tx(&full[stage], nsub * S::KB_BYTES * CG);
                    }
                    for (int j = 0; j < nsub; ++j, ++kb, it.next(p)) {
                        const int k0 = (kb_base + it.kb()) * BK;
                        if constexpr (CONV == 2) {
                            // 32 pixels of one output row: dO's row (A), and per
                            // tap of the tile the input pixels it reads for them
                            // (B, MN-major)
                            if (elect_one()) {
                                const int w0 = dw_wb * BK;
#pragma unroll
                                for (int h = 0; h < (X3 ? 2 : 1); ++h) {
                                    uint8_t* sa = smem + stage * S::STAGE_BYTES + j * S::KB_BYTES +
                                                  h * S::PAIR_BYTES;
                                    uint8_t* sb = sa + S::A_BYTES;
                                    tma_load_5d<CG>(sa, &p.tmA[h], fb, w0, dw_oh, bi[1] * p.M + m0, dw_img, 0);
#pragma unroll
                                    for (int c = 0; c < 8; ++c) {
                                        if (c >= nbox) break;
                                        if (p.dw_chunked)
                                            tma_load_5d<CG>(sb + c * p.cv_cblocks * a_chunk_bytes, &p.tmB[h], fb, 0,
                                                            w0 + bx_w[c], bx_c[c], dw_oh + bx_h[c], dw_img);
                                        else
                                            tma_load_5d<CG>(sb + c * a_chunk_bytes, &p.tmB[h], fb, bx_c[c],
                                                            w0 + bx_w[c], dw_oh + bx_h[c], dw_img, 0);
                                    }
                                }
                            }
                            if (++dw_wb == p.dw_wblocks) {
                                dw_wb = 0;
                                if (++dw_oh == p.dw_H) {
                                    dw_oh = 0;
                                    ++dw_img;
                                }
                            }
                            continue;
                        }
                        if (!elect_one()) continue;
#pragma unroll
                        for (int h = 0; h < (X3 ? 2 : 1); ++h) {  // X3: hi, then lo planes
                            uint8_t* sa = smem + stage * S::STAGE_BYTES + j * S::KB_BYTES +
                                          h * S::PAIR_BYTES;
                            uint8_t* sb = sa + S::A_BYTES;
                            if (p.a_chunked) {
                                tma_load_5d<CG>(sa, &p.tmA[h], fb, 0, k0, m0 >> 5, a0, a1);
                            } else if (p.a_mn) {
#pragma unroll
                                for (int c = 0; c < BM / 32; ++c)
                                    tma_load_5d<CG>(sa + c * a_chunk_bytes, &p.tmA[h], fb,
                                                    m0 + 32 * c, k0, a0, a1, a2);
                            } else {
                                tma_load_5d<CG>(sa, &p.tmA[h], fb, k0, m0, a0, a1, a2);
                            }
                            if constexpr (CONV == 1) {
                                // cv_rows boxes, one per output row of the tile
                                const int kb = k0 / BK;
                                const int tap = kb / p.cv_cblocks, cb = kb - tap * p.cv_cblocks;
                                const int kh = tap / p.cv_kW, kw = tap - kh * p.cv_kW;
                                const int c = bi[1] * p.cv_c_group + cb * 32;
                                const int oh0 = tc.n * p.cv_rows;
                                tma_load_5d<CG>(sb, &p.tmB[h], fb, c, kw - p.cv_pad_w, oh0 - p.cv_pad_h + kh,
                                                bi[0], 0);
                            } else if (p.b_chunked) {
                                tma_load_5d<CG>(sb, &p.tmB[h], fb, 0, k0, n0 >> 5, b0, b1);
                            } else if (p.b_mn) {
#pragma unroll
                                for (int c = 0; c < S::B_COLS / 32; ++c)
                                    tma_load_5d<CG>(sb + c * a_chunk_bytes, &p.tmB[h], fb,
                                                    n0 + 32 * c, k0, b0, b1, b2);
                            } else {
                                tma_load_5d<CG>(sb, &p.tmB[h], fb, k0, n0, b0, b1, b2);
                            }
                        }
                    }
                    pend |= 1u << stage;
                    pend_par = (pend_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok && leader && lane == 0) {
                // Drain: wait (bounded) for loads still in flight into shared memory
                // (the leader's full barriers count both CTAs' bytes).
                for (int s = 0; s < STAGES; ++s) {
                    if (!(pend & (1u << s))) continue;
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(&full[s], (pend_par >> s) & 1u) &&
                           globaltimer() - t0 < p.timeout_ns) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA) ----------------
        // The whole warp runs the loop; each tcgen05 operation comes from one
        // elected lane (elect_one), the waits from lane 0 (warp_wait_bounded).
        if (leader) {
            // kind::tf32: D fp32 (bits 4-5 = 1), A/B TF32 (bits 7-9, 10-12 = 2),
            // A/B major (bits 15, 16), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
            const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) |
                                   ((uint32_t)p.a_mn << 15) | ((uint32_t)p.b_mn << 16) |
                                   ((uint32_t)((CONV ? p.tile_n : UN) >> 3) << 17) |
                                   ((uint32_t)((CONV && p.m64 ? 64 : S::TILE_M) >> 4) << 24);
            const uint32_t chunk = 32 * BK * 4;  // bytes between 32-wide MN chunks
            // Descriptors of stage 0, k-step 0; a stage / k-step moves only the
            // start-address field (bits 0-13, address >> 4), so later ones are
            // one add away.  MN-major: k-step j starts 8 k-rows (1 KB) further;
            // chunks of 32 MN elements are `chunk` bytes apart (leading
            // offset), 4-row k groups 512 B apart (stride offset).  K-major:
            // 32 B further along the 128-byte rows; 8-row atoms 1 KB apart.
            const uint32_t s0 = smem_u32(smem);
            const uint64_t a_desc0 = p.a_mn ? smem_desc(s0, chunk, 512, kSw128Atom32)
                                            : smem_desc(s0, 16, 1024, kSw128);
            const uint64_t b_desc0 = p.b_mn ? smem_desc(s0 + S::A_BYTES, chunk, 512, kSw128Atom32)
                                            : smem_desc(s0 + S::A_BYTES, 16, 1024, kSw128);
            const uint32_t a_step = (p.a_mn ? 1024u : UMMA_K * 4u) >> 4;
            const uint32_t b_step = (p.b_mn ? 1024u : UMMA_K * 4u) >> 4;
            constexpr uint32_t lo_off = S::PAIR_BYTES >> 4;  // hi -> lo copy of a tile
            const uint32_t empty_addr = smem_u32(&empty[0]);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t acc_ph = 0;  // bit a: phase parity of accumulator a
            int acc = 0;
            bool ok = true;
            bool issued = false;
            for (int64_t t = unit; ok && t < p.num_tiles; t += units) {
                uint32_t d = 0;
                KbIter it;
                it.start(p);
                for (int kb = 0; kb < p.k_blocks;) {
                    // the stage holds up to SUBS k-blocks of one chunk (as loaded)
                    const int nsub = min(S::SUBS, it.left_in_chunk());
                    if (it.first()) {
                        // a fresh accumulator for this chunk, once the epilogues drained it
                        if (!warp_wait_bounded(&tempty[acc], ((acc_ph >> acc) & 1u) ^ 1u, abort_flag,
                                               p.timeout_ns, p.err, 2, kGemmSleepNs)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        d = tmem_base + (uint32_t)(acc * UN);
                    }
                    if (!warp_wait_bounded(&full[stage], phase, abort_flag, p.timeout_ns, p.err, 3,
                                           kGemmSleepNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    bool chunk_end = false;
                    for (int s = 0; s < nsub; ++s, ++kb, it.next(p)) {
                        const bool first = it.first();
                        chunk_end = it.last();
                        const uint32_t soff =
                            (uint32_t)(stage * S::STAGE_BYTES + s * S::KB_BYTES) >> 4;
                        const uint64_t ad = a_desc0 + soff, bd = b_desc0 + soff;
                        // CONV = 2: a row's last pixel block may hold fewer than
                        // BK pixels; its k-steps past the row are not issued
                        int ksteps = BK / UMMA_K;
                        if constexpr (CONV == 2)
                            if (it.kb() % p.dw_wblocks == p.dw_wblocks - 1) ksteps = p.dw_last_ksteps;
                        if constexpr (X3) {
                            // lo(A).hi(B) + hi(A).lo(B) + hi(A).hi(B): small terms first
#pragma unroll
                            for (int j = 0; j < BK / UMMA_K; ++j)
                                if (j < ksteps && elect_one())
                                    umma_tf32<CG>(d, ad + lo_off + j * a_step, bd + j * b_step, idesc,
                                                  (!first || j > 0) ? 1u : 0u);
#pragma unroll
                            for (int j = 0; j < BK / UMMA_K; ++j)
                                if (j < ksteps && elect_one())
                                    umma_tf32<CG>(d, ad + j * a_step, bd + lo_off + j * b_step, idesc, 1u);
#pragma unroll
                            for (int j = 0; j < BK / UMMA_K; ++j)
                                if (j < ksteps && elect_one())
                                    umma_tf32<CG>(d, ad + j * a_step, bd + j * b_step, idesc, 1u);
                        } else {
#pragma unroll
                            for (int j = 0; j < BK / UMMA_K; ++j)
                                if (j < ksteps && elect_one())
                                    umma_tf32<CG>(d, ad + j * a_step, bd + j * b_step, idesc,
                                                  (!first || j > 0) ? 1u : 0u);
                        }
                    }
                    issued = true;
                    // free the stage in every CTA once these MMAs finish
                    if (elect_one()) {
                        if constexpr (CG == 2)
                            umma_commit_both(empty_addr + 8u * stage);
                        else
                            umma_commit<CG>(empty_addr + 8u * stage);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (chunk_end) {
                        // chunk accumulator ready for the epilogues of both CTAs
                        if (elect_one()) {
                            if constexpr (CG == 2)
                                umma_commit_both(smem_u32(&tfull[acc]));
                            else
                                umma_commit<CG>(smem_u32(&tfull[acc]));
                        }
                        acc_ph ^= 1u << acc;
                        acc ^= 1;
                    }
                }
            }
            if (!ok && issued && elect_one()) {
                // Drain MMAs still reading shared memory / writing TMEM (the
                // elected lane is the one that issued them).
                umma_commit<CG>(smem_u32(drain));
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < p.timeout_ns) {
                }
            }
            __syncwarp();
        }
    } else {
        // ---------------- epilogue (warps 2.., both CTAs) ----------------
        // A warp may access only TMEM lane quarter warp % 4; with 8 epilogue
        // warps two share a quarter and split the columns.
        const int q = warp & 3;
        const int col_half = (warp - 2) >> 2;  // 0 with 4 epilogue warps
        // m64: lanes 16..31 of a quarter hold no row (their row is set past M)
        const bool m64 = CONV && p.m64;
        const int row_in_tile = m64 ? (lane < 16 ? q * 16 + lane : p.M) : q * 32 + lane;
        const uint32_t tempty_leader = CG == 2 ? mapa(smem_u32(&tempty[0]), 0) : 0u;
        uint32_t acc_ph = 0;  // bit a: phase parity of accumulator a
        int acc = 0;
        bool ok = true;
        for (int64_t t = unit; ok && t < p.num_tiles; t += units) {
            const TileCoord tc = tile_coord(p, t);
            int bi[kMaxBatchDims];
            batch_coords(p, tc.b, bi);
            int64_t oc = 0;
#pragma unroll
            for (int i = 0; i < kMaxBatchDims; ++i) oc += (int64_t)bi[i] * p.cbs[i];
            const int64_t row = m64 ? (int64_t)row_in_tile
                                    : (int64_t)tc.m * S::TILE_M + (int)rank * BM + row_in_tile;
            const int tn = CONV ? p.tile_n : UN;  // output columns of a tile
            const int n0 = tc.n * tn + col_half * S::EPI_COLS;
            // CONV: the tile's columns end here (TMEM columns past its width
            // hold nothing of it); otherwise the matrix's
            const int nlim = CONV ? min(p.N, tc.n * tn + tn) : p.N;
            float* crow = p.C + oc + row * p.c_rs;
            float rb = 0.0f;  // CONV: this row's bias
            if constexpr (CONV == 1) {
                if (p.bias && row < p.M) rb = p.bias[bi[1] * p.bias_group + row];
            }
            float sum[X3 ? S::EPI_COLS : 1];
#pragma unroll
            for (int j = 0; j < (X3 ? S::EPI_COLS : 1); ++j) sum[j] = 0.0f;
            for (int ch = 0; ch < p.num_chunks; ++ch) {
                ok = warp_wait_bounded(&tfull[acc], (acc_ph >> acc) & 1u, abort_flag, p.timeout_ns,
                                       p.err, 4, kGemmSleepNs);  // one branch per warp
                if (!ok) break;
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) +
                                       (uint32_t)(acc * UN + col_half * S::EPI_COLS);
                if constexpr (X3) {
                    // 16-column loads: the sums already hold EPI_COLS registers
#pragma unroll
                    for (int c = 0; c < S::EPI_COLS / 16; ++c) {
                        uint32_t r[16];
                        tmem_ld16(taddr + c * 16, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            sum[c * 16 + j] = __fadd_rn(sum[c * 16 + j], __uint_as_float(r[j]));
                    }
                } else {
                    // This warp's 32 x 32 staging square: 128-byte rows whose
                    // 16-byte chunks are XOR-swizzled by row, so both the
                    // row-per-thread writes and the row-per-8-lanes reads
                    // touch every bank once per 16-byte column.
                    float* stg = reinterpret_cast<float*>(smem + STAGES * S::STAGE_BYTES) +
                                 (warp - 2) * 32 * 32;
                    const int64_t row0 = m64 ? q * 16 : row - lane;  // the warp's first output row
                    const int rows_here = m64 ? 16 : 32;            // of the staging square's rows
#pragma unroll 1
                    for (int c = 0; c < S::EPI_COLS / 32; ++c) {
                        uint32_t r[32];
                        tmem_ld32(taddr + c * 32, r);
                        tmem_wait_ld();
                        const int col0 = n0 + c * 32;
                        if (CONV && col0 >= nlim) continue;  // past the tile (warp-uniform)
                        if (p.tma_c && (!CONV || col0 + 32 <= nlim || nlim == p.N)) {  // warp-uniform
                            // The square goes out with one TMA store (rows and
                            // columns past M, N clipped by the tensor map; in a
                            // CONV tile, a square that would reach the next
                            // tile's columns takes the element-wise path).
                            if (col0 >= p.N || row0 >= p.M) continue;
                            if (p.bias || p.apply_scale) {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    if (col0 + j < nlim)
                                        r[j] = __float_as_uint((CONV ? tc_epilogue_row(p, __uint_as_float(r[j]), rb) : tc_epilogue(p, __uint_as_float(r[j]), col0 + j)));
                            }
                            if (lane == 0) bulk_wait_read_all();  // the previous square was read out
                            __syncwarp();
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                *reinterpret_cast<uint4*>(stg + lane * 32 + ((j ^ (lane & 7)) << 2)) =
                                    make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_5d(&p.tmC, stg, col0, (int)row0, bi[0], bi[1], bi[2]);
                                bulk_commit_group();
                            }
                        } else if (p.vec_c && col0 + 32 <= nlim) {  // warp-uniform
                            if (p.bias || p.apply_scale) {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    r[j] = __float_as_uint((CONV ? tc_epilogue_row(p, __uint_as_float(r[j]), rb) : tc_epilogue(p, __uint_as_float(r[j]), col0 + j)));
                            }
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                *reinterpret_cast<uint4*>(stg + lane * 32 + ((j ^ (lane & 7)) << 2)) =
                                    make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
                            __syncwarp();
                            const int sub = lane & 7;
#pragma unroll
                            for (int it = 0; it < 8; ++it) {
                                const int rr = it * 4 + (lane >> 3);
                                const float4 v =
                                    *reinterpret_cast<const float4*>(stg + rr * 32 + ((sub ^ (rr & 7)) << 2));
                                if (rr < rows_here && row0 + rr < p.M)
                                    *reinterpret_cast<float4*>(p.C + oc + (row0 + rr) * p.c_rs + col0 + sub * 4) = v;
                            }
                            __syncwarp();
                        } else if (row < p.M) {
                            if (p.bias || p.apply_scale) {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    if (col0 + j < nlim)
                                        r[j] = __float_as_uint((CONV ? tc_epilogue_row(p, __uint_as_float(r[j]), rb) : tc_epilogue(p, __uint_as_float(r[j]), col0 + j)));
                            }
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (col0 + j < nlim) crow[col0 + j] = __uint_as_float(r[j]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (CG == 2 && !leader)
                        mbar_arrive_remote(tempty_leader + 8u * acc);
                    else
                        mbar_arrive(&tempty[acc]);
                }
                acc_ph ^= 1u << acc;
                acc ^= 1;
            }
            if constexpr (X3) {
                if (ok && row < p.M) {
#pragma unroll
                    for (int c = 0; c < S::EPI_COLS / 32; ++c) {
                        const int col0 = n0 + c * 32;
                        if (p.bias || p.apply_scale) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (col0 + j < nlim) sum[c * 32 + j] = (CONV ? tc_epilogue_row(p, sum[c * 32 + j], rb) : tc_epilogue(p, sum[c * 32 + j], col0 + j));
                        }
                        if (p.vec_c && col0 + 32 <= nlim) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<float4*>(crow + col0 + j) =
                                    make_float4(sum[c * 32 + j], sum[c * 32 + j + 1],
                                                sum[c * 32 + j + 2], sum[c * 32 + j + 3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (col0 + j < nlim) crow[col0 + j] = sum[c * 32 + j];
                        }
                    }
                }
            }
        }
    }

    // TMA stores of C still reading the staging squares / writing C complete
    // before the CTA's shared memory goes away.
    if constexpr (!X3) {
        if (warp >= 2 && lane == 0 && p.tma_c) bulk_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    // CG = 2: neither CTA frees its TMEM or exits while the pair's MMAs or the
    // peer's remote arrivals may still touch its memory.
    if constexpr (CG == 2) cluster_sync();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();  // .sync.aligned: the whole warp, converged
        tmem_dealloc<CG>(tmem_base, S::TMEM_COLS);
    }
}

// hi = tf32 round-to-nearest(x) (low 13 mantissa bits zero), lo = x - hi
// (exact in fp32): the 3xTF32 operand split.
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        uint32_t h;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
        const float hf = __uint_as_float(h);
        hi[i] = hf;
        lo[i] = __fsub_rn(v, hf);
    }
}

// lo = x - trunc_tf32(x) (exact in fp32): the 3xTF32 low part when the high
// part is the operand itself, which the tensor cores read truncated to TF32.
__global__ void split_lo_kernel(const float* __restrict__ x, float* __restrict__ lo, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        lo[i] = __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xFFFFE000u));
    }
}

// Tiny kernel for the failure-detection test: waits on an mbarrier that
// nothing ever arrives on, with the same bounded wait as the GEMM, and
// records the timeout in *err.
__global__ void bounded_wait_selftest_kernel(uint64_t timeout_ns, int* err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (!wait_bounded(&bar, 0, &abort_flag, timeout_ns, err, 99)) return;
        *err = -1;  // unreachable unless the barrier completed
    }
}

// ---- host side ------------------------------------------------------------------------


// One operand as a 5-D tensor map: dims {inner, outer, batch0..2}.
struct OperandMap {
    const float* base;
    int64_t inner, outer;     // extents (elements)
    int64_t outer_stride;     // elements
    int64_t bsz[kMaxBatchDims];
    int64_t bstride[kMaxBatchDims];  // elements; 0 = broadcast
    uint32_t box_inner, box_outer;
    bool mn_major;  // MN-major TF32 tiles use 32-byte swizzle granules
    // MN-major with inner % 32 == 0 and at most two batch dims: 32-wide chunks
    // per box (the map steps over chunks in its third dim), else 0
    uint32_t box_chunks;
};

int encode(CUtensorMap* map, const OperandMap& o) {
    if (o.box_chunks)
        return encode_chunked(map, o.base, o.inner, o.outer, o.outer_stride, o.bsz, o.bstride,
                              o.box_outer, o.box_chunks, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    return encode_tiled(map, o.base, o.inner, o.outer, o.outer_stride, o.bsz, o.bstride,
                        o.box_inner, o.box_outer,
                        o.mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
}



int64_t span_elems(int64_t inner, int64_t outer, int64_t os, const int64_t* bsz,
                   const int64_t* bstr, int nb) {
    int64_t hi = (inner - 1) + (outer - 1) * os;
    for (int i = 0; i < nb; ++i)
        if (bstr[i]) hi += (bsz[i] - 1) * bstr[i];
    return hi + 1;
}

struct TcScratch {
    void* p[6] = {};
    cudaStream_t s;
    explicit TcScratch(cudaStream_t st) : s(st) {}
    ~TcScratch() {
        for (void* q : p) scratch_free(q, s);
    }
};

int grid_split(int64_t n) {
    int64_t g = (n + 255) / 256;
    return (int)(g > 148 * 16 ? 148 * 16 : (g < 1 ? 1 : g));
}

// Re-lays an operand with unaligned strides/base as a dense [batch..., outer,
// round4(inner)] buffer (zero padding), so TMA can read it.
int repack(OperandMap& o, int nb, TcScratch& sc, int slot, cudaStream_t s) {
    const int64_t pitch = (o.inner + 3) & ~int64_t(3);
    int64_t total = pitch * o.outer;
    int64_t bsz_eff[kMaxBatchDims];
    for (int i = 0; i < nb; ++i) {
        bsz_eff[i] = o.bstride[i] ? o.bsz[i] : 1;
        total *= bsz_eff[i];
    }
    TLC_TRY(scratch_alloc(&sc.p[slot], sizeof(float) * (size_t)std::max<int64_t>(total, 1), s));
    float* dst = static_cast<float*>(sc.p[slot]);
    TLC_CUDA_TRY(cudaMemsetAsync(dst, 0, sizeof(float) * (size_t)total, s));
    // Copy view [b0, b1, b2, outer, inner] -> dense with pitch.
    int64_t sizes[5], sstr[5], dstr[5];
    int nd = 0;
    int64_t dense = pitch * o.outer;
    int64_t dstride_b[kMaxBatchDims];
    for (int i = nb - 1; i >= 0; --i) {
        dstride_b[i] = dense;
        dense *= bsz_eff[i];
    }
    for (int i = 0; i < nb; ++i) {
        sizes[nd] = bsz_eff[i];
        sstr[nd] = o.bstride[i];
        dstr[nd] = dstride_b[i];
        ++nd;
    }
    sizes[nd] = o.outer;
    sstr[nd] = o.outer_stride;
    dstr[nd] = pitch;
    ++nd;
    sizes[nd] = o.inner;
    sstr[nd] = 1;
    dstr[nd] = 1;
    ++nd;
    TLC_TRY(launch_strided_copy_to(o.base, nd, sizes, sstr, dst, dstr, s));
    o.base = dst;
    o.outer_stride = pitch;
    for (int i = 0; i < nb; ++i) o.bstride[i] = o.bstride[i] ? dstride_b[i] : 0;
    return TLC_OK;
}

// Device address of g_tc_error on the current device (per context).
int* error_word() {
    static DeviceOnce once;
    static int* words[64] = {};
    int dev = 0;
    const int st = device_once(once, [](int d) -> int {
        int* p = nullptr;
        TLC_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_tc_error));
        words[d] = p;
        return TLC_OK;
    }, &dev);
    return st == TLC_OK ? words[dev] : nullptr;
}

template <int CG, int UN, bool X3, int CONV = 0>
int launch_variant(const TcParams& prm, cudaStream_t s) {
    using S = Cfg<CG, UN, X3>;
    auto kernel = tc_gemm_kernel<CG, UN, X3, CONV>;
    static DeviceOnce once;
    static int max_units[64] = {};
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(S::THREADS, 1, 1);
    cfg.dynamicSmemBytes = S::TOTAL;
    cfg.stream = s;
    if (CG == 2) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    int dev = 0;
    TLC_TRY(device_once(once, [&](int d) -> int {
        TLC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          S::TOTAL));
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
        int units = CG == 2 ? sms / 2 : sms;
        if (CG == 2) {
            // How many CTA pairs can be resident at once (pairs share a GPC).
            int clusters = 0;
            cfg.gridDim = dim3(2 * units, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess &&
                clusters > 0)
                units = std::min(units, clusters);
            cudaGetLastError();
        }
        max_units[d] = units;
        return TLC_OK;
    }, &dev));
    const int64_t units = std::min<int64_t>(prm.num_tiles, max_units[dev]);
    cfg.gridDim = dim3((unsigned)(units * CG), 1, 1);
    TLC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, prm));
    count_launch();
    return check_launch("tc_gemm");
}

// The variant for a problem: CTA pairs (CG = 2) for more than 128 rows;
// N = 256 tiles for more than 128 columns, except single-CTA 3xTF32, whose
// four 256-column tiles per k-block would leave two pipeline stages.  A
// problem whose pair tiles would occupy fewer than half the SMs (a 512^3
// GEMM is four 256 x 256 tiles: 8 SMs) takes single-CTA 128 x 128 tiles,
// which spread the same work over four times as many SMs.
void pick_variant(const Gemm& g, bool x3, int* cg, int* un) {
    *cg = g.M > 128 ? 2 : 1;
    *un = (g.N > 128 && !(x3 && *cg == 1)) ? 256 : 128;
    if (*cg == 2) {
        int sms = 148, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int64_t pairs = g.batch() * ((g.M + 255) / 256) * ((g.N + *un - 1) / *un);
        if (4 * pairs < sms) {
            *cg = 1;
            *un = 128;
        }
    }
}

// Fills the tile/launch fields of `prm` for a variant and launches it.
int launch_tc(TcParams& prm, const Gemm& g, bool x3, cudaStream_t s) {
    int cg, un;
    pick_variant(g, x3, &cg, &un);
    prm.m_tiles = (int)((g.M + BM * cg - 1) / (BM * cg));
    prm.n_tiles = (int)((g.N + un - 1) / un);
    prm.num_tiles = (int64_t)prm.m_tiles * prm.n_tiles * g.batch();
    if (x3) {
        if (cg == 1) return launch_variant<1, 128, true>(prm, s);
        return un == 256 ? launch_variant<2, 256, true>(prm, s) : launch_variant<2, 128, true>(prm, s);
    }
    if (un == 256)
        return cg == 2 ? launch_variant<2, 256, false>(prm, s) : launch_variant<1, 256, false>(prm, s);
    return cg == 2 ? launch_variant<2, 128, false>(prm, s) : launch_variant<1, 128, false>(prm, s);
}

// The parts of TcParams that do not depend on the kernel variant.
void fill_common(TcParams& prm, const Gemm& g, const OperandMap& A, const OperandMap& B,
                 bool a_mn, bool b_mn, bool x3) {
    prm.C = g.C;
    prm.c_rs = g.c_rs;
    prm.nb = g.nb;
    for (int i = 0; i < kMaxBatchDims; ++i) {
        prm.bsz[i] = i < g.nb ? (int)g.bsz[i] : 1;
        prm.cbs[i] = i < g.nb ? g.cbs[i] : 0;
        prm.a_bc[i] = (i < g.nb && A.bstride[i] != 0 && g.bsz[i] > 1) ? 1 : 0;
        prm.b_bc[i] = (i < g.nb && B.bstride[i] != 0 && g.bsz[i] > 1) ? 1 : 0;
    }
    prm.M = (int)g.M;
    prm.N = (int)g.N;
    prm.K = (int)g.K;
    prm.k_blocks = (int)((g.K + BK - 1) / BK);
    // The tensor cores' fp32 accumulation error grows linearly with the
    // length of the accumulation chain (measured: ~2.4e-9 x K relative,
    // biased towards zero), which puts long-K 3xTF32 above 1e-5.  3xTF32
    // therefore restarts the TMEM accumulator every 256 k (8 k-blocks) and
    // sums the chunks in fp32 round-to-nearest; TF32 keeps one chain.
    prm.chunk_kb = x3 ? std::min(prm.k_blocks, 8) : prm.k_blocks;
    prm.num_chunks = (prm.k_blocks + prm.chunk_kb - 1) / prm.chunk_kb;
    prm.a_mn = a_mn ? 1 : 0;
    prm.b_mn = b_mn ? 1 : 0;
    prm.a_chunked = A.box_chunks ? 1 : 0;
    prm.b_chunked = B.box_chunks ? 1 : 0;
    prm.vec_c = (al16(g.C) && (g.c_rs & 3) == 0) ? 1 : 0;
    for (int i = 0; i < g.nb; ++i)
        if (g.cbs[i] & 3) prm.vec_c = 0;
    prm.timeout_ns = 2000000000ull;  // 2 s per wait: far above any legitimate wait
    prm.bias = g.bias;
    prm.scale = g.scale;
    prm.apply_scale = g.apply_scale;
}

// A and B as tensor maps' operand descriptions (memory order: A K-major =
// {K, M}, M-major = {M, K}; B N-major = {N, K}, K-major = {K, N}).  The box
// of the outer dim is the tile extent a CTA loads; it is the same for every
// variant's A (128 rows) and, for B, at most the largest B_COLS (128).
void operand_maps(const Gemm& g, bool a_mn, bool b_mn, OperandMap& A, OperandMap& B,
                  uint32_t b_box_cols) {
    A = OperandMap{};
    B = OperandMap{};
    A.base = g.A;
    A.inner = a_mn ? g.M : g.K;
    A.outer = a_mn ? g.K : g.M;
    A.outer_stride = a_mn ? g.a_cs : g.a_rs;
    B.base = g.B;
    B.inner = b_mn ? g.N : g.K;
    B.outer = b_mn ? g.K : g.N;
    B.outer_stride = b_mn ? g.b_rs : g.b_cs;
    for (int i = 0; i < kMaxBatchDims; ++i) {
        A.bsz[i] = B.bsz[i] = i < g.nb ? g.bsz[i] : 1;
        A.bstride[i] = i < g.nb ? g.abs_[i] : 0;
        B.bstride[i] = i < g.nb ? g.bbs[i] : 0;
    }
    A.box_inner = B.box_inner = 32;
    A.box_outer = a_mn ? BK : BM;
    B.box_outer = b_mn ? BK : b_box_cols;
    A.mn_major = a_mn;
    B.mn_major = b_mn;
    // Fewer, larger TMA boxes feed the tensor cores faster (measured: a
    // 2048^3 batch with N-major B at 4 boxes per k-block runs 3-4 % slower
    // than with K-major B at 1).  Whole 32-wide chunks only: a partial last
    // chunk would read past the end of a row.
    if (a_mn && g.M % 32 == 0 && g.nb <= 2) A.box_chunks = BM / 32;
    if (b_mn && g.N % 32 == 0 && g.nb <= 2) B.box_chunks = b_box_cols / 32;
}

// B columns a CTA loads per stage for the variant launch_tc will pick.
uint32_t b_cols_for(const Gemm& g, bool x3) {
    int cg, un;
    pick_variant(g, x3, &cg, &un);
    return (uint32_t)(un / cg);
}

}  // namespace

namespace {

// 1 / 0 per device: whether the tensor cores read an fp32 operand truncated
// to TF32; -1 while unknown.
int g_tf32_truncates[64] = {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1,
                            -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1,
                            -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1,
                            -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1};

// One TF32 product whose inputs tell truncation from rounding: every A value
// is 1 + 2^-11 + 2^-12 (fp32 bits 0x3F801800), which TF32 truncation makes 1
// and any round-to-nearest makes 1 + 2^-10; B is all ones and K = 32, so
// C[m,n] = 32 under truncation and 32.03125 under rounding.  Sets
// g_tf32_truncates[dev] to 1 only if all 128 x 128 outputs are exactly 32.
int check_tf32_truncation(int dev) {
    constexpr int M = 128, N = 128, K = 32;
    std::vector<float> a(M * K), b(K * N, 1.0f), c(M * N, 0.0f);
    const uint32_t bits = 0x3F801800u;
    float av;
    std::memcpy(&av, &bits, sizeof(av));
    std::fill(a.begin(), a.end(), av);
    float* d = nullptr;
    TLC_CUDA_TRY(cudaMalloc(&d, sizeof(float) * (M * K + K * N + M * N)));
    cudaStream_t st = nullptr;
    int rc = TLC_OK;
    do {
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
            rc = set_error(TLC_ERR_CUDA, "tf32 check: cudaStreamCreate failed");
            break;
        }
        if (cudaMemcpy(d, a.data(), sizeof(float) * M * K, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d + M * K, b.data(), sizeof(float) * K * N, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = set_error(TLC_ERR_CUDA, "tf32 check: copy failed");
            break;
        }
        Gemm g{};
        g.M = M;
        g.N = N;
        g.K = K;
        g.A = d;
        g.a_rs = K;
        g.a_cs = 1;
        g.B = d + M * K;
        g.b_rs = N;
        g.b_cs = 1;
        g.C = d + M * K + K * N;
        g.c_rs = N;
        if ((rc = gemm_tc(g, TLC_MODE_TF32, st)) != TLC_OK) break;
        if (cudaStreamSynchronize(st) != cudaSuccess ||
            cudaMemcpy(c.data(), g.C, sizeof(float) * M * N, cudaMemcpyDeviceToHost) != cudaSuccess) {
            rc = set_error(TLC_ERR_CUDA, "tf32 check: the product failed");
            break;
        }
        g_tf32_truncates[dev] = std::all_of(c.begin(), c.end(), [](float v) { return v == 32.0f; }) ? 1 : 0;
    } while (false);
    if (st) cudaStreamDestroy(st);
    cudaFree(d);
    return rc;
}

}  // namespace

bool tf32_reads_truncated(cudaStream_t s) {
    // No set-up work while `s` is being captured into a graph: the split
    // that does not depend on the answer serves until the check has run.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        int dev = 0;
        cudaGetDevice(&dev);
        return dev >= 0 && dev < 64 && g_tf32_truncates[dev] == 1;
    }
    static DeviceOnce once;
    int dev = 0;
    if (device_once(once, check_tf32_truncation, &dev) != TLC_OK) {
        clear_error();
        cudaGetLastError();
        return false;
    }
    return g_tf32_truncates[dev] == 1;
}

int tc_error_word(int** p) {
    *p = error_word();
    return *p ? TLC_OK : set_error(TLC_ERR_CUDA, "no device error word");
}

// Splits of K for a 3xTF32 problem whose single-CTA tiles would occupy at
// most a quarter of the SMs (three MMAs per k-step on one issuing thread make
// a few tiles with a long K a long serial chain): as many as fill the SMs, at
// least 4 k-blocks each, at most 8; 1 = none.  Measured on 512^3 (16 tiles,
// CUDA-graph replays): 3xTF32 22.4 -> 18.5 us with 4 splits, but TF32
// 10.3 -> 12.4 us (the partial writes and their sum cost more than the
// shorter chain saves), so TF32 does not split.  Only for a dense C without
// an epilogue, at most two batch dims.
int split_k_for(const Gemm& g, const TcParams& prm, bool x3) {
    if (!x3 || g.bias || g.apply_scale || g.nb > 2 || prm.k_blocks < 8) return 1;
    int cg, un;
    pick_variant(g, x3, &cg, &un);
    if (cg != 1) return 1;
    // C dense: [batch..][M][N] contiguous
    if (g.c_rs != g.N) return 1;
    int64_t stride = g.M * g.N;
    for (int i = g.nb - 1; i >= 0; --i) {
        if (g.bsz[i] > 1 && g.cbs[i] != stride) return 1;
        stride *= g.bsz[i];
    }
    if (!al16(g.C)) return 1;
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t tiles = g.batch() * ((g.M + BM - 1) / BM) * ((g.N + un - 1) / un);
    if (tiles * 4 > sms) return 1;
    const int64_t sp = std::min<int64_t>({sms / tiles, prm.k_blocks / 4, 8});
    return (int)std::max<int64_t>(sp, 1);
}

namespace {
// The tensor-core GEMM; a_lo / b_lo (3xTF32 with truncating reads only): lo
// planes of A and B split already, in the operands' layouts.
int gemm_tc_body(const Gemm& g, int mode, cudaStream_t s, const float* a_lo, const float* b_lo) {
    if (g.batch() == 0 || g.M == 0 || g.N == 0) return TLC_OK;
    if (g.K == 0) return gemm_exact(g, s);  // writes zeros
    if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX)
        return set_error(TLC_ERR_UNSUPPORTED, "tensor-core GEMM: a dimension exceeds 2^31");
    for (int i = 0; i < g.nb; ++i)
        if (g.bsz[i] > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "batch dim too large");

    const bool x3 = mode == TLC_MODE_3XTF32;
    const bool a_mn = g.a_cs != 1;  // a_rs == 1
    const bool b_mn = g.b_cs == 1;  // else b_rs == 1
    OperandMap A, B;
    operand_maps(g, a_mn, b_mn, A, B, b_cols_for(g, x3));

    TcScratch sc(s);
    if (!tma_ok(A.base, A.outer_stride, A.bstride, g.nb)) TLC_TRY(repack(A, g.nb, sc, 0, s));
    if (!tma_ok(B.base, B.outer_stride, B.bstride, g.nb)) TLC_TRY(repack(B, g.nb, sc, 1, s));

    TcParams prm;
    memset(&prm, 0, sizeof(prm));
    if (x3) {
        // When kind::tf32 reads an fp32 input truncated to TF32 (its low 13
        // mantissa bits ignored; checked once per device), hi is the operand
        // itself and only lo = x - trunc(x), exact in fp32, is written, into a
        // plane of the operand's layout.  Otherwise hi = round(x) and
        // lo = x - hi are both written.
        const bool lo_only = tf32_reads_truncated(s);
        OperandMap* ops[2] = {&A, &B};
        CUtensorMap* maps[2] = {prm.tmA, prm.tmB};
        const float* given[2] = {a_lo, b_lo};
        for (int o = 0; o < 2; ++o) {
            if (given[o] && lo_only) {
                OperandMap l = *ops[o];
                l.base = given[o];
                TLC_TRY(encode(&maps[o][0], *ops[o]));
                TLC_TRY(encode(&maps[o][1], l));
                continue;
            }
            const int64_t n = span_elems(ops[o]->inner, ops[o]->outer, ops[o]->outer_stride,
                                         ops[o]->bsz, ops[o]->bstride, g.nb);
            TLC_TRY(scratch_alloc(&sc.p[2 + o], sizeof(float) * (size_t)n * (lo_only ? 1 : 2), s));
            float* plane = static_cast<float*>(sc.p[2 + o]);
            OperandMap h = *ops[o], l = *ops[o];
            if (lo_only) {
                split_lo_kernel<<<grid_split(n), 256, 0, s>>>(ops[o]->base, plane, n);
                l.base = plane;
            } else {
                split_tf32_kernel<<<grid_split(n), 256, 0, s>>>(ops[o]->base, plane, plane + n, n);
                h.base = plane;
                l.base = plane + n;
            }
            count_launch();
            TLC_TRY(check_launch("split_tf32"));
            TLC_TRY(encode(&maps[o][0], h));
            TLC_TRY(encode(&maps[o][1], l));
        }
    } else {
        TLC_TRY(encode(&prm.tmA[0], A));
        TLC_TRY(encode(&prm.tmB[0], B));
    }
    fill_common(prm, g, A, B, a_mn, b_mn, x3);
    if (!x3 && prm.vec_c) {
        // C as a tensor map for the epilogue's TMA stores (16-byte aligned
        // base and strides: what vec_c already checked)
        if (encode_tiled(&prm.tmC, g.C, g.N, g.M, g.c_rs, B.bsz, g.cbs, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B) == TLC_OK)
            prm.tma_c = 1;
        else
            clear_error();
    }
    prm.err = error_word();
    if (!prm.err) return set_error(TLC_ERR_CUDA, "device error word unavailable");
    prm.split_dim = -1;
    int splits = split_k_for(g, prm, x3);
    if (splits > 1) {
        // Partial products [splits][batch..][M][N] (dense), then their sum in
        // split order into C: a short-K chain per tile instead of one long one
        // on a few SMs.  Only for a dense C and no epilogue (checked above).
        const int64_t mn = g.M * g.N, total = g.batch() * mn;
        TLC_TRY(scratch_alloc(&sc.p[4], sizeof(float) * (size_t)(splits * total), s));
        float* part = static_cast<float*>(sc.p[4]);
        int64_t bsz[kMaxBatchDims] = {1, 1, 1}, cbs[kMaxBatchDims] = {0, 0, 0};
        int64_t stride = mn;
        for (int i = g.nb - 1; i >= 0; --i) {
            bsz[i] = g.bsz[i];
            cbs[i] = stride;
            stride *= g.bsz[i];
        }
        bsz[g.nb] = splits;
        cbs[g.nb] = total;
        const int kps = (prm.k_blocks + splits - 1) / splits;
        prm.C = part;
        prm.c_rs = g.N;
        prm.nb = g.nb + 1;
        for (int i = 0; i < kMaxBatchDims; ++i) {
            prm.bsz[i] = (int)bsz[i];
            prm.cbs[i] = cbs[i];
        }
        prm.a_bc[g.nb] = prm.b_bc[g.nb] = 0;
        prm.split_dim = g.nb;
        prm.kps = kps;
        prm.k_blocks = kps;
        prm.K = kps * BK;
        prm.chunk_kb = x3 ? std::min(kps, 8) : kps;
        prm.num_chunks = (kps + prm.chunk_kb - 1) / prm.chunk_kb;
        // float4 / TMA stores of the partials need rows (and so every batch and
        // split stride) a multiple of 4 floats; the buffer itself is 256-byte aligned
        prm.vec_c = g.N % 4 == 0 ? 1 : 0;
        prm.tma_c = 0;
        if (!x3 && prm.vec_c) {
            if (encode_tiled(&prm.tmC, part, g.N, g.M, g.N, bsz, cbs, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) == TLC_OK)
                prm.tma_c = 1;
            else
                clear_error();
        }
        int cg = 1, un = 128;
        pick_variant(g, x3, &cg, &un);  // cg == 1 here (split_k_for)
        prm.m_tiles = (int)((g.M + BM - 1) / BM);
        prm.n_tiles = (int)((g.N + un - 1) / un);
        prm.num_tiles = (int64_t)prm.m_tiles * prm.n_tiles * g.batch() * splits;
        if (x3)
            TLC_TRY((launch_variant<1, 128, true>(prm, s)));
        else if (un == 256)
            TLC_TRY((launch_variant<1, 256, false>(prm, s)));
        else
            TLC_TRY((launch_variant<1, 128, false>(prm, s)));
        return launch_sum_dim(part, g.C, 1, splits, total, s);
    }
    return launch_tc(prm, g, x3, s);
}

// Batch chunks of a large batched 3xTF32 product whose lo planes are split on
// a side stream ahead of the GEMMs (1: no pipeline).  One batch dim, operands
// TMA-ready as given, each batched operand's entries apart by at least one
// entry's span (so a chunk's entries are one contiguous range of the plane),
// and enough work per chunk to fill the SMs many times over.
int x3_pipeline_chunks(const Gemm& g, const OperandMap& A, const OperandMap& B) {
    constexpr int kChunks = 4;
    if (g.nb != 1 || g.bsz[0] < 2 * kChunks || (g.abs_[0] == 0 && g.bbs[0] == 0)) return 1;
    if ((double)g.M * g.N * g.K * (double)(g.bsz[0] / kChunks) < 4.0 * 2048 * 2048 * 2048) return 1;
    const int64_t one = 1;
    const int64_t span_a = span_elems(A.inner, A.outer, A.outer_stride, &one, A.bstride, 0);
    const int64_t span_b = span_elems(B.inner, B.outer, B.outer_stride, &one, B.bstride, 0);
    if ((g.abs_[0] != 0 && g.abs_[0] < span_a) || (g.bbs[0] != 0 && g.bbs[0] < span_b)) return 1;
    if (!tma_ok(A.base, A.outer_stride, A.bstride, g.nb) || !tma_ok(B.base, B.outer_stride, B.bstride, g.nb))
        return 1;
    return kChunks;
}
}  // namespace

// 3xTF32 with truncating reads writes only the lo planes before the GEMM
// (an HBM-bound pass, about an eighth of a large product's time).  For a
// large batched product, x3_pipeline_chunks splits the batch: chunk c's lo
// planes are written on a side stream while the GEMM of chunk c - 1 runs
// (the split kernels use no shared memory and fit beside the GEMM's CTAs),
// and chunk c's GEMM waits for its own split only.  Each output is the same
// chain as in one launch: the same bits.
int gemm_tc(const Gemm& g, int mode, cudaStream_t s) {
    if (mode != TLC_MODE_3XTF32 || g.batch() == 0 || g.M == 0 || g.N == 0 || g.K == 0 ||
        g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX || g.bsz[0] > INT32_MAX)
        return gemm_tc_body(g, mode, s, nullptr, nullptr);
    OperandMap A, B;
    operand_maps(g, g.a_cs != 1, g.b_cs == 1, A, B, b_cols_for(g, true));
    const int nch = x3_pipeline_chunks(g, A, B);
    if (nch < 2 || !tf32_reads_truncated(s)) return gemm_tc_body(g, mode, s, nullptr, nullptr);
    const int64_t one = 1;
    const int64_t span_a = span_elems(A.inner, A.outer, A.outer_stride, &one, A.bstride, 0);
    const int64_t span_b = span_elems(B.inner, B.outer, B.outer_stride, &one, B.bstride, 0);
    const int64_t nb0 = g.bsz[0];
    const int64_t n_a = g.abs_[0] ? (nb0 - 1) * g.abs_[0] + span_a : span_a;
    const int64_t n_b = g.bbs[0] ? (nb0 - 1) * g.bbs[0] + span_b : span_b;
    TcScratch sc(s);  // freed after `fork` joins (declared first)
    TLC_TRY(scratch_alloc(&sc.p[0], sizeof(float) * (size_t)n_a, s));
    TLC_TRY(scratch_alloc(&sc.p[1], sizeof(float) * (size_t)n_b, s));
    float* lo_a = static_cast<float*>(sc.p[0]);
    float* lo_b = static_cast<float*>(sc.p[1]);
    Fork fork(s);
    cudaStream_t side = fork.begin();
    if (!side) return gemm_tc_body(g, mode, s, nullptr, nullptr);
    cudaEvent_t ready[8] = {};
    struct Events {
        cudaEvent_t* e;
        ~Events() {
            for (int i = 0; i < 8; ++i)
                if (e[i]) cudaEventDestroy(e[i]);
        }
    } guard{ready};
    const int64_t per = (nb0 + nch - 1) / nch;
    // the splits, chunk by chunk, on the side stream
    for (int c = 0; c < nch; ++c) {
        const int64_t b0 = c * per, b1 = std::min(nb0, b0 + per);
        if (b0 >= b1) break;
        const float* srcs[2] = {g.A, g.B};
        float* dsts[2] = {lo_a, lo_b};
        const int64_t strides[2] = {g.abs_[0], g.bbs[0]}, spans[2] = {span_a, span_b};
        for (int o = 0; o < 2; ++o) {
            int64_t off = 0, len = 0;
            if (strides[o]) {
                off = b0 * strides[o];
                len = (b1 - b0 - 1) * strides[o] + spans[o];
            } else if (c == 0) {
                len = spans[o];  // a broadcast operand: whole, with the first chunk
            }
            if (!len) continue;
            split_lo_kernel<<<grid_split(len), 256, 0, side>>>(srcs[o] + off, dsts[o] + off, len);
            count_launch();
            TLC_TRY(check_launch("split_tf32"));
        }
        if (cudaEventCreateWithFlags(&ready[c], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventRecord(ready[c], side) != cudaSuccess)
            return set_error(TLC_ERR_CUDA, "3xTF32 split pipeline: event");
    }
    // the GEMMs of the chunks, each after its split
    for (int c = 0; c < nch; ++c) {
        const int64_t b0 = c * per, b1 = std::min(nb0, b0 + per);
        if (b0 >= b1) break;
        if (cudaStreamWaitEvent(s, ready[c], 0) != cudaSuccess)
            return set_error(TLC_ERR_CUDA, "3xTF32 split pipeline: stream wait");
        Gemm gc = g;
        gc.A = g.A + b0 * g.abs_[0];
        gc.B = g.B + b0 * g.bbs[0];
        gc.C = g.C + b0 * g.cbs[0];
        gc.bsz[0] = b1 - b0;
        TLC_TRY(gemm_tc_body(gc, mode, s, lo_a + b0 * g.abs_[0], lo_b + b0 * g.bbs[0]));
    }
    return TLC_OK;
}

namespace {
// The NHWC tensor a convolution's B tiles come from, as {C, W, H, N, 1} with
// boxes {32 channels, W_out columns, rows, 1, 1}, 128-byte swizzle (each box
// is the tile's rows * W_out K-major pixel rows of 32 channels, output row by
// output row); reads outside the tensor fill zeros.
int encode_conv_b(CUtensorMap* map, const float* x, const ConvTma& c) {
    auto fn = encode_fn();
    if (!fn) return set_error(TLC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    cuuint64_t dims[5] = {(cuuint64_t)c.C, (cuuint64_t)c.W, (cuuint64_t)c.H, (cuuint64_t)c.N, 1};
    cuuint64_t strides[4] = {(cuuint64_t)c.C * 4, (cuuint64_t)c.W * c.C * 4,
                             (cuuint64_t)c.H * c.W * c.C * 4, (cuuint64_t)c.N * c.H * c.W * c.C * 4};
    cuuint32_t box[5] = {32, (cuuint32_t)c.W_out, (cuuint32_t)c.rows, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(x), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TLC_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled (conv input) failed (" +
                                                  std::to_string((int)r) + ")");
    return TLC_OK;
}
}  // namespace

// Implicit-GEMM convolution on the tensor cores (the CONV variants, TcParams): A (the
// repacked weights) and C as in gemm_tc; B read through encode_conv_b.
int gemm_tc_conv(const Gemm& g, const ConvTma& c, int mode, cudaStream_t s) {
    if (g.batch() == 0 || g.M == 0 || g.N == 0) return TLC_OK;
    const bool x3 = mode == TLC_MODE_3XTF32;
    const int tile = c.rows * c.W_out;
    if (g.nb != 2 || g.K % BK || c.cblocks < 1 || c.W_out % 8 || tile > 256 || tile % 16 ||
        (int64_t)c.kH * c.kW * c.cblocks * BK != g.K || c.C % 4 || (x3 && (!c.x_lo || tile > 128)) ||
        g.M > INT32_MAX || g.N > INT32_MAX || g.bsz[0] > INT32_MAX || g.bsz[1] > INT32_MAX)
        return set_error(TLC_ERR_UNSUPPORTED, "implicit-GEMM convolution: unsupported shape");
    const bool a_mn = g.a_cs != 1;
    Gemm gb = g;  // B has no matrix layout here: a dummy K-major operand for the bookkeeping
    gb.B = g.A;
    gb.b_rs = 1;
    gb.b_cs = g.K;
    for (int i = 0; i < kMaxBatchDims; ++i) gb.bbs[i] = 0;
    OperandMap A, B;
    operand_maps(gb, a_mn, false, A, B, 256);
    TcScratch sc(s);
    if (!tma_ok(A.base, A.outer_stride, A.bstride, g.nb)) TLC_TRY(repack(A, g.nb, sc, 0, s));
    TcParams prm;
    memset(&prm, 0, sizeof(prm));
    prm.a_box_rows = (!a_mn && g.M <= 64) ? 64 : BM;
    A.box_outer = a_mn ? A.box_outer : (uint32_t)prm.a_box_rows;
    if (x3) {
        const bool lo_only = tf32_reads_truncated(s);
        const int64_t n = span_elems(A.inner, A.outer, A.outer_stride, A.bsz, A.bstride, g.nb);
        TLC_TRY(scratch_alloc(&sc.p[2], sizeof(float) * (size_t)n * (lo_only ? 1 : 2), s));
        float* plane = static_cast<float*>(sc.p[2]);
        OperandMap h = A, l = A;
        if (lo_only) {
            split_lo_kernel<<<grid_split(n), 256, 0, s>>>(A.base, plane, n);
            l.base = plane;
        } else {
            split_tf32_kernel<<<grid_split(n), 256, 0, s>>>(A.base, plane, plane + n, n);
            h.base = plane;
            l.base = plane + n;
        }
        count_launch();
        TLC_TRY(check_launch("split_tf32"));
        TLC_TRY(encode(&prm.tmA[0], h));
        TLC_TRY(encode(&prm.tmA[1], l));
        TLC_TRY(encode_conv_b(&prm.tmB[0], c.x, c));
        TLC_TRY(encode_conv_b(&prm.tmB[1], c.x_lo, c));
    } else {
        TLC_TRY(encode(&prm.tmA[0], A));
        TLC_TRY(encode_conv_b(&prm.tmB[0], c.x, c));
    }
    fill_common(prm, gb, A, B, a_mn, false, x3);
    prm.m64 = prm.a_box_rows == 64 && !a_mn ? 1 : 0;  // (a TMA store square spans 32 rows)
    if (!x3 && prm.vec_c && !prm.m64) {
        if (encode_tiled(&prm.tmC, g.C, g.N, g.M, g.c_rs, A.bsz, g.cbs, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B) == TLC_OK)
            prm.tma_c = 1;
        else
            clear_error();
    }
    prm.cv_cblocks = c.cblocks;
    prm.cv_kW = c.kW;
    prm.cv_pad_h = c.pad_h;
    prm.cv_pad_w = c.pad_w;
    prm.cv_rows = c.rows;
    prm.cv_W_out = c.W_out;
    prm.cv_c_group = c.c_group;
    if (c.row_bias) {
        prm.bias = c.row_bias;
        prm.bias_group = c.row_bias_group;
    }
    prm.err = error_word();
    if (!prm.err) return set_error(TLC_ERR_CUDA, "device error word unavailable");
    prm.m_tiles = (int)((g.M + BM - 1) / BM);
    prm.n_tiles = (int)((g.N + tile - 1) / tile);
    prm.num_tiles = (int64_t)prm.m_tiles * prm.n_tiles * g.batch();
    prm.tile_n = tile;
    if (x3) return launch_variant<1, 128, true, 1>(prm, s);  // tile <= 128 (checked above)
    return tile > 128 ? launch_variant<1, 256, false, 1>(prm, s) : launch_variant<1, 128, false, 1>(prm, s);
}

namespace {
// A dense 4-D tensor {d0 (contiguous), d1, d2, d3} as a 5-D map (last dim 1)
// with the given box and swizzle; reads outside the tensor fill zeros.
int encode_dense4(CUtensorMap* map, const float* base, const int64_t (&dims)[4], const uint32_t (&box)[4],
                  CUtensorMapSwizzle swizzle, const char* what) {
    auto fn = encode_fn();
    if (!fn) return set_error(TLC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    cuuint64_t d[5] = {(cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2], (cuuint64_t)dims[3], 1};
    cuuint64_t st[4];
    st[0] = (cuuint64_t)dims[0] * 4;
    st[1] = st[0] * (cuuint64_t)dims[1];
    st[2] = st[1] * (cuuint64_t)dims[2];
    st[3] = st[2] * (cuuint64_t)dims[3];
    cuuint32_t b[5] = {box[0], box[1], box[2], box[3], 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(base), d, st, b, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TLC_ERR_UNSUPPORTED, std::string("cuTensorMapEncodeTiled (") + what + ") failed (" +
                                                  std::to_string((int)r) + ")");
    return TLC_OK;
}

// The NHWC input as {32, W, C / 32, H, N}: 32 channels (contiguous), the
// pixels of a row, the 32-channel chunks (128 bytes apart), rows, images;
// box {32, 32, C_in_g / 32, 1, 1} is one tap's chunks for 32 pixels, chunk
// after chunk (the MN-major B layout, 4 KB per chunk).  C % 32 == 0.
int encode_dw_chunked(CUtensorMap* map, const float* x, const ConvDw& c) {
    auto fn = encode_fn();
    if (!fn) return set_error(TLC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    cuuint64_t d[5] = {32, (cuuint64_t)c.W, (cuuint64_t)c.C / 32, (cuuint64_t)c.H, (cuuint64_t)c.N};
    cuuint64_t st[4] = {(cuuint64_t)c.C * 4, 128, (cuuint64_t)c.W * c.C * 4, (cuuint64_t)c.H * c.W * c.C * 4};
    cuuint32_t b[5] = {32, BK, (cuuint32_t)(c.C_in_g / 32), 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(x), d, st, b, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TLC_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled (conv input chunks) failed (" +
                                                  std::to_string((int)r) + ")");
    return TLC_OK;
}

int64_t dw_cols(const ConvDw& c) { return (int64_t)c.kH * c.kW * ((c.C_in_g + 31) / 32 * 32); }

// Whether B boxes take all channel chunks of a tap at once: channels a
// multiple of 32, and a tap's chunks fit the column tile.
bool dw_chunked(const ConvDw& c, int cap) { return c.C % 32 == 0 && c.C_in_g % 32 == 0 && c.C_in_g <= cap; }

// The weight-gradient GEMM's column tile: whole taps when chunked; the
// widest tile whose padded columns stay within 1/8 of the fewest (a narrow
// MMA costs about as much to issue as a wide one).
int dw_tile_for(const ConvDw& c, int cap) {
    const int64_t N = dw_cols(c);
    const int step = dw_chunked(c, cap) ? c.C_in_g : 32;  // C_in_g is then a multiple of 32
    int64_t fewest = -1;
    for (int t = cap / step * step; t >= step; t -= step) {
        const int64_t cols = (N + t - 1) / t * t;
        if (fewest < 0 || cols < fewest) fewest = cols;
    }
    for (int t = cap / step * step; t >= step; t -= step)
        if ((N + t - 1) / t * t * 8 <= fewest * 9) return t;
    return step;
}
}  // namespace

// As many splits of the output rows as leave each SM one tile.
int conv_dw_splits(const ConvDw& c, int mode, int* splits, int* rows) {
    const int64_t N = dw_cols(c);
    const int tile = dw_tile_for(c, mode == TLC_MODE_3XTF32 ? 128 : 256);
    const int64_t per_split = (int64_t)((c.C_out_g + BM - 1) / BM) * ((N + tile - 1) / tile) * c.groups;
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t total = (int64_t)c.N * c.H_out;
    if (total < 1 || per_split < 1) return set_error(TLC_ERR_UNSUPPORTED, "implicit-GEMM weight gradient: empty");
    int64_t sp = std::min<int64_t>(std::max<int64_t>(1, sms / per_split), total);
    const int64_t r = (total + sp - 1) / sp;
    sp = (total + r - 1) / r;
    if (r > INT32_MAX || sp > 65535) return set_error(TLC_ERR_UNSUPPORTED, "implicit-GEMM weight gradient: too many rows");
    *splits = (int)sp;
    *rows = (int)r;
    return TLC_OK;
}

// The weight-gradient variant (CONV = 2) of the tensor-core GEMM; part is
// [splits][groups][C_out_g][kH * kW * round32(C_in_g)].
int gemm_tc_conv_dw(const ConvDw& c, int splits, int rows, float* part, int mode, cudaStream_t s) {
    const bool x3 = mode == TLC_MODE_3XTF32;
    const int64_t c_pad = (c.C_in_g + 31) / 32 * 32, taps = (int64_t)c.kH * c.kW, N = dw_cols(c);
    const int cap = x3 ? 128 : 256;
    const int tile = dw_tile_for(c, cap);
    const bool chunked = dw_chunked(c, cap);
    const int wblocks = (c.W_out + BK - 1) / BK;
    const int last = c.W_out - (wblocks - 1) * BK;
    const int64_t kb = (int64_t)rows * wblocks;
    if (splits < 1 || rows < 1 || c.W_out < 8 || c.W_out % 8 || c.C % 4 || c.C_out_g < 1 ||
        (c.groups > 1 && c.C_in_g % 32) || (x3 && !c.x_lo) || N > INT32_MAX || kb * BK > INT32_MAX ||
        (int64_t)splits * rows < (int64_t)c.N * c.H_out || (int64_t)splits * rows > INT32_MAX ||
        (int64_t)c.groups * c.C_out_g != c.C_out || (int64_t)c.groups * c.C_in_g != c.C ||
        !al16(c.go) || !al16(c.x) || (x3 && !al16(c.x_lo)) || !al16(part))
        return set_error(TLC_ERR_UNSUPPORTED, "implicit-GEMM weight gradient: unsupported shape");
    TcScratch sc(s);
    TcParams prm;
    memset(&prm, 0, sizeof(prm));
    prm.a_box_rows = c.C_out_g <= 64 ? 64 : BM;
    const int64_t adims[4] = {c.W_out, c.H_out, c.C_out, c.N};
    const uint32_t abox[4] = {BK, 1, (uint32_t)prm.a_box_rows, 1};  // 32 pixels of one row, the channels
    const int64_t bdims[4] = {c.C, c.W, c.H, c.N};
    const uint32_t bbox[4] = {32, BK, 1, 1};  // 32 channels, 32 pixels: an MN-major chunk
    const float* a_hi = c.go;
    const float* a_lo = nullptr;
    if (x3) {
        const bool lo_only = tf32_reads_truncated(s);
        const int64_t n = (int64_t)c.N * c.C_out * c.H_out * c.W_out;
        TLC_TRY(scratch_alloc(&sc.p[0], sizeof(float) * (size_t)n * (lo_only ? 1 : 2), s));
        float* plane = static_cast<float*>(sc.p[0]);
        if (lo_only) {
            split_lo_kernel<<<grid_split(n), 256, 0, s>>>(c.go, plane, n);
            a_lo = plane;
        } else {
            split_tf32_kernel<<<grid_split(n), 256, 0, s>>>(c.go, plane, plane + n, n);
            a_hi = plane;
            a_lo = plane + n;
        }
        count_launch();
        TLC_TRY(check_launch("split_tf32"));
        TLC_TRY(encode_dense4(&prm.tmA[1], a_lo, adims, abox, CU_TENSOR_MAP_SWIZZLE_128B, "conv dO"));
        if (chunked)
            TLC_TRY(encode_dw_chunked(&prm.tmB[1], c.x_lo, c));
        else
            TLC_TRY(encode_dense4(&prm.tmB[1], c.x_lo, bdims, bbox, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                                  "conv input"));
    }
    TLC_TRY(encode_dense4(&prm.tmA[0], a_hi, adims, abox, CU_TENSOR_MAP_SWIZZLE_128B, "conv dO"));
    if (chunked)
        TLC_TRY(encode_dw_chunked(&prm.tmB[0], c.x, c));
    else
        TLC_TRY(encode_dense4(&prm.tmB[0], c.x, bdims, bbox, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, "conv input"));
    prm.C = part;
    prm.c_rs = N;
    prm.nb = 2;
    int64_t bsz[kMaxBatchDims] = {splits, c.groups, 1};
    int64_t cbs[kMaxBatchDims] = {(int64_t)c.groups * c.C_out_g * N, (int64_t)c.C_out_g * N, 0};
    for (int i = 0; i < kMaxBatchDims; ++i) {
        prm.bsz[i] = (int)bsz[i];
        prm.cbs[i] = cbs[i];
    }
    prm.M = c.C_out_g;
    prm.N = (int)N;
    prm.K = (int)(kb * BK);
    prm.k_blocks = (int)kb;
    prm.chunk_kb = x3 ? std::min(prm.k_blocks, 8) : prm.k_blocks;
    prm.num_chunks = (prm.k_blocks + prm.chunk_kb - 1) / prm.chunk_kb;
    prm.a_mn = 0;
    prm.b_mn = 1;
    prm.vec_c = 1;  // part is 16-byte aligned and N, the strides are multiples of 32
    prm.timeout_ns = 2000000000ull;
    prm.m64 = prm.a_box_rows == 64 ? 1 : 0;
    if (!x3 && !prm.m64) {
        if (encode_tiled(&prm.tmC, part, N, c.C_out_g, N, bsz, cbs, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) == TLC_OK)
            prm.tma_c = 1;
        else
            clear_error();
    }
    prm.tile_n = tile;
    prm.cv_cblocks = (int)(c_pad / 32);
    prm.cv_kW = c.kW;
    prm.cv_pad_h = c.pad_h;
    prm.cv_pad_w = c.pad_w;
    prm.cv_c_group = c.C_in_g;
    prm.dw_rows = rows;
    prm.dw_wblocks = wblocks;
    prm.dw_last_ksteps = last / UMMA_K;
    prm.dw_H = c.H_out;
    prm.dw_taps = (int)taps;
    prm.dw_chunked = chunked ? 1 : 0;
    prm.dw_c_oob = chunked ? c.C / 32 : (c.C + 31) / 32 * 32;  // a chunk / channel past the tensor
    prm.err = error_word();
    if (!prm.err) return set_error(TLC_ERR_CUDA, "device error word unavailable");
    prm.m_tiles = (c.C_out_g + BM - 1) / BM;
    prm.n_tiles = (int)((N + tile - 1) / tile);
    prm.num_tiles = (int64_t)prm.m_tiles * prm.n_tiles * splits * c.groups;
    if (x3) return launch_variant<1, 128, true, 2>(prm, s);  // tile <= 128
    return tile > 128 ? launch_variant<1, 256, false, 2>(prm, s) : launch_variant<1, 128, false, 2>(prm, s);
}

int bounded_wait_selftest(uint64_t timeout_ns, cudaStream_t s) {
    int* err = error_word();
    if (!err) return set_error(TLC_ERR_CUDA, "device error word unavailable");
    bounded_wait_selftest_kernel<<<1, 32, 0, s>>>(timeout_ns, err);
    count_launch();
    return check_launch("bounded_wait_selftest");
}

// ---- 3xTF32 GEMM without any device allocation ---------------------------------------
//
// The regular 3xTF32 path takes its hi / lo operand planes from the stream-
// ordered memory pool.  Some callers of this library may not let it allocate
// device memory at all: a host application whose device memory is entirely
// owned by its own arena allocator (memory taken behind its back breaks its
// budget), or a latency-critical loop where an allocation that can block on
// the device or fail under memory pressure is not acceptable.  For them,
// tlc_gemm_3xtf32_noalloc runs the same split + tensor-core kernels with the
// planes in this fixed, file-scope device array instead.
//
// Properties a caller must know:
//  - Every GPU that loads the library holds these 64 MiB until the process exits.
//  - Host code cannot use the array's name as a device address (it is a host-
//    side stand-in); the device address comes from cudaGetSymbolAddress, taken
//    once per device, with that device current, by the first call on it.  That
//    first call therefore does set-up work and should come before any stream
//    capture.
//  - All calls share the one array and it keeps the last call's contents.
//    Each call rewrites, with the split pre-pass, every element its GEMM then
//    reads, so nothing has to start at zero; but two calls whose work overlaps
//    on the GPU (different streams, or different host threads on one device)
//    race on the array.  Serialise them.
//  - Operands must already suit TMA (16-byte aligned, strides multiples of 4
//    floats): unaligned operands would need a repacking copy, i.e. more memory.

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {

// Device address of g_noalloc_scratch on the current device: looked up once
// per device, with that device current, and again if the device's context
// is re-created (cudaDeviceReset), since the old address then dangles.
int noalloc_scratch(float** out) {
    static DeviceOnce once;
    static float* addr[64] = {};
    int dev = 0;
    TLC_TRY(device_once(once, [](int d) -> int {
        float* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(TLC_ERR_CUDA, std::string("cudaGetSymbolAddress(g_noalloc_scratch): ") +
                                               cudaGetErrorString(e));
        addr[d] = p;
        return TLC_OK;
    }, &dev));
    *out = addr[dev];
    return TLC_OK;
}

int64_t pad64(int64_t n) { return (n + 63) & ~int64_t(63); }  // keeps planes 256-byte aligned

int gemm_3xtf32_noalloc(const tlc_gemm_desc* d, cudaStream_t s) {
    if (!d) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gemm_3xtf32_noalloc: desc is NULL");
    if (d->M < 0 || d->N < 0 || d->K < 0 || d->batch_ndim < 0 || d->batch_ndim > 3)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gemm_3xtf32_noalloc: bad sizes");
    Gemm g{};
    g.M = d->M;
    g.N = d->N;
    g.K = d->K;
    g.A = d->A;
    g.B = d->B;
    g.C = d->C;
    g.c_rs = d->c_rs;
    g.a_rs = d->a_rs;
    g.a_cs = d->a_cs;
    g.b_rs = d->b_rs;
    g.b_cs = d->b_cs;
    g.nb = d->batch_ndim;
    for (int i = 0; i < g.nb; ++i) {
        if (d->batch_sizes[i] < 0)
            return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gemm_3xtf32_noalloc: bad batch size");
        g.bsz[i] = d->batch_sizes[i];
        g.abs_[i] = d->a_bstride[i];
        g.bbs[i] = d->b_bstride[i];
        g.cbs[i] = d->c_bstride[i];
    }
    if (g.batch() == 0 || g.M == 0 || g.N == 0) return TLC_OK;
    if (g.K == 0) return gemm_exact(g, s);  // writes zeros, uses no scratch
    if (g.a_cs != 1 && g.a_rs != 1)
        return set_error(TLC_ERR_INVALID_ARGUMENT,
                         "tlc_gemm_3xtf32_noalloc: A needs a unit stride in one matrix dim");
    if (g.b_cs != 1 && g.b_rs != 1)
        return set_error(TLC_ERR_INVALID_ARGUMENT,
                         "tlc_gemm_3xtf32_noalloc: B needs a unit stride in one matrix dim");
    if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX)
        return set_error(TLC_ERR_UNSUPPORTED, "tlc_gemm_3xtf32_noalloc: a dimension exceeds 2^31");
    for (int i = 0; i < g.nb; ++i)
        if (g.bsz[i] > INT32_MAX)
            return set_error(TLC_ERR_UNSUPPORTED, "tlc_gemm_3xtf32_noalloc: batch dim too large");

    const bool a_mn = g.a_cs != 1;
    const bool b_mn = g.b_cs == 1;
    OperandMap A, B;
    operand_maps(g, a_mn, b_mn, A, B, b_cols_for(g, true));
    if (!tma_ok(A.base, A.outer_stride, A.bstride, g.nb) ||
        !tma_ok(B.base, B.outer_stride, B.bstride, g.nb))
        return set_error(TLC_ERR_UNSUPPORTED,
                         "tlc_gemm_3xtf32_noalloc: operands must be 16-byte aligned with strides "
                         "that are multiples of 4 floats (repacking them would need memory)");

    const int64_t na = span_elems(A.inner, A.outer, A.outer_stride, A.bsz, A.bstride, g.nb);
    const int64_t nb = span_elems(B.inner, B.outer, B.outer_stride, B.bsz, B.bstride, g.nb);
    const int64_t need = 2 * (pad64(na) + pad64(nb));  // hi + lo plane of each operand
    const int64_t cap = (int64_t)(kNoAllocScratchBytes / sizeof(float));
    if (need > cap)
        return set_error(TLC_ERR_INVALID_ARGUMENT,
                         "tlc_gemm_3xtf32_noalloc: operands need " +
                             std::to_string(need * 4 / 1024) + " KiB of split planes, above the " +
                             std::to_string(kNoAllocScratchBytes >> 20) +
                             " MiB static scratch; use tlc_gemm with TLC_MODE_3XTF32");

    float* base = nullptr;
    TLC_TRY(noalloc_scratch(&base));
    float* planes[4] = {base, base + pad64(na), base + 2 * pad64(na),
                        base + 2 * pad64(na) + pad64(nb)};  // A hi, A lo, B hi, B lo
    TcParams prm;
    memset(&prm, 0, sizeof(prm));
    split_tf32_kernel<<<grid_split(na), 256, 0, s>>>(A.base, planes[0], planes[1], na);
    count_launch();
    TLC_TRY(check_launch("split_tf32"));
    split_tf32_kernel<<<grid_split(nb), 256, 0, s>>>(B.base, planes[2], planes[3], nb);
    count_launch();
    TLC_TRY(check_launch("split_tf32"));
    OperandMap ah = A, al = A, bh = B, bl = B;
    ah.base = planes[0];
    al.base = planes[1];
    bh.base = planes[2];
    bl.base = planes[3];
    TLC_TRY(encode(&prm.tmA[0], ah));
    TLC_TRY(encode(&prm.tmA[1], al));
    TLC_TRY(encode(&prm.tmB[0], bh));
    TLC_TRY(encode(&prm.tmB[1], bl));
    fill_common(prm, g, A, B, a_mn, b_mn, true);
    prm.err = error_word();
    if (!prm.err) return set_error(TLC_ERR_CUDA, "device error word unavailable");
    return launch_tc(prm, g, true, s);
}

}  // namespace
}  // namespace tlc

extern "C" int tlc_gemm_3xtf32_noalloc(const tlc_gemm_desc* desc, void* stream) {
    tlc::clear_error();
    return tlc::gemm_3xtf32_noalloc(desc, static_cast<cudaStream_t>(stream));
}
