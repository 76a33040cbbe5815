// flash_attention (src/ops.cpp:1038-1137 of torchlite-cpp) and
// FlashAttentionBackward (src/autograd.cpp:575-669) on the GPU, for one head
// [S, d] as the reference takes it, or a batch of heads [..., S, d].
//
// Forward (TLC_MODE_EXACT and _3XTF32, and TF32 where the tensor-core kernel
// of flash_tc.cu does not apply): one fused kernel, fp32 FFMA, no S x S buffer.  A CTA owns 64
// query rows; for each 64-key tile it computes T = (Q_i . K_j^T) * scale
// (each dot an ascending-c fmaf chain), then the reference's online-softmax
// update per row: m_new = max(m, max_j T), corr = exp(m - m_new),
// p = exp(T - m_new), l = l * corr + sum_j p, O = O * corr + P . V_j; at the
// end O = O * (1 / l) and L = m + log(l) (kept for the backward).  Tiles of
// Q, K, V and P sit in shared memory; each thread holds a 4 x 4 block of T
// (columns 16 apart, so the K-row reads of a warp hit distinct banks) and a
// 4 x (DM/16) block of O in registers; row max and row sum are shuffles
// among the 16 threads that share a row.
//
// Backward, TLC_MODE_TF32 with 32 <= d <= 64: the fused tensor-core kernels of
// flash_bwd_tc.cu.  Otherwise the reference's recompute scheme as batched
// GEMMs on the device (mode as for tl::matmul), per chunk of heads: D = rowsum(dO * O);
// T = Q . K^T; P = exp(T * scale - L); dV = P^T . dO; dP = dO . V^T;
// dS' = scale * (P * (dP - D)); dQ = dS' . K; dK = dS'^T . Q.  The sums over
// keys (dQ) and queries (dV, dK) run in ascending order as the reference's
// accumulation loops do; the S x S buffers hold whole heads, at most 1 GiB
// each, instead of the reference's 64 x 64 tiles.
//
// Parity with the reference is to tolerance: CUDA's expf / logf are not the
// C library's, and the row sums and the backward's accumulations run in a
// different order (the reference's own test holds flash attention to 1e-4 of
// the materialised softmax path).
#include "common.cuh"

#include <algorithm>
#include <cmath>
#include <string>

namespace tlc {
namespace {

constexpr int BQ = 64, BK = 64;

template <int DM>
struct FaCfg {
    static constexpr int DP = DM + 4;       // row pitch of the Q, K, V tiles (floats)
    static constexpr int PP = BK + 4;       // row pitch of the P tile
    static constexpr int OC = DM / 16;      // O columns per thread
    static constexpr int SMEM = sizeof(float) * (3 * BQ * DP + BQ * PP);
};

// Loads rows r0 .. r0 + 63 of a [S, d] head into a [64][DP] tile, zeros past
// row S and column d; float4 loads when VEC (d % 4 == 0, 16-byte aligned base).
template <int DM, bool VEC>
__device__ __forceinline__ void load_tile(float* t, const float* __restrict__ g, int r0, int S, int d,
                                          int tid) {
    using C = FaCfg<DM>;
    if (VEC) {
        for (int i = tid; i < BQ * (DM / 4); i += 256) {
            const int r = i / (DM / 4), c = 4 * (i - r * (DM / 4));
            float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (r0 + r < S && c < d) x = __ldg(reinterpret_cast<const float4*>(g + (int64_t)(r0 + r) * d + c));
            *reinterpret_cast<float4*>(&t[r * C::DP + c]) = x;
        }
    } else {
        for (int i = tid; i < BQ * DM; i += 256) {
            const int r = i / DM, c = i - r * DM;
            t[r * C::DP + c] = (r0 + r < S && c < d) ? __ldg(g + (int64_t)(r0 + r) * d + c) : 0.0f;
        }
    }
}

// grid (tiles * heads), tile = blockIdx.x % tiles (the tiles of one head run
// next to each other and share its K, V in L2); 256 threads: ty = tid / 16
// owns rows 4 ty .. 4 ty + 3, tx = tid % 16 owns T columns tx + 16 j and O
// columns tx * OC .. tx * OC + OC - 1.
template <int DM, bool VEC>
__global__ void __launch_bounds__(256) flash_fwd_kernel(const float* __restrict__ Q,
                                                        const float* __restrict__ K,
                                                        const float* __restrict__ V,
                                                        float* __restrict__ O, float* __restrict__ L,
                                                        int S, int d, int tiles, float scale) {
    using C = FaCfg<DM>;
    extern __shared__ float4 sm4[];
    float* sQ = reinterpret_cast<float*>(sm4);
    float* sK = sQ + BQ * C::DP;
    float* sV = sK + BK * C::DP;
    float* sP = sV + BK * C::DP;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int64_t head = blockIdx.x / tiles;
    const int q0 = (int)(blockIdx.x - head * tiles) * BQ;
    const float* Qh = Q + head * S * (int64_t)d;
    const float* Kh = K + head * S * (int64_t)d;
    const float* Vh = V + head * S * (int64_t)d;

    load_tile<DM, VEC>(sQ, Qh, q0, S, d, tid);
    float m[4], l[4], o[4][C::OC];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < C::OC; ++j) o[i][j] = 0.0f;
    }
    for (int k0 = 0; k0 < S; k0 += BK) {
        __syncthreads();  // the previous tile's K, V and P are no longer read
        load_tile<DM, VEC>(sK, Kh, k0, S, d, tid);
        load_tile<DM, VEC>(sV, Vh, k0, S, d, tid);
        __syncthreads();
        // T block: rows 4 ty + i, key columns tx + 16 j; ascending-c chains
        float t[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) t[i][j] = 0.0f;
        for (int c = 0; c < DM; c += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(&sQ[(4 * ty + i) * C::DP + c]);
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(&sK[(tx + 16 * j) * C::DP + c]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    t[i][j] = fmaf(qv[i].x, kv[j].x, t[i][j]);
                    t[i][j] = fmaf(qv[i].y, kv[j].y, t[i][j]);
                    t[i][j] = fmaf(qv[i].z, kv[j].z, t[i][j]);
                    t[i][j] = fmaf(qv[i].w, kv[j].w, t[i][j]);
                }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mb = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                t[i][j] = (k0 + tx + 16 * j < S) ? __fmul_rn(t[i][j], scale) : -INFINITY;
                mb = fmaxf(mb, t[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
            const float m_new = fmaxf(m[i], mb);
            const float corr = expf(__fsub_rn(m[i], m_new));
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = expf(__fsub_rn(t[i][j], m_new));
                sP[(4 * ty + i) * C::PP + tx + 16 * j] = p;
                rs = __fadd_rn(rs, p);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs = __fadd_rn(rs, __shfl_xor_sync(0xffffffffu, rs, off));
            l[i] = fmaf(l[i], corr, rs);
#pragma unroll
            for (int j = 0; j < C::OC; ++j) o[i][j] = __fmul_rn(o[i][j], corr);
            m[i] = m_new;
        }
        __syncthreads();
        // O += P . V_j
        for (int key = 0; key < BK; ++key) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = sP[(4 * ty + i) * C::PP + key];
            const float* vr = &sV[key * C::DP + tx * C::OC];
            float v[C::OC];
            if constexpr (C::OC % 4 == 0) {
#pragma unroll
                for (int j = 0; j < C::OC; j += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(vr + j);
                    v[j] = q4.x;
                    v[j + 1] = q4.y;
                    v[j + 2] = q4.z;
                    v[j + 3] = q4.w;
                }
            } else {
                static_assert(C::OC == 2, "head dims 32, 64, 128");
                const float2 q2 = *reinterpret_cast<const float2*>(vr);
                v[0] = q2.x;
                v[1] = q2.y;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < C::OC; ++j) o[i][j] = fmaf(p[i], v[j], o[i][j]);
        }
    }
    float* Oh = O + head * S * (int64_t)d;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = q0 + 4 * ty + i;
        if (row >= S) continue;
        const float inv = __fdiv_rn(1.0f, l[i]);
#pragma unroll
        for (int j = 0; j < C::OC; ++j) {
            const int col = tx * C::OC + j;
            if (col < d) Oh[(int64_t)row * d + col] = __fmul_rn(o[i][j], inv);
        }
        if (tx == 0 && L) L[head * S + row] = __fadd_rn(m[i], logf(l[i]));
    }
}

// D[r] = sum_c dO[r, c] * O[r, c] (ascending c)
__global__ void fa_rowdot_kernel(const float* __restrict__ dO, const float* __restrict__ O,
                                 float* __restrict__ D, int64_t rows, int d) {
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows;
         r += (int64_t)gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int c = 0; c < d; ++c) acc = fmaf(dO[r * d + c], O[r * d + c], acc);
        D[r] = acc;
    }
}

// P = exp(T * scale - L[row]) in place over [rows, S] (the reference's
// T = dot * sm_scale, then exp(T - L_i))
__global__ void fa_p_kernel(float* __restrict__ T, const float* __restrict__ L, int64_t rows, int S,
                            float scale) {
    const int64_t n = rows * S;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        T[i] = expf(__fsub_rn(__fmul_rn(T[i], scale), L[i / S]));
}

// dS' = scale * (P * (dP - D[row])) in place of dP: the factor the reference
// multiplies K_j and Q_i by (sm_scale * dS_ij, src/autograd.cpp:655-661)
__global__ void fa_ds_kernel(const float* __restrict__ P, float* __restrict__ dP, const float* __restrict__ D,
                             int64_t rows, int S, float scale) {
    const int64_t n = rows * S;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dP[i] = __fmul_rn(scale, __fmul_rn(P[i], __fsub_rn(dP[i], D[i / S])));
}

// The same two operations row by row when S is a multiple of 4 and the
// buffers 16-byte aligned: the row's L (or D) once, float4 along the row, no
// per-element 64-bit division.  Same expressions, so the same results.
__global__ void fa_p_rows_kernel(float* __restrict__ T, const float* __restrict__ L, int64_t rows, int S4,
                                 float scale) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float l = L[r];
        float4* t = reinterpret_cast<float4*>(T + r * (int64_t)S4 * 4);
        for (int j = threadIdx.x; j < S4; j += blockDim.x) {
            float4 x = t[j];
            x.x = expf(__fsub_rn(__fmul_rn(x.x, scale), l));
            x.y = expf(__fsub_rn(__fmul_rn(x.y, scale), l));
            x.z = expf(__fsub_rn(__fmul_rn(x.z, scale), l));
            x.w = expf(__fsub_rn(__fmul_rn(x.w, scale), l));
            t[j] = x;
        }
    }
}

__global__ void fa_ds_rows_kernel(const float* __restrict__ P, float* __restrict__ dP, const float* __restrict__ D,
                                  int64_t rows, int S4, float scale) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float dr = D[r];
        const float4* pr = reinterpret_cast<const float4*>(P + r * (int64_t)S4 * 4);
        float4* g = reinterpret_cast<float4*>(dP + r * (int64_t)S4 * 4);
        for (int j = threadIdx.x; j < S4; j += blockDim.x) {
            const float4 pv = pr[j];
            float4 x = g[j];
            x.x = __fmul_rn(scale, __fmul_rn(pv.x, __fsub_rn(x.x, dr)));
            x.y = __fmul_rn(scale, __fmul_rn(pv.y, __fsub_rn(x.y, dr)));
            x.z = __fmul_rn(scale, __fmul_rn(pv.z, __fsub_rn(x.z, dr)));
            x.w = __fmul_rn(scale, __fmul_rn(pv.w, __fsub_rn(x.w, dr)));
            g[j] = x;
        }
    }
}

int grid_n(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 32)); }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct Heads {
    int64_t heads = 1;
    int S = 0, d = 0;
};

int resolve(int mode, int& out) {
    if (mode == TLC_MODE_DEFAULT) mode = tlc_default_mode();
    if (mode != TLC_MODE_EXACT && mode != TLC_MODE_TF32 && mode != TLC_MODE_3XTF32)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "unknown GEMM mode " + std::to_string(mode));
    out = mode;
    return TLC_OK;
}

bool dense(const tlc_tensor* t) {
    int64_t e = 1, n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= t->sizes[i];
    if (n == 0) return true;
    for (int i = t->ndim - 1; i >= 0; --i) {
        if (t->sizes[i] != 1 && t->strides[i] != e) return false;
        e *= t->sizes[i];
    }
    return true;
}

// q, k, v (and the others given) dense with one shape [..., S, d], d <= 128
int heads_of(const tlc_tensor* const* ts, int n, const char* name, Heads& h) {
    const tlc_tensor* q = ts[0];
    if (!q || q->ndim < 2) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": tensors must be at least 2-D [S, d]");
    for (int i = 0; i < n; ++i) {
        if (!ts[i]) continue;
        if (ts[i]->ndim != q->ndim) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": shapes differ");
        for (int j = 0; j < q->ndim; ++j)
            if (ts[i]->sizes[j] != q->sizes[j]) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": shapes differ");
        if (!dense(ts[i])) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": tensors must be contiguous");
    }
    h.S = (int)q->sizes[q->ndim - 2];
    h.d = (int)q->sizes[q->ndim - 1];
    if (q->sizes[q->ndim - 2] > INT32_MAX / 2) return set_error(TLC_ERR_UNSUPPORTED, std::string(name) + ": S too large");
    if (h.d > 128) return set_error(TLC_ERR_UNSUPPORTED, std::string(name) + ": head dim above 128");
    for (int j = 0; j < q->ndim - 2; ++j) h.heads *= q->sizes[j];
    return TLC_OK;
}

template <int DM, bool VEC>
int launch_fwd_t(const float* q, const float* k, const float* v, float* o, float* l, const Heads& h,
                 float scale, cudaStream_t s) {
    static DeviceOnce once;
    TLC_TRY(smem_limit_once(once, flash_fwd_kernel<DM, VEC>, FaCfg<DM>::SMEM));
    const int64_t tiles = (h.S + BQ - 1) / BQ;
    if (tiles * h.heads > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "flash_attention: too many tiles");
    flash_fwd_kernel<DM, VEC><<<(unsigned)(tiles * h.heads), 256, FaCfg<DM>::SMEM, s>>>(
        q, k, v, o, l, h.S, h.d, (int)tiles, scale);
    count_launch();
    return check_launch("flash_attention");
}

template <int DM>
int launch_fwd(const float* q, const float* k, const float* v, float* o, float* l, const Heads& h,
               float scale, cudaStream_t s) {
    const bool vec = h.d % 4 == 0 && ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0;
    return vec ? launch_fwd_t<DM, true>(q, k, v, o, l, h, scale, s)
               : launch_fwd_t<DM, false>(q, k, v, o, l, h, scale, s);
}

// one batched GEMM over `heads` heads: C_h = A_h . B_h
int head_gemm(const float* A, int64_t a_rs, int64_t a_cs, int64_t a_bs, const float* B, int64_t b_rs,
              int64_t b_cs, int64_t b_bs, float* Cm, int64_t c_bs, int64_t M, int64_t N, int64_t K,
              int64_t heads, int mode, cudaStream_t s) {
    Gemm g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.A = A;
    g.a_rs = a_rs;
    g.a_cs = a_cs;
    g.B = B;
    g.b_rs = b_rs;
    g.b_cs = b_cs;
    g.C = Cm;
    g.c_rs = N;
    g.nb = 1;
    g.bsz[0] = heads;
    g.abs_[0] = a_bs;
    g.bbs[0] = b_bs;
    g.cbs[0] = c_bs;
    if (mode == TLC_MODE_EXACT) return gemm_exact(g, s);
    return gemm_tc(g, mode, s);
}

struct Buf {
    void* p = nullptr;
    cudaStream_t s;
    explicit Buf(cudaStream_t st) : s(st) {}
    ~Buf() { scratch_free(p, s); }
    float* f() const { return static_cast<float*>(p); }
};

// The S x S buffers of the backward are sized for at most this many bytes each
// (whole heads; one head at a time when a single head is larger).
constexpr int64_t kBwdChunkBytes = int64_t(1) << 30;

}  // namespace
}  // namespace tlc

using namespace tlc;

extern "C" int tlc_flash_attention(const tlc_tensor* q, const tlc_tensor* k, const tlc_tensor* v,
                                   float sm_scale, tlc_tensor* out, tlc_tensor* lse, int mode,
                                   void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve(mode, m));
    if (!out) return set_error(TLC_ERR_INVALID_ARGUMENT, "flash_attention: out is NULL");
    Heads h;
    const tlc_tensor* ts[4] = {q, k, v, out};
    TLC_TRY(heads_of(ts, 4, "flash_attention", h));
    if (lse) {
        bool ok = lse->ndim == q->ndim - 1 && dense(lse);
        for (int j = 0; ok && j < lse->ndim; ++j) ok = lse->sizes[j] == q->sizes[j];
        if (!ok) return set_error(TLC_ERR_INVALID_ARGUMENT, "flash_attention: lse must be contiguous [..., S]");
    }
    if (h.heads * h.S == 0) return TLC_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* l = lse ? lse->data : nullptr;
    if (m == TLC_MODE_TF32 && flash_tc_supported(h.d, q->data, k->data, v->data))
        return flash_forward_tc(q->data, k->data, v->data, out->data, l, h.heads, h.S, h.d, sm_scale, s);
    if (h.d <= 32) return launch_fwd<32>(q->data, k->data, v->data, out->data, l, h, sm_scale, s);
    if (h.d <= 64) return launch_fwd<64>(q->data, k->data, v->data, out->data, l, h, sm_scale, s);
    return launch_fwd<128>(q->data, k->data, v->data, out->data, l, h, sm_scale, s);
}

extern "C" int tlc_flash_attention_backward(const tlc_tensor* grad_out, const tlc_tensor* q,
                                            const tlc_tensor* k, const tlc_tensor* v,
                                            const tlc_tensor* out, const tlc_tensor* lse,
                                            float sm_scale, tlc_tensor* dq, tlc_tensor* dk,
                                            tlc_tensor* dv, int mode, void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve(mode, m));
    if (!dq || !dk || !dv) return set_error(TLC_ERR_INVALID_ARGUMENT, "flash_attention_backward: NULL gradient");
    Heads h;
    const tlc_tensor* ts[8] = {q, k, v, out, grad_out, dq, dk, dv};
    TLC_TRY(heads_of(ts, 8, "flash_attention_backward", h));
    bool ok = lse && lse->ndim == q->ndim - 1 && dense(lse);
    for (int j = 0; ok && j < lse->ndim; ++j) ok = lse->sizes[j] == q->sizes[j];
    if (!ok) return set_error(TLC_ERR_INVALID_ARGUMENT, "flash_attention_backward: lse must be contiguous [..., S]");
    const int64_t S = h.S, d = h.d, sd = S * d, ss = S * S;
    if (h.heads * sd == 0) return TLC_OK;  // every gradient is empty
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float* ops[9] = {grad_out->data, q->data, k->data, v->data, out->data, lse->data,
                           dq->data, dk->data, dv->data};
    if (m == TLC_MODE_TF32 && flash_bwd_tc_supported(h.d, ops, 9))
        return flash_backward_tc(grad_out->data, q->data, k->data, v->data, out->data, lse->data, dq->data,
                                 dk->data, dv->data, h.heads, h.S, h.d, sm_scale, s);
    const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(h.heads, kBwdChunkBytes / (ss * 4)));
    Buf T(s), dP(s), D(s);
    TLC_TRY(scratch_alloc(&T.p, sizeof(float) * (size_t)(chunk * ss), s));
    TLC_TRY(scratch_alloc(&dP.p, sizeof(float) * (size_t)(chunk * ss), s));
    TLC_TRY(scratch_alloc(&D.p, sizeof(float) * (size_t)(chunk * S), s));
    for (int64_t h0 = 0; h0 < h.heads; h0 += chunk) {
        const int64_t nh = std::min(chunk, h.heads - h0), rows = nh * S, off = h0 * sd;
        const float *Qc = q->data + off, *Kc = k->data + off, *Vc = v->data + off;
        const float *Oc = out->data + off, *Gc = grad_out->data + off, *Lc = lse->data + h0 * S;
        // D = rowsum(dO * O)
        fa_rowdot_kernel<<<grid_n(rows), 256, 0, s>>>(Gc, Oc, D.f(), rows, (int)d);
        count_launch();
        TLC_TRY(check_launch("flash_attention_backward"));
        // T = Q . K^T; P = exp(T * scale - L) in place
        TLC_TRY(head_gemm(Qc, d, 1, sd, Kc, 1, d, sd, T.f(), ss, S, S, d, nh, m, s));
        if (S % 4 == 0 && aligned16(T.f()))
            fa_p_rows_kernel<<<(unsigned)std::min<int64_t>(rows, 148 * 16), 256, 0, s>>>(T.f(), Lc, rows,
                                                                                      (int)(S / 4), sm_scale);
        else
            fa_p_kernel<<<grid_n(rows * S), 256, 0, s>>>(T.f(), Lc, rows, (int)S, sm_scale);
        count_launch();
        TLC_TRY(check_launch("flash_attention_backward"));
        // dV = P^T . dO
        TLC_TRY(head_gemm(T.f(), 1, S, ss, Gc, d, 1, sd, dv->data + off, sd, S, d, S, nh, m, s));
        // dP = dO . V^T, then dS' = scale * P * (dP - D) in place
        TLC_TRY(head_gemm(Gc, d, 1, sd, Vc, 1, d, sd, dP.f(), ss, S, S, d, nh, m, s));
        if (S % 4 == 0 && aligned16(T.f()) && aligned16(dP.f()))
            fa_ds_rows_kernel<<<(unsigned)std::min<int64_t>(rows, 148 * 16), 256, 0, s>>>(
                T.f(), dP.f(), D.f(), rows, (int)(S / 4), sm_scale);
        else
            fa_ds_kernel<<<grid_n(rows * S), 256, 0, s>>>(T.f(), dP.f(), D.f(), rows, (int)S, sm_scale);
        count_launch();
        TLC_TRY(check_launch("flash_attention_backward"));
        // dQ = dS' . K;  dK = dS'^T . Q
        TLC_TRY(head_gemm(dP.f(), S, 1, ss, Kc, d, 1, sd, dq->data + off, sd, S, d, S, nh, m, s));
        TLC_TRY(head_gemm(dP.f(), 1, S, ss, Qc, d, 1, sd, dk->data + off, sd, S, d, S, nh, m, s));
    }
    return TLC_OK;
}
