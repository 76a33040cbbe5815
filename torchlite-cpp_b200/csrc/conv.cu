// conv2d (src/ops.cpp:1443-1548 of torchlite-cpp) and Conv2dBackward
// (src/autograd.cpp:386-517) on the GPU: im2col into one column buffer for
// all images and groups, then ONE batched GEMM per product instead of the
// reference's per-image, per-group matmul calls.
//
// The reference per image n and group g:
//   col_ng [patch, HW] = im2col (patch p = c*kH*kW + kh*kW + kw, c local to g)
//   out[n, g] = W_g [C_out_g, patch] . col_ng                (matmul)
//   out += bias (broadcast add over N, H_out, W_out)
// backward, grad_w / grad_input / grad_bias from zeros:
//   grad_w[g] += dO_ng . col_ng^T            for n = 0, 1, ... (in order)
//   grad_col  = W_g^T . dO_ng;  grad_input[pixel] += grad_col[...] in the
//               loop order c, kh, kw, oh, ow (col2im)
//   grad_bias[c] += dO[n, c, oh, ow] for n, oh, ow in order
// Here:
//   forward   im2col_kernel -> col [N, groups, patch, HW]; one GEMM with batch
//             dims (N, groups), W_g broadcast over n (stride 0); bias: one add
//             kernel.  Every output is the same ascending-patch chain.
//   grad_w    one GEMM G[n, g] = dO_ng . col_ng^T (col read transposed in
//             place), then a sequential sum over n (the reference's +=).
//   grad_in   one GEMM grad_col[n, g] = W_g^T . dO_ng (W read transposed in
//             place), then col2im as a gather: each input pixel adds its
//             contributions in (kh, kw) order, the order in which the
//             reference's loop reaches that pixel; no atomics.
//   grad_bias one chain per channel over (n, oh, ow), the reference's order.
// In exact mode all of it is bit-identical to the reference.
#include "common.cuh"

#include <algorithm>
#include <string>

namespace tlc {
namespace {

struct ConvShape {
    int64_t N, C_in, H, W, C_out, kH, kW, stride, padding, groups;
    int64_t C_in_g, C_out_g, H_out, W_out, patch, HW;
};

// col[n, g, p, hw] = input[n, g*C_in_g + c, ih, iw] or 0 outside the image.
// One block row per (n, g, p) line of HW outputs: the patch decode happens
// once per block, threads walk hw with 32-bit index math (writes coalesced;
// reads along iw for consecutive ow).
__global__ void im2col_kernel(const float* __restrict__ in, float* __restrict__ col, ConvShape s) {
    const int64_t lines = s.N * s.groups * s.patch;
    const int HW = (int)s.HW, W_out = (int)s.W_out, H = (int)s.H, W = (int)s.W;
    const int stride = (int)s.stride, pad = (int)s.padding;
    const int khw = (int)(s.kH * s.kW), kW = (int)s.kW;
    for (int64_t line = blockIdx.x; line < lines; line += gridDim.x) {
        const int p = (int)(line % s.patch);
        const int64_t ng = line / s.patch;
        const int g = (int)(ng % s.groups);
        const int64_t n = ng / s.groups;
        const int c = g * (int)s.C_in_g + p / khw;
        const int kh = (p % khw) / kW, kw = p % kW;
        const float* src = in + (n * s.C_in + c) * (int64_t)H * W;
        float* dst = col + line * s.HW;
        for (int hw = threadIdx.x; hw < HW; hw += blockDim.x) {
            const int oh = hw / W_out, ow = hw - oh * W_out;
            const int ih = oh * stride - pad + kh, iw = ow * stride - pad + kw;
            dst[hw] = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? src[ih * W + iw] : 0.0f;
        }
    }
}

// im2col when W_out is a multiple of 4 (so is HW): each thread writes runs of
// 4 outputs along a row as one float4 (one division per 4 outputs instead of
// one per output), the reads stay coalesced across the warp.  One block per
// line (n, g, p), as above.
__global__ void im2col_vec4_kernel(const float* __restrict__ in, float* __restrict__ col, ConvShape s) {
    const int64_t lines = s.N * s.groups * s.patch;
    const int W_out = (int)s.W_out, q = W_out >> 2, n4 = (int)s.HW >> 2;
    const int H = (int)s.H, W = (int)s.W;
    const int stride = (int)s.stride, pad = (int)s.padding;
    const int khw = (int)(s.kH * s.kW), kW = (int)s.kW;
    for (int64_t line = blockIdx.x; line < lines; line += gridDim.x) {
        const int p = (int)(line % s.patch);
        const int64_t ng = line / s.patch;
        const int g = (int)(ng % s.groups);
        const int64_t n = ng / s.groups;
        const int c = g * (int)s.C_in_g + p / khw;
        const int kh = (p % khw) / kW, kw = p % kW;
        const float* src = in + (n * s.C_in + c) * (int64_t)H * W;
        float4* dst = reinterpret_cast<float4*>(col + line * s.HW);
        for (int t = threadIdx.x; t < n4; t += blockDim.x) {
            const int oh = t / q, c4 = t - oh * q;
            const int ih = oh * stride - pad + kh;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (ih >= 0 && ih < H) {
                const float* srow = src + (int64_t)ih * W;
                const int iw0 = c4 * 4 * stride - pad + kw;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int iw = iw0 + e * stride;
                    if (iw >= 0 && iw < W) v[e] = srow[iw];
                }
            }
            dst[t] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
}

// im2col with the input plane staged in shared memory (W_out a multiple of 4,
// the plane at most kIm2colPlaneMax bytes): one block per (n, c) input plane
// reads it from global memory once and writes all kH * kW of its lines, where
// the line-per-block kernels read each plane kH * kW times through L2.
constexpr int kIm2colPlaneMax = 96 * 1024;
__global__ void __launch_bounds__(256) im2col_plane_kernel(const float* __restrict__ in, float* __restrict__ col,
                                                           ConvShape s) {
    extern __shared__ float plane_s[];
    const int64_t planes = s.N * s.C_in;
    const int H = (int)s.H, W = (int)s.W, HWin = H * W;
    const int W_out = (int)s.W_out, H_out = (int)s.H_out, q = W_out >> 2, n4 = (int)s.HW >> 2;
    const int stride = (int)s.stride, pad = (int)s.padding, kH = (int)s.kH, kW = (int)s.kW, khw = kH * kW;
    const int rpp = (int)blockDim.x / q;  // output rows per pass (the host keeps q <= blockDim.x)
    const int r0 = (int)threadIdx.x / q, c4 = (int)threadIdx.x - r0 * q;
    for (int64_t plane = blockIdx.x; plane < planes; plane += gridDim.x) {
        const int c = (int)(plane % s.C_in);
        const int64_t n = plane / s.C_in;
        const int g = c / (int)s.C_in_g, cl = c % (int)s.C_in_g;
        const float* src = in + plane * (int64_t)HWin;
        __syncthreads();  // the previous plane's readers are done
        for (int i = threadIdx.x; i < HWin; i += blockDim.x) plane_s[i] = src[i];
        __syncthreads();
        // this channel's lines: p = cl * kH * kW + kh * kW + kw.  Thread
        // (r0, c4) writes float4 c4 of rows r0, r0 + rpp, .. of the
        // concatenated (k, oh) rows, walking k = kh * kW + kw and oh with
        // counters (no division per output).
        float4* lines = reinterpret_cast<float4*>(col + ((n * s.groups + g) * s.patch + (int64_t)cl * kH * kW) * s.HW);
        if (r0 < rpp) {
            int k = 0, kh = 0, kw = 0, oh = r0;
            while (oh >= H_out && k < khw) {
                oh -= H_out;
                ++k;
                if (++kw == kW) {
                    kw = 0;
                    ++kh;
                }
            }
            while (k < khw) {
                const int ih = oh * stride - pad + kh;
                float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (ih >= 0 && ih < H) {
                    const int iw0 = c4 * 4 * stride - pad + kw;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int iw = iw0 + e * stride;
                        if (iw >= 0 && iw < W) v[e] = plane_s[ih * W + iw];
                    }
                }
                lines[(int64_t)k * n4 + oh * q + c4] = make_float4(v[0], v[1], v[2], v[3]);
                oh += rpp;
                while (oh >= H_out && k < khw) {
                    oh -= H_out;
                    ++k;
                    if (++kw == kW) {
                        kw = 0;
                        ++kh;
                    }
                }
            }
        }
    }
}

// The column buffer transposed: colT[n, g, hw, p] = col[n, g, p, hw], so that
// the weight gradient's GEMM dO_ng . col_ng^T reads it as a row-major [HW,
// patch] B (the exact kernel's packed-FMA layout) instead of a K-major one.
// One block per output row (n, g, oh): the kH input rows it reads, for the
// group's channels and the columns its W_out outputs reach, are staged in
// shared memory (zero outside the image); then each thread writes its patch
// entries p = tid, tid + blockDim.x, .. of every output pixel of the row
// (coalesced along p).
__global__ void __launch_bounds__(256) im2col_t_kernel(const float* __restrict__ in, float* __restrict__ colT,
                                                       ConvShape s, int span) {
    extern __shared__ float xs[];  // [C_in_g][kH][span]
    const int kH = (int)s.kH, kW = (int)s.kW, stride = (int)s.stride, pad = (int)s.padding;
    const int H = (int)s.H, W = (int)s.W, W_out = (int)s.W_out, H_out = (int)s.H_out;
    const int Cg = (int)s.C_in_g, patch = (int)s.patch;
    const int64_t lines = s.N * s.groups * s.H_out;
    for (int64_t line = blockIdx.x; line < lines; line += gridDim.x) {
        const int oh = (int)(line % H_out);
        const int64_t ng = line / H_out;
        const int g = (int)(ng % s.groups);
        const int64_t n = ng / s.groups;
        __syncthreads();  // the previous line's readers are done
        const int staged = Cg * kH * span;
        for (int i = threadIdx.x; i < staged; i += blockDim.x) {
            const int col = i % span, ck = i / span;
            const int kh = ck % kH, c = ck / kH;
            const int ih = oh * stride - pad + kh, iw = col - pad;
            float v = 0.0f;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                v = in[((n * s.C_in + (int64_t)g * Cg + c) * H + ih) * (int64_t)W + iw];
            xs[i] = v;
        }
        __syncthreads();
        float* dst = colT + (ng * s.HW + (int64_t)oh * W_out) * patch;
        for (int p = threadIdx.x; p < patch; p += blockDim.x) {
            const int kw = p % kW, ck = p / kW;  // ck = c * kH + kh
            const float* src = xs + ck * span + kw;
            for (int ow = 0; ow < W_out; ++ow) dst[(int64_t)ow * patch + p] = src[ow * stride];
        }
    }
}

// grad_in[n, c, ih, iw] = 0 + sum over (kh, kw) ascending of grad_col at the
// (oh, ow) that read this pixel.  One block per (n, c) plane.
__global__ void col2im_kernel(const float* __restrict__ gcol, float* __restrict__ gin, ConvShape s) {
    const int64_t planes = s.N * s.C_in;
    const int H = (int)s.H, W = (int)s.W, HW = (int)s.HW, H_out = (int)s.H_out, W_out = (int)s.W_out;
    const int stride = (int)s.stride, pad = (int)s.padding, kH = (int)s.kH, kW = (int)s.kW;
    for (int64_t plane = blockIdx.x; plane < planes; plane += gridDim.x) {
        const int c = (int)(plane % s.C_in);
        const int64_t n = plane / s.C_in;
        const int g = c / (int)s.C_in_g, cl = c % (int)s.C_in_g;
        const float* base = gcol + ((n * s.groups + g) * s.patch + (int64_t)cl * kH * kW) * s.HW;
        float* dst = gin + plane * (int64_t)H * W;
        for (int pix = threadIdx.x; pix < H * W; pix += blockDim.x) {
            const int ih = pix / W, iw = pix - ih * W;
            float acc = 0.0f;
            for (int kh = 0; kh < kH; ++kh) {
                const int th = ih + pad - kh;
                if (th < 0 || th % stride) continue;
                const int oh = th / stride;
                if (oh >= H_out) continue;
                for (int kw = 0; kw < kW; ++kw) {
                    const int tw = iw + pad - kw;
                    if (tw < 0 || tw % stride) continue;
                    const int ow = tw / stride;
                    if (ow >= W_out) continue;
                    acc = __fadd_rn(acc, base[(int64_t)(kh * kW + kw) * HW + oh * W_out + ow]);
                }
            }
            dst[pix] = acc;
        }
    }
}

// col2im when W is a multiple of 4: each thread gathers 4 consecutive pixels
// of a row and stores them as one float4; every pixel still adds its terms in
// (kh, kw) ascending order from 0, as col2im_kernel does (the same sums, bit
// for bit).  STRIDE1 drops the divisibility tests of the general stride.
template <bool STRIDE1>
__global__ void col2im_vec4_kernel(const float* __restrict__ gcol, float* __restrict__ gin, ConvShape s) {
    const int64_t planes = s.N * s.C_in;
    const int H = (int)s.H, W = (int)s.W, HW = (int)s.HW, H_out = (int)s.H_out, W_out = (int)s.W_out;
    const int stride = STRIDE1 ? 1 : (int)s.stride, pad = (int)s.padding, kH = (int)s.kH, kW = (int)s.kW;
    const int q = W >> 2, n4 = H * q;
    for (int64_t plane = blockIdx.x; plane < planes; plane += gridDim.x) {
        const int c = (int)(plane % s.C_in);
        const int64_t n = plane / s.C_in;
        const int g = c / (int)s.C_in_g, cl = c % (int)s.C_in_g;
        const float* base = gcol + ((n * s.groups + g) * s.patch + (int64_t)cl * kH * kW) * s.HW;
        float4* dst = reinterpret_cast<float4*>(gin + plane * (int64_t)H * W);
        for (int t = threadIdx.x; t < n4; t += blockDim.x) {
            const int ih = t / q, iw0 = (t - ih * q) * 4;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int kh = 0; kh < kH; ++kh) {
                const int th = ih + pad - kh;
                if (th < 0) continue;
                if (!STRIDE1 && th % stride) continue;
                const int oh = STRIDE1 ? th : th / stride;
                if (oh >= H_out) continue;
                const float* row = base + (int64_t)(kh * kW) * HW + (int64_t)oh * W_out;
                for (int kw = 0; kw < kW; ++kw) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int tw = iw0 + e + pad - kw;
                        if (tw < 0) continue;
                        if (!STRIDE1 && tw % stride) continue;
                        const int ow = STRIDE1 ? tw : tw / stride;
                        if (ow >= W_out) continue;
                        acc[e] = __fadd_rn(acc[e], row[(int64_t)kw * HW + ow]);
                    }
                }
            }
            dst[t] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        }
    }
}

// grad_bias[c] = 0 + dO[n, c, hw] for n, then hw, ascending: a chain of
// N * HW dependent adds per channel.  One block per channel: warps 1-7 stage
// the chain's values, BIAS_TILE at a time, into a double-buffered shared
// ring (coalesced reads of each image's HW run); lane 0 of warp 0 adds them
// in order, loading each group of 8 before its adds so the loads stay off
// the chain.
constexpr int BIAS_TILE = 2048;
constexpr int BIAS_THREADS = 256, BIAS_STAGERS = BIAS_THREADS - 32;
__global__ void __launch_bounds__(BIAS_THREADS) bias_grad_kernel(const float* __restrict__ go,
                                                                 float* __restrict__ gb, ConvShape s) {
    __shared__ __align__(16) float tile[2][BIAS_TILE];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t total = s.N * s.HW;
    const int64_t tiles = (total + BIAS_TILE - 1) / BIAS_TILE;
    for (int64_t c = blockIdx.x; c < s.C_out; c += gridDim.x) {
        // value j of the chain: dO[j / HW, c, j % HW]
        auto stage = [&](int64_t t, int buf) {
            const int64_t j0 = t * BIAS_TILE;
            for (int k = (int)threadIdx.x - 32; k < BIAS_TILE; k += BIAS_STAGERS) {
                const int64_t j = j0 + k;
                float v = 0.0f;
                if (j < total) {
                    const int64_t n = j / s.HW, hw = j - n * s.HW;
                    v = __ldg(go + (n * s.C_out + c) * s.HW + hw);
                }
                tile[buf][k] = v;
            }
        };
        if (warp > 0 && tiles > 0) stage(0, 0);
        __syncthreads();
        float acc = 0.0f;
        for (int64_t t = 0; t < tiles; ++t) {
            const int buf = (int)(t & 1);
            if (warp > 0) {
                if (t + 1 < tiles) stage(t + 1, buf ^ 1);
            } else if (lane == 0) {
                // the same ascending chain; each group of 8 values is loaded
                // before its adds, so the loads are off the chain's critical path
                const int cnt = (int)min((int64_t)BIAS_TILE, total - t * BIAS_TILE);
                const float4* t4 = reinterpret_cast<const float4*>(tile[buf]);
                int k = 0;
#pragma unroll 4
                for (; k + 8 <= cnt; k += 8) {
                    const float4 a = t4[k >> 2], b = t4[(k >> 2) + 1];
                    acc = __fadd_rn(acc, a.x);
                    acc = __fadd_rn(acc, a.y);
                    acc = __fadd_rn(acc, a.z);
                    acc = __fadd_rn(acc, a.w);
                    acc = __fadd_rn(acc, b.x);
                    acc = __fadd_rn(acc, b.y);
                    acc = __fadd_rn(acc, b.z);
                    acc = __fadd_rn(acc, b.w);
                }
                for (; k < cnt; ++k) acc = __fadd_rn(acc, tile[buf][k]);
            }
            __syncthreads();
        }
        if (warp == 0 && lane == 0) gb[c] = acc;
        __syncthreads();
    }
}

// Non-exact modes: the bias gradient as a tree.  One block per (channel c,
// image n) sums dO[n, c, :] (a contiguous run of HW values) into
// part[c * N + n]; the sums over images follow (launch_sum_dim).  Within the
// modes' tolerance of the reference's chain, and the same on every run.
__global__ void __launch_bounds__(256) bias_part_kernel(const float* __restrict__ go, float* __restrict__ part,
                                                        ConvShape s) {
    __shared__ float red[8];
    const int64_t pairs = s.C_out * s.N;
    for (int64_t i = blockIdx.x; i < pairs; i += gridDim.x) {
        const int64_t c = i / s.N, n = i - c * s.N;
        const float* src = go + (n * s.C_out + c) * s.HW;
        float acc = 0.0f;
        for (int64_t k = threadIdx.x; k < s.HW; k += blockDim.x) acc += src[k];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.0f;
            for (int w = 0; w < 8; ++w) t += red[w];
            part[i] = t;
        }
        __syncthreads();
    }
}

// The same partial sums, one warp per (channel, image) pair with float4 loads
// (HW a multiple of 4, dO 16-byte aligned): each lane adds its float4s in
// order, then a fixed shuffle tree.
__global__ void __launch_bounds__(256) bias_part_v4_kernel(const float* __restrict__ go, float* __restrict__ part,
                                                           ConvShape s) {
    const int64_t pairs = s.C_out * s.N;
    const int lane = threadIdx.x & 31;
    const int64_t n4 = s.HW / 4;
    for (int64_t i = blockIdx.x * (int64_t)8 + (threadIdx.x >> 5); i < pairs; i += (int64_t)gridDim.x * 8) {
        const int64_t c = i / s.N, n = i - c * s.N;
        const float4* src = reinterpret_cast<const float4*>(go + (n * s.C_out + c) * s.HW);
        float acc = 0.0f;
        for (int64_t k = lane; k < n4; k += 32) {
            const float4 v = __ldg(src + k);
            acc += (v.x + v.y) + (v.z + v.w);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) part[i] = acc;
    }
}

int resolve(int mode, int& out) {
    if (mode == TLC_MODE_DEFAULT) mode = tlc_default_mode();
    if (mode != TLC_MODE_EXACT && mode != TLC_MODE_TF32 && mode != TLC_MODE_3XTF32)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "unknown GEMM mode " + std::to_string(mode));
    out = mode;
    return TLC_OK;
}

int gemm(const Gemm& g, int mode, cudaStream_t s) {
    if (g.batch() == 0 || g.M == 0 || g.N == 0) return TLC_OK;
    if (mode == TLC_MODE_EXACT || g.K == 0) return gemm_exact(g, s);
    return gemm_tc(g, mode, s);
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

// Shape checks of src/ops.cpp:1444-1465, with the reference's messages.
int conv_shape(const tlc_tensor* in, const tlc_tensor* w, int64_t stride, int64_t padding, int64_t groups,
               ConvShape& s) {
    if (!in || !w) return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: input or weight is NULL");
    if (in->ndim != 4 || w->ndim != 4)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: input and weight must be 4-D");
    s.N = in->sizes[0];
    s.C_in = in->sizes[1];
    s.H = in->sizes[2];
    s.W = in->sizes[3];
    s.C_out = w->sizes[0];
    s.kH = w->sizes[2];
    s.kW = w->sizes[3];
    s.stride = stride;
    s.padding = padding;
    s.groups = groups;
    if (groups <= 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: groups must be > 0");
    if (s.C_in % groups != 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: groups doesn't divide C_in");
    if (s.C_out % groups != 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: groups doesn't divide C_out");
    if (w->sizes[1] != s.C_in / groups)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: weight.sizes()[1] must equal C_in / groups");
    if (stride <= 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: stride must be > 0");
    if (padding < 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d: padding must be >= 0");
    s.C_in_g = s.C_in / groups;
    s.C_out_g = s.C_out / groups;
    // (H + 2p - kH) / stride + 1 with C++'s truncating division, as the
    // reference computes it.  A negative result fails there in one of two
    // places: the [N, C_out, H_out * W_out] buffer (a negative product) or
    // the final reshape to [N, C_out, H_out, W_out] (both negative).
    s.H_out = (s.H + 2 * padding - s.kH) / stride + 1;
    s.W_out = (s.W + 2 * padding - s.kW) / stride + 1;
    if (s.H_out < 0 || s.W_out < 0)
        return set_error(TLC_ERR_INVALID_ARGUMENT, s.H_out * s.W_out < 0
                                                       ? "Tensor size must be positive integer"
                                                       : "reshape: negative dims not allowed");
    s.patch = s.C_in_g * s.kH * s.kW;
    s.HW = s.H_out * s.W_out;
    // the kernels index within one image plane / column line in 32 bits
    if (s.H * s.W > INT32_MAX || s.HW > INT32_MAX || s.patch > INT32_MAX || s.kH * s.kW > INT32_MAX)
        return set_error(TLC_ERR_UNSUPPORTED, "conv2d: an image plane above 2^31 elements");
    return TLC_OK;
}

struct Buf {
    void* p = nullptr;
    cudaStream_t s;
    explicit Buf(cudaStream_t st) : s(st) {}
    ~Buf() { scratch_free(p, s); }
    float* f() const { return static_cast<float*>(p); }
};

// input (and weight) as dense NCHW: the tensor itself or a contiguous copy
int dense_copy(const tlc_tensor* t, Buf& b, const float** out, cudaStream_t s) {
    if (dense(t)) {
        *out = t->data;
        return TLC_OK;
    }
    int64_t n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= t->sizes[i];
    TLC_TRY(scratch_alloc(&b.p, sizeof(float) * (size_t)n, s));
    TLC_TRY(launch_strided_copy(t->data, t->ndim, t->sizes, t->strides, b.f(), s));
    *out = b.f();
    return TLC_OK;
}

int check_dense_out(const tlc_tensor* t, const int64_t* sizes, int nd, const char* name) {
    if (!t) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + " is NULL");
    if (t->ndim != nd) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": wrong rank");
    int64_t n = 1;
    for (int i = 0; i < nd; ++i) {
        if (t->sizes[i] != sizes[i]) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": wrong shape");
        n *= sizes[i];
    }
    if (!dense(t)) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + " must be contiguous");
    if (n > 0 && !t->data) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": NULL data");
    return TLC_OK;
}

// col [N, groups, patch, HW] of a dense input
int make_col(const float* in, const ConvShape& s, Buf& col, cudaStream_t st) {
    const int64_t n = s.N * s.groups * s.patch * s.HW;
    TLC_TRY(scratch_alloc(&col.p, sizeof(float) * (size_t)std::max<int64_t>(n, 1), st));
    if (n) {
        const int64_t lines = s.N * s.groups * s.patch;
        const int64_t plane_bytes = s.H * s.W * (int64_t)sizeof(float);
        if (s.W_out % 4 == 0 && s.W_out / 4 <= 256 && plane_bytes <= kIm2colPlaneMax) {
            static DeviceOnce once;  // function attributes are per device
            TLC_TRY(smem_limit_once(once, im2col_plane_kernel, kIm2colPlaneMax));
            im2col_plane_kernel<<<(unsigned)std::min<int64_t>(s.N * s.C_in, 148 * 16), 256, (size_t)plane_bytes,
                                  st>>>(in, col.f(), s);
        } else if (s.W_out % 4 == 0)
            im2col_vec4_kernel<<<(unsigned)std::min<int64_t>(lines, 148 * 64), 256, 0, st>>>(in, col.f(), s);
        else
            im2col_kernel<<<(unsigned)std::min<int64_t>(lines, 148 * 64), 256, 0, st>>>(in, col.f(), s);
        count_launch();
        TLC_TRY(check_launch("im2col"));
    }
    return TLC_OK;
}

// colT [N, groups, HW, patch] of a dense input, or TLC_ERR_UNSUPPORTED when a
// block's staged rows would not fit in shared memory.
constexpr int kIm2colTMax = 96 * 1024;
int make_col_t(const float* in, const ConvShape& s, Buf& col, cudaStream_t st) {
    const int64_t span = (s.W_out - 1) * s.stride + s.kW;
    const int64_t bytes = s.C_in_g * s.kH * span * (int64_t)sizeof(float);
    if (s.W_out < 1 || bytes > kIm2colTMax || s.patch > INT32_MAX / 2) return TLC_ERR_UNSUPPORTED;
    const int64_t n = s.N * s.groups * s.patch * s.HW;
    TLC_TRY(scratch_alloc(&col.p, sizeof(float) * (size_t)std::max<int64_t>(n, 1), st));
    if (n) {
        static DeviceOnce once;
        TLC_TRY(smem_limit_once(once, im2col_t_kernel, kIm2colTMax));
        im2col_t_kernel<<<(unsigned)std::min<int64_t>(s.N * s.groups * s.H_out, 148 * 16), 256, (size_t)bytes,
                          st>>>(in, col.f(), s, (int)span);
        count_launch();
        TLC_TRY(check_launch("im2col (transposed)"));
    }
    return TLC_OK;
}

// ---- implicit-GEMM convolution (TF32 / 3xTF32, stride 1) -----------------------------
//
// The column buffer of im2col is replaced by TMA boxes of an NHWC copy of the
// input (gemm_tc_conv): for tap (kh, kw) and 32 input channels, an output row
// of W_out pixels is one box starting at input column kw - pad of input row
// oh - pad + kh, zero-filled where it reaches past the image (the padding).
// The weights are repacked to [C_out][kh][kw][channels rounded up to 32]
// (zero past the group's channels) so that the GEMM's k order is (kh, kw, c).
// The input gradient at stride 1 is the same convolution of dO with the
// flipped, transposed weights and padding k - 1 - p.  Exact mode keeps
// im2col, whose k order is the reference's.

// y[n][p][c] = x[n][c][p] (NCHW -> NHWC, p = h * W + w).  split 1: also
// lo = x - trunc_tf32(x); split 2: y = round_tf32(x), lo = x - y (the 3xTF32
// planes of the B operand; hi is y).
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y,
                                    float* __restrict__ lo, int64_t C, int64_t P, int split) {
    __shared__ float t[32][33];
    const int64_t n = blockIdx.z, p0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
    const float* xi = x + n * C * P;
    for (int k = 0; k < 32; k += 8) {
        const int64_t c = c0 + threadIdx.y + k, p = p0 + threadIdx.x;
        t[threadIdx.y + k][threadIdx.x] = (c < C && p < P) ? xi[c * P + p] : 0.0f;
    }
    __syncthreads();
    for (int k = 0; k < 32; k += 8) {
        const int64_t p = p0 + threadIdx.y + k, c = c0 + threadIdx.x;
        if (p >= P || c >= C) continue;
        float v = t[threadIdx.x][threadIdx.y + k];
        const int64_t o = (n * P + p) * C + c;
        if (split == 1) {
            lo[o] = __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xFFFFE000u));
        } else if (split == 2) {
            uint32_t h;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
            lo[o] = __fsub_rn(v, __uint_as_float(h));
            v = __uint_as_float(h);
        }
        y[o] = v;
    }
}

// The same transpose in tiles of 32 channels x 128 pixels with float4 loads
// and stores (C and P multiples of 4, 16-byte aligned tensors).  In a warp the
// loads cover 4 channel rows x 128 bytes and the stores 4 pixels x 32
// channels; the shared tile's odd pitch keeps both phases free of bank
// conflicts.
constexpr int kT4C = 32, kT4P = 128;
// One tile (image n, pixel tile bx, channel tile by) of that transpose, by a
// block of 256 threads, staged in `t`.  With `bsum`, the tile's channel sums
// over its pixels go to bsum[(n * bx_n + bx) * C + c]: warp w adds pixels
// 16w .. 16w + 15 in order, then warp 0 the eight warp sums in order.
__device__ __forceinline__ void nhwc_v4_tile(float (*t)[kT4P + 1], const float* __restrict__ x, float* __restrict__ y,
                                             float* __restrict__ lo, int64_t C, int64_t P, int split, int64_t n,
                                             int64_t bx, int64_t by, float* __restrict__ bsum = nullptr,
                                             int64_t bx_n = 0) {
    const int64_t p0 = bx * kT4P, c0 = by * kT4C;
    const float* xi = x + n * C * P;
    const int tid = threadIdx.x, lane = tid & 31;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int wl = i * 8 + (tid >> 5);  // 0 .. 31
        const int row = (wl & 7) * 4 + (lane >> 3), col4 = (wl >> 3) * 8 + (lane & 7);
        const int64_t c = c0 + row, p = p0 + 4 * col4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < C && p < P) v = __ldg(reinterpret_cast<const float4*>(xi + c * P + p));
        t[row][4 * col4] = v.x;
        t[row][4 * col4 + 1] = v.y;
        t[row][4 * col4 + 2] = v.z;
        t[row][4 * col4 + 3] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int pp = (tid >> 3) + 32 * i, c4 = tid & 7;
        const int64_t p = p0 + pp, c = c0 + 4 * c4;
        if (p >= P || c >= C) continue;
        float v[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] = t[4 * c4 + e][pp];
            l[e] = 0.0f;
            if (split == 1) {
                l[e] = __fsub_rn(v[e], __uint_as_float(__float_as_uint(v[e]) & 0xFFFFE000u));
            } else if (split == 2) {
                uint32_t h;
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v[e]));
                l[e] = __fsub_rn(v[e], __uint_as_float(h));
                v[e] = __uint_as_float(h);
            }
        }
        const int64_t o = (n * P + p) * C + c;
        *reinterpret_cast<float4*>(y + o) = make_float4(v[0], v[1], v[2], v[3]);
        if (split) *reinterpret_cast<float4*>(lo + o) = make_float4(l[0], l[1], l[2], l[3]);
    }
    if (bsum) {
        // the tile is zero past P and C; lane = channel row, so the reads of
        // one warp fall in 32 different banks (odd pitch)
        __shared__ float red[8][kT4C];
        const int w = tid >> 5;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) acc = __fadd_rn(acc, t[lane][16 * w + j]);
        red[w][lane] = acc;
        __syncthreads();
        if (w == 0 && c0 + lane < C) {
            float r = red[0][lane];
#pragma unroll
            for (int k = 1; k < 8; ++k) r = __fadd_rn(r, red[k][lane]);
            bsum[(n * bx_n + bx) * C + c0 + lane] = r;
        }
    }
}

__global__ void __launch_bounds__(256) nchw_to_nhwc_v4_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                              float* __restrict__ lo, int64_t C, int64_t P,
                                                              int split) {
    __shared__ float t[kT4C][kT4P + 1];
    nhwc_v4_tile(t, x, y, lo, C, P, split, blockIdx.z, blockIdx.x, blockIdx.y);
}

// Weights as the implicit GEMM's A: dst[r][kh][kw][q], q < q_pad (zero past
// the real count).  flip 0 (forward): r = output channel o, q = input
// channel c of o's group: W[o][q][kh][kw].  flip 1 (input gradient): r =
// input channel g * C_in_g + c, q = output channel o of group g:
// W[g * C_out_g + q][c][kH - 1 - kh][kW - 1 - kw].
// Elements first, first + step, .. of that repack.
template <typename I>
__device__ __forceinline__ void conv_weights_range(const float* __restrict__ w, float* __restrict__ dst,
                                                   const ConvShape& s, int flip, int64_t q_pad_, I first, I step) {
    const I kH = (I)s.kH, kW = (I)s.kW, khw = kH * kW, q_pad = (I)q_pad_;
    const I C_in_g = (I)s.C_in_g, C_out_g = (I)s.C_out_g;
    const I rows = (I)(flip ? s.C_in : s.C_out), per_row = khw * q_pad;
    const I n = rows * per_row;
    for (I i = first; i < n; i += step) {
        const I r = i / per_row, rem = i - r * per_row;
        const I tap = rem / q_pad, q = rem - tap * q_pad;
        const I kh = tap / kW, kw = tap - kh * kW;
        float v = 0.0f;
        if (!flip) {
            if (q < C_in_g) v = w[((int64_t)r * C_in_g + q) * khw + kh * kW + kw];
        } else if (q < C_out_g) {
            const I g = r / C_in_g, c = r - g * C_in_g;
            v = w[(((int64_t)g * C_out_g + q) * C_in_g + c) * khw + (kH - 1 - kh) * kW + (kW - 1 - kw)];
        }
        dst[i] = v;
    }
}

template <typename I>
__global__ void conv_weights_kernel(const float* __restrict__ w, float* __restrict__ dst, ConvShape s,
                                    int flip, int64_t q_pad) {
    conv_weights_range<I>(w, dst, s, flip, q_pad, (I)blockIdx.x * (I)blockDim.x + (I)threadIdx.x,
                          (I)gridDim.x * (I)blockDim.x);
}

// The preparation of an implicit convolution in one launch: up to two NCHW ->
// NHWC transposes (float4 tiles) and one weight repack (32-bit indices).
// Blocks [0, t[0].blocks) take the first transpose's tiles, the next t[1].blocks
// the second's, the rest stride over the weights.
struct NhwcTask {
    const float* x;
    float* y;
    float* lo;
    float* bsum;  // optional: per-tile channel sums (the bias gradient's partials)
    int64_t C, P;
    int split;
    int64_t bx_n, by_n, blocks;  // tiles along pixels, channels; bx_n * by_n * images
};
struct ConvPrep {
    NhwcTask t[2];
    int nt;
    const float* w;
    float* wdst;
    int flip;
    int64_t q_pad;
    int64_t w_blocks;
};
__global__ void __launch_bounds__(256) conv_prep_kernel(const __grid_constant__ ConvPrep p, ConvShape s) {
    __shared__ float t[kT4C][kT4P + 1];
    int64_t b = blockIdx.x;
    for (int k = 0; k < p.nt; ++k) {
        const NhwcTask& q = p.t[k];
        if (b < q.blocks) {
            const int64_t bx = b % q.bx_n, r = b / q.bx_n;
            nhwc_v4_tile(t, q.x, q.y, q.lo, q.C, q.P, q.split, r / q.by_n, bx, r % q.by_n, q.bsum, q.bx_n);
            return;
        }
        b -= q.blocks;
    }
    if (p.w) conv_weights_range<int>(p.w, p.wdst, s, p.flip, p.q_pad, (int)b * 256 + (int)threadIdx.x,
                                     (int)p.w_blocks * 256);
}

// conv_weights_kernel over nwp elements, in 32-bit index math when that fits
void launch_conv_weights(const float* w, float* dst, const ConvShape& s, int flip, int64_t q_pad, int64_t nwp,
                         cudaStream_t st) {
    const unsigned grid = (unsigned)std::min<int64_t>((nwp + 255) / 256, 148 * 16);
    if (nwp < (int64_t(1) << 31) - 148 * 16 * 256)
        conv_weights_kernel<int><<<grid, 256, 0, st>>>(w, dst, s, flip, q_pad);
    else
        conv_weights_kernel<int64_t><<<grid, 256, 0, st>>>(w, dst, s, flip, q_pad);
}

int64_t round32(int64_t v) { return (v + 31) / 32 * 32; }

// grad_w[g * C_out_g + o][c][kh][kw] = the sum over splits of
// part[s][g][o][(kh * kW + kw) * c_pad + c] (the implicit weight-gradient
// GEMM's partial sums).  A block takes 32 outputs (lane = output, consecutive
// channels of one tap); its 8 warps each add one contiguous eighth of the
// splits in order, and warp 0 adds the eight partial sums in order: the same
// sums on every run.  Blocks [0, dw_blocks) do that; the ones after, with
// b.part set, finish the bias gradient: grad_bias[c] = the sum of
// b.part[k * C_out + c] over k < b.count (a warp per channel, lane-strided
// runs in order, then a fixed shuffle tree).
struct BiasFinish {
    const float* part;
    float* out;
    int64_t count;
};
__global__ void __launch_bounds__(256) conv_dw_reduce_kernel(const float* __restrict__ part,
                                                             float* __restrict__ gw, ConvShape s,
                                                             int64_t splits, int64_t c_pad, int64_t dw_blocks,
                                                             BiasFinish b) {
    __shared__ float red[8][32];
    if (blockIdx.x >= dw_blocks) {
        const int64_t c = (blockIdx.x - dw_blocks) * 8 + (threadIdx.x >> 5);
        const int lane = threadIdx.x & 31;
        if (!b.part || c >= s.C_out) return;
        float acc = 0.0f;
        for (int64_t k = lane; k < b.count; k += 32) acc = __fadd_rn(acc, __ldg(b.part + k * s.C_out + c));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0) b.out[c] = acc;
        return;
    }
    const int64_t taps = s.kH * s.kW, cols = taps * c_pad;
    const int64_t n = s.C_out * taps * s.C_in_g;
    const int64_t split_stride = s.C_out * cols;  // groups * C_out_g * cols
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t per = (splits + 7) / 8, k0 = warp * per, k1 = min(splits, k0 + per);
    for (int64_t base = blockIdx.x * (int64_t)32; base < n; base += dw_blocks * 32) {
        const int64_t i = base + lane;
        float acc = 0.0f;
        int64_t row = 0, tap = 0, c = 0;
        if (i < n) {
            // i = (row, tap, c), c fastest; row = g * C_out_g + o
            c = i % s.C_in_g;
            const int64_t rt = i / s.C_in_g;
            tap = rt % taps;
            row = rt / taps;
            const float* src = part + row * cols + tap * c_pad + c;
            for (int64_t k = k0; k < k1; ++k) acc = __fadd_rn(acc, __ldg(src + k * split_stride));
        }
        red[warp][lane] = acc;
        __syncthreads();
        if (warp == 0 && i < n) {
            float t = red[0][lane];
#pragma unroll
            for (int w = 1; w < 8; ++w) t = __fadd_rn(t, red[w][lane]);
            gw[(row * s.C_in_g + c) * taps + tap] = t;
        }
        __syncthreads();
    }
}

// Output rows per implicit-GEMM tile for an output row width: the most rows
// whose pixels fit `cap` columns as a multiple of 16 (0: none fits).
int conv_tile_rows(int64_t width, int cap) {
    if (width <= 0 || width % 8) return 0;
    for (int64_t r = cap / width; r >= 1; --r)
        if ((r * width) % 16 == 0) return (int)r;
    return 0;
}

// Whether a convolution of `C` input channels (C_g per group) over planes of
// H x W giving rows of `out_w` runs as an implicit GEMM in this mode.
bool conv_tma_ok(const ConvShape& s, int64_t C, int64_t C_g, int64_t H, int64_t W, int64_t out_w,
                 int mode) {
    const int64_t lim = int64_t(1) << 30;
    return mode != TLC_MODE_EXACT && s.stride == 1 && C % 4 == 0 &&
           (s.groups == 1 || C_g % 32 == 0) && H < lim && W < lim && C < lim && s.N < lim &&
           s.N <= 65535 && conv_tile_rows(out_w, mode == TLC_MODE_3XTF32 ? 128 : 256) > 0 &&
           s.kH * s.kW * round32(C_g) < lim;
}

// Whether the weight gradient runs as the implicit split-K GEMM in this mode.
bool conv_dw_ok(const ConvShape& s, const float* go, int mode) {
    const int64_t lim = int64_t(1) << 30;
    return mode != TLC_MODE_EXACT && s.stride == 1 && s.W_out >= 8 && s.W_out % 8 == 0 &&
           s.C_in % 4 == 0 && (s.groups == 1 || s.C_in_g % 32 == 0) &&
           (reinterpret_cast<uintptr_t>(go) & 15) == 0 && s.H < lim && s.W < lim && s.C_in < lim &&
           s.C_out < lim && s.N * s.H_out < lim && s.kH * s.kW * round32(s.C_in_g) < lim;
}

// NHWC copy (and 3xTF32 lo plane) of a dense NCHW tensor [N, C, H*W].
int to_nhwc(const float* x, int64_t N, int64_t C, int64_t P, int mode, Buf& hi, Buf& lo,
            cudaStream_t st) {
    const int64_t n = N * C * P;
    int split = 0;
    if (mode == TLC_MODE_3XTF32) split = tf32_reads_truncated(st) ? 1 : 2;
    TLC_TRY(scratch_alloc(&hi.p, sizeof(float) * (size_t)std::max<int64_t>(n, 1), st));
    if (split) TLC_TRY(scratch_alloc(&lo.p, sizeof(float) * (size_t)std::max<int64_t>(n, 1), st));
    if (!n) return TLC_OK;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (C % 4 == 0 && P % 4 == 0 && a16(x) && a16(hi.p) && (!split || a16(lo.p))) {
        dim3 grid((unsigned)((P + kT4P - 1) / kT4P), (unsigned)((C + kT4C - 1) / kT4C), (unsigned)N);
        nchw_to_nhwc_v4_kernel<<<grid, 256, 0, st>>>(x, hi.f(), split ? lo.f() : nullptr, C, P, split);
    } else {
        dim3 grid((unsigned)((P + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)N);
        nchw_to_nhwc_kernel<<<grid, dim3(32, 8), 0, st>>>(x, hi.f(), split ? lo.f() : nullptr, C, P, split);
    }
    count_launch();
    return check_launch("nchw_to_nhwc");
}

// Allocates the NHWC copy (and 3xTF32 lo plane) of a dense NCHW tensor
// [N, C, H*W]; when the float4 tile transpose applies, describes it in *t for
// a combined launch (*deferred = true), else launches the general transpose.
int prep_nhwc(const float* x, int64_t N, int64_t C, int64_t P, int mode, Buf& hi, Buf& lo, cudaStream_t st,
              NhwcTask* t, bool* deferred) {
    *deferred = false;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const int64_t n = N * C * P;
    if (!(n > 0 && C % 4 == 0 && P % 4 == 0 && a16(x))) return to_nhwc(x, N, C, P, mode, hi, lo, st);
    int split = 0;
    if (mode == TLC_MODE_3XTF32) split = tf32_reads_truncated(st) ? 1 : 2;
    TLC_TRY(scratch_alloc(&hi.p, sizeof(float) * (size_t)n, st));
    if (split) TLC_TRY(scratch_alloc(&lo.p, sizeof(float) * (size_t)n, st));
    if (!a16(hi.p) || (split && !a16(lo.p))) {
        dim3 grid((unsigned)((P + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)N);
        nchw_to_nhwc_kernel<<<grid, dim3(32, 8), 0, st>>>(x, hi.f(), split ? lo.f() : nullptr, C, P, split);
        count_launch();
        return check_launch("nchw_to_nhwc");
    }
    t->x = x;
    t->y = hi.f();
    t->lo = split ? lo.f() : nullptr;
    t->bsum = nullptr;
    t->C = C;
    t->P = P;
    t->split = split;
    t->bx_n = (P + kT4P - 1) / kT4P;
    t->by_n = (C + kT4C - 1) / kT4C;
    t->blocks = t->bx_n * t->by_n * N;
    *deferred = true;
    return TLC_OK;
}

// Launches a ConvPrep: its transposes and, if p.w is set, the weight repack of
// nwp elements (a repack too large for 32-bit indices goes alone).
int launch_prep(ConvPrep& p, int64_t nwp, const ConvShape& s, cudaStream_t st) {
    if (p.w && nwp >= (int64_t(1) << 31) - 148 * 4 * 256) {
        launch_conv_weights(p.w, p.wdst, s, p.flip, p.q_pad, nwp, st);
        count_launch();
        TLC_TRY(check_launch("conv weights"));
        p.w = nullptr;
    }
    p.w_blocks = p.w ? std::max<int64_t>(1, std::min<int64_t>((nwp + 255) / 256, 148 * 4)) : 0;
    int64_t blocks = p.w_blocks;
    for (int k = 0; k < p.nt; ++k) blocks += p.t[k].blocks;
    if (blocks == 0) return TLC_OK;
    if (blocks > INT32_MAX) return set_error(TLC_ERR_UNSUPPORTED, "conv2d: too many transpose tiles");
    conv_prep_kernel<<<(unsigned)blocks, 256, 0, st>>>(p, s);
    count_launch();
    return check_launch("conv prep");
}

// out[n, g] (M x H_o * W_o) = A[g] . im2col(x_nhwc[n, g]) as an implicit GEMM.
// x_nhwc / x_nhwc_lo: the NHWC copy (and lo plane) of x, made already.
int conv_tma_gemm(const float* x_nhwc, const float* x_nhwc_lo, int64_t C, int64_t C_g, int64_t H, int64_t W,
                  const float* a, int64_t M, int64_t H_o, int64_t W_o, int64_t pad_h, int64_t pad_w, float* out,
                  int64_t out_img, const float* bias, const ConvShape& s, int mode, cudaStream_t st) {
    const int64_t c_pad = round32(C_g), K = s.kH * s.kW * c_pad, P = H_o * W_o;
    Gemm g{};
    g.M = M;
    g.N = P;
    g.K = K;
    g.A = a;
    g.a_rs = K;
    g.a_cs = 1;
    g.C = out;
    g.c_rs = P;
    g.nb = 2;
    g.bsz[0] = s.N;
    g.bsz[1] = s.groups;
    g.abs_[0] = 0;
    g.abs_[1] = M * K;
    g.cbs[0] = out_img;
    g.cbs[1] = M * P;
    ConvTma c{};
    c.x = x_nhwc;
    c.x_lo = mode == TLC_MODE_3XTF32 ? x_nhwc_lo : nullptr;
    c.N = (int)s.N;
    c.H = (int)H;
    c.W = (int)W;
    c.C = (int)C;
    c.W_out = (int)W_o;
    c.rows = conv_tile_rows(W_o, mode == TLC_MODE_3XTF32 ? 128 : 256);
    c.kH = (int)s.kH;
    c.kW = (int)s.kW;
    c.pad_h = (int)pad_h;
    c.pad_w = (int)pad_w;
    c.cblocks = (int)(c_pad / 32);
    c.c_group = (int)C_g;
    if (bias) {
        c.row_bias = bias;
        c.row_bias_group = M;
    }
    return gemm_tc_conv(g, c, mode, st);
}

int forward(const tlc_tensor* in_t, const tlc_tensor* w_t, const tlc_tensor* bias, int64_t stride,
            int64_t padding, int64_t groups, tlc_tensor* out, int mode, cudaStream_t st) {
    ConvShape s;
    TLC_TRY(conv_shape(in_t, w_t, stride, padding, groups, s));
    const int64_t osz[4] = {s.N, s.C_out, s.H_out, s.W_out};
    TLC_TRY(check_dense_out(out, osz, 4, "out"));
    const tlc_tensor* b = (bias && bias->ndim > 0) ? bias : nullptr;
    if (b) {
        int64_t nb = 1;
        for (int i = 0; i < b->ndim; ++i) nb *= b->sizes[i];
        if (nb != s.C_out)  // reshape(bias, {1, C_out, 1, 1}), src/ops.cpp:1524
            return set_error(TLC_ERR_INVALID_ARGUMENT, "reshape: new shape must have same number of elements");
    }
    if (s.N * s.C_out * s.HW == 0) return TLC_OK;
    Buf bin(st), bw(st), col(st), bb(st);
    const float *in, *w;
    TLC_TRY(dense_copy(in_t, bin, &in, st));
    TLC_TRY(dense_copy(w_t, bw, &w, st));
    if (s.patch > 0 && conv_tma_ok(s, s.C_in, s.C_in_g, s.H, s.W, s.W_out, mode)) {
        // implicit GEMM: no column buffer; the bias (one value per output
        // channel: a GEMM row) added in the epilogue, the same fp32 add
        // the NHWC copy of the input and the repacked weights in one launch
        const int64_t q_pad = round32(s.C_in_g), nwp = s.C_out * s.kH * s.kW * q_pad;
        Buf wp(st), xh(st), xl(st);
        TLC_TRY(scratch_alloc(&wp.p, sizeof(float) * (size_t)nwp, st));
        ConvPrep cp{};
        bool deferred = false;
        TLC_TRY(prep_nhwc(in, s.N, s.C_in, s.H * s.W, mode, xh, xl, st, &cp.t[0], &deferred));
        cp.nt = deferred ? 1 : 0;
        cp.w = w;
        cp.wdst = wp.f();
        cp.flip = 0;
        cp.q_pad = q_pad;
        TLC_TRY(launch_prep(cp, nwp, s, st));
        const float* bd = nullptr;
        if (b) TLC_TRY(dense_copy(b, bb, &bd, st));
        return conv_tma_gemm(xh.f(), xl.f(), s.C_in, s.C_in_g, s.H, s.W, wp.f(), s.C_out_g, s.H_out, s.W_out,
                             s.padding, s.padding, out->data, s.C_out * s.HW, bd, s, mode, st);
    }
    TLC_TRY(make_col(in, s, col, st));
    // out[n, g] (C_out_g x HW) = W_g (C_out_g x patch) . col[n, g] (patch x HW)
    Gemm g{};
    g.M = s.C_out_g;
    g.N = s.HW;
    g.K = s.patch;
    g.A = w;
    g.a_rs = s.patch;
    g.a_cs = 1;
    g.B = col.f();
    g.b_rs = s.HW;
    g.b_cs = 1;
    g.C = out->data;
    g.c_rs = s.HW;
    g.nb = 2;
    g.bsz[0] = s.N;
    g.bsz[1] = s.groups;
    g.abs_[0] = 0;
    g.abs_[1] = s.C_out_g * s.patch;
    g.bbs[0] = s.groups * s.patch * s.HW;
    g.bbs[1] = s.patch * s.HW;
    g.cbs[0] = s.C_out * s.HW;
    g.cbs[1] = s.C_out_g * s.HW;
    TLC_TRY(gemm(g, mode, st));
    if (b) {
        // add(result, reshape(bias, {1, C_out, 1, 1})): in place, out = out + bias[c]
        const float* bd;
        TLC_TRY(dense_copy(b, bb, &bd, st));
        const int64_t sz[3] = {s.N, s.C_out, s.HW};
        const int64_t sa[3] = {s.C_out * s.HW, s.HW, 1}, sbias[3] = {0, 1, 0};
        TLC_TRY(launch_elementwise(out->data, bd, 0.0f, out->data, s.N * s.C_out * s.HW, 3, sz, sa, sbias,
                                   0, st));
    }
    return TLC_OK;
}

int backward(const tlc_tensor* go_t, const tlc_tensor* in_t, const tlc_tensor* w_t, int64_t stride,
             int64_t padding, int64_t groups, tlc_tensor* d_in, tlc_tensor* d_w, tlc_tensor* d_b, int mode,
             cudaStream_t st) {
    ConvShape s;
    TLC_TRY(conv_shape(in_t, w_t, stride, padding, groups, s));
    const int64_t osz[4] = {s.N, s.C_out, s.H_out, s.W_out};
    if (!go_t || go_t->ndim != 4)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d_backward: grad_output must be 4-D");
    for (int i = 0; i < 4; ++i)
        if (go_t->sizes[i] != osz[i])
            return set_error(TLC_ERR_INVALID_ARGUMENT, "conv2d_backward: grad_output has the wrong shape");
    if (d_in) TLC_TRY(check_dense_out(d_in, in_t->sizes, 4, "d_input"));
    if (d_w) TLC_TRY(check_dense_out(d_w, w_t->sizes, 4, "d_weight"));
    const int64_t bsz[1] = {s.C_out};
    if (d_b) TLC_TRY(check_dense_out(d_b, bsz, 1, "d_bias"));
    Buf bgo(st), bin(st), bw(st), col(st), prod(st), gcol(st), bpart(st);
    const float *go, *in, *w;
    TLC_TRY(dense_copy(go_t, bgo, &go, st));
    TLC_TRY(dense_copy(in_t, bin, &in, st));
    TLC_TRY(dense_copy(w_t, bw, &w, st));
    // Exact mode's bias gradient is one dependent chain of N * HW adds per
    // channel (the reference's order): it runs on a side stream from the
    // start, beside the weight- and input-gradient GEMMs, which leave SMs
    // free for its one block per channel (the join is in `fork`'s destructor,
    // before the buffers above are freed).
    Fork fork(st);
    bool bias_done = false;
    if (d_b && s.C_out && (mode == TLC_MODE_EXACT || s.N * s.HW == 0)) {
        cudaStream_t bs = fork.begin();
        if (!bs) bs = st;
        bias_grad_kernel<<<(unsigned)std::min<int64_t>(s.C_out, 148 * 16), BIAS_THREADS, 0, bs>>>(go, d_b->data, s);
        count_launch();
        TLC_TRY(check_launch("conv bias grad"));
        bias_done = true;
    }
    const bool dw_implicit = d_w && s.N * s.C_out * s.patch != 0 && s.HW > 0 && conv_dw_ok(s, go, mode);
    const bool dx_implicit = d_in && s.N * s.C_in * s.H * s.W > 0 && s.kH - 1 - s.padding >= 0 &&
                             s.kW - 1 - s.padding >= 0 &&
                             conv_tma_ok(s, s.C_out, s.C_out_g, s.H_out, s.W_out, s.W, mode);
    // The implicit GEMMs' operand copies in one launch: the input in NHWC
    // (weight gradient), dO in NHWC and the flipped, transposed weights
    // (input gradient).  The dO tiles also write the bias gradient's partial
    // sums (per image, 128-pixel run and channel), which the weight-gradient
    // sum launch (or a launch of its own) then adds in order.
    Buf xh(st), xl(st), gh(st), gl(st);
    const int64_t dx_q_pad = round32(s.C_out_g), dx_nwp = s.C_in * s.kH * s.kW * dx_q_pad;
    BiasFinish bias_fin{};
    if (dw_implicit || dx_implicit) {
        ConvPrep cp{};
        bool deferred = false;
        if (dw_implicit) {
            TLC_TRY(prep_nhwc(in, s.N, s.C_in, s.H * s.W, mode, xh, xl, st, &cp.t[cp.nt], &deferred));
            cp.nt += deferred ? 1 : 0;
        }
        if (dx_implicit) {
            TLC_TRY(prep_nhwc(go, s.N, s.C_out, s.H_out * s.W_out, mode, gh, gl, st, &cp.t[cp.nt], &deferred));
            if (deferred && d_b && s.C_out && !bias_done) {
                NhwcTask& q = cp.t[cp.nt];
                const int64_t count = s.N * q.bx_n;
                TLC_TRY(scratch_alloc(&bpart.p, sizeof(float) * (size_t)(count * s.C_out), st));
                q.bsum = bpart.f();
                bias_fin.part = bpart.f();
                bias_fin.out = d_b->data;
                bias_fin.count = count;
            }
            cp.nt += deferred ? 1 : 0;
            TLC_TRY(scratch_alloc(&gcol.p, sizeof(float) * (size_t)dx_nwp, st));
            cp.w = w;
            cp.wdst = gcol.f();
            cp.flip = 1;
            cp.q_pad = dx_q_pad;
        }
        TLC_TRY(launch_prep(cp, dx_implicit ? dx_nwp : 0, s, st));
    }
    if (d_w) {
        // G[n, g] (C_out_g x patch) = dO[n, g] (C_out_g x HW) . col[n, g]^T, then sum over n
        if (s.N * s.C_out * s.patch == 0) {
            if (s.C_out * s.patch) TLC_TRY(launch_fill_zero(d_w->data, s.C_out * s.patch, st));
        } else if (dw_implicit) {
            // implicit split-K GEMM over TMA boxes of dO and of an NHWC copy
            // of the input (no column buffer), then the ordered sum of the splits
            ConvDw c{};
            c.go = go;
            c.x = xh.f();
            c.x_lo = mode == TLC_MODE_3XTF32 ? xl.f() : nullptr;
            c.N = (int)s.N;
            c.C = (int)s.C_in;
            c.H = (int)s.H;
            c.W = (int)s.W;
            c.C_out = (int)s.C_out;
            c.H_out = (int)s.H_out;
            c.W_out = (int)s.W_out;
            c.kH = (int)s.kH;
            c.kW = (int)s.kW;
            c.pad_h = (int)s.padding;
            c.pad_w = (int)s.padding;
            c.groups = (int)s.groups;
            c.C_in_g = (int)s.C_in_g;
            c.C_out_g = (int)s.C_out_g;
            int splits = 0, rows = 0;
            TLC_TRY(conv_dw_splits(c, mode, &splits, &rows));
            const int64_t c_pad = round32(s.C_in_g);
            TLC_TRY(scratch_alloc(&prod.p, sizeof(float) * (size_t)(splits * s.C_out * s.kH * s.kW * c_pad), st));
            TLC_TRY(gemm_tc_conv_dw(c, splits, rows, prod.f(), mode, st));
            const int64_t n = s.C_out * s.patch, dw_blocks = std::min<int64_t>((n + 31) / 32, 148 * 32);
            const int64_t b_blocks = bias_fin.part ? (s.C_out + 7) / 8 : 0;
            conv_dw_reduce_kernel<<<(unsigned)(dw_blocks + b_blocks), 256, 0, st>>>(prod.f(), d_w->data, s, splits,
                                                                                  c_pad, dw_blocks, bias_fin);
            count_launch();
            TLC_TRY(check_launch("conv weight-gradient sum"));
            if (bias_fin.part) bias_done = true;
        } else {
            // exact mode: the column buffer transposed ([HW, patch] per image and
            // group), so the FFMA GEMM reads an N-major B (its packed path);
            // otherwise, or when its rows do not fit, col read transposed in place
            bool transposed = false;
            if (mode == TLC_MODE_EXACT) {
                const int r = make_col_t(in, s, col, st);
                if (r != TLC_OK && r != TLC_ERR_UNSUPPORTED) return r;
                transposed = r == TLC_OK;
            }
            if (!transposed) TLC_TRY(make_col(in, s, col, st));
            TLC_TRY(scratch_alloc(&prod.p, sizeof(float) * (size_t)(s.N * s.C_out * s.patch), st));
            Gemm g{};
            g.M = s.C_out_g;
            g.N = s.patch;
            g.K = s.HW;
            g.A = go;
            g.a_rs = s.HW;
            g.a_cs = 1;
            g.B = col.f();  // (hw, p) at hw*patch + p (colT), or at p*HW + hw (col)
            g.b_rs = transposed ? s.patch : 1;
            g.b_cs = transposed ? 1 : s.HW;
            g.C = prod.f();
            g.c_rs = s.patch;
            g.nb = 2;
            g.bsz[0] = s.N;
            g.bsz[1] = s.groups;
            g.abs_[0] = s.C_out * s.HW;
            g.abs_[1] = s.C_out_g * s.HW;
            g.bbs[0] = s.groups * s.patch * s.HW;
            g.bbs[1] = s.patch * s.HW;
            g.cbs[0] = s.C_out * s.patch;
            g.cbs[1] = s.C_out_g * s.patch;
            if (s.HW == 0) {
                TLC_TRY(launch_fill_zero(prod.f(), s.N * s.C_out * s.patch, st));
            } else {
                TLC_TRY(gemm(g, mode, st));
            }
            // grad_w = 0 + G[0] + G[1] + ... (the reference's += over images)
            TLC_TRY(launch_sum_dim(prod.f(), d_w->data, 1, s.N, s.C_out * s.patch, st));
        }
    }
    if (dx_implicit) {
        // stride 1: dX = the convolution of dO with the flipped, transposed
        // weights, padding k - 1 - p, as the same implicit GEMM
        TLC_TRY(conv_tma_gemm(gh.f(), gl.f(), s.C_out, s.C_out_g, s.H_out, s.W_out, gcol.f(), s.C_in_g, s.H, s.W,
                              s.kH - 1 - s.padding, s.kW - 1 - s.padding, d_in->data,
                              s.C_in * s.H * s.W, nullptr, s, mode, st));
    } else if (d_in) {
        const int64_t ni = s.N * s.C_in * s.H * s.W;
        if (ni) {
            const int64_t nc = s.N * s.groups * s.patch * s.HW;
            TLC_TRY(scratch_alloc(&gcol.p, sizeof(float) * (size_t)std::max<int64_t>(nc, 1), st));
            if (nc) {
                // grad_col[n, g] (patch x HW) = W_g^T (patch x C_out_g) . dO[n, g] (C_out_g x HW)
                Gemm g{};
                g.M = s.patch;
                g.N = s.HW;
                g.K = s.C_out_g;
                g.A = w;  // W_g read as its transpose: (p, o) at o*patch + p
                g.a_rs = 1;
                g.a_cs = s.patch;
                g.B = go;
                g.b_rs = s.HW;
                g.b_cs = 1;
                g.C = gcol.f();
                g.c_rs = s.HW;
                g.nb = 2;
                g.bsz[0] = s.N;
                g.bsz[1] = s.groups;
                g.abs_[0] = 0;
                g.abs_[1] = s.C_out_g * s.patch;
                g.bbs[0] = s.C_out * s.HW;
                g.bbs[1] = s.C_out_g * s.HW;
                g.cbs[0] = s.groups * s.patch * s.HW;
                g.cbs[1] = s.patch * s.HW;
                TLC_TRY(gemm(g, mode, st));
            }
            const unsigned grid = (unsigned)std::min<int64_t>(s.N * s.C_in, 148 * 64);
            if (s.W % 4 == 0 && (reinterpret_cast<uintptr_t>(d_in->data) & 15) == 0) {
                if (s.stride == 1)
                    col2im_vec4_kernel<true><<<grid, 256, 0, st>>>(gcol.f(), d_in->data, s);
                else
                    col2im_vec4_kernel<false><<<grid, 256, 0, st>>>(gcol.f(), d_in->data, s);
            } else {
                col2im_kernel<<<grid, 256, 0, st>>>(gcol.f(), d_in->data, s);
            }
            count_launch();
            TLC_TRY(check_launch("col2im"));
        }
    }
    if (bias_fin.part && !bias_done) {
        conv_dw_reduce_kernel<<<(unsigned)((s.C_out + 7) / 8), 256, 0, st>>>(nullptr, nullptr, s, 0, 0, 0, bias_fin);
        count_launch();
        TLC_TRY(check_launch("conv bias grad"));
        bias_done = true;
    }
    if (d_b && s.C_out && !bias_done) {
        // TF32 / 3xTF32: a tree, which those modes' tolerance allows
        TLC_TRY(scratch_alloc(&bpart.p, sizeof(float) * (size_t)(s.C_out * s.N), st));
        if (s.HW % 4 == 0 && (reinterpret_cast<uintptr_t>(go) & 15) == 0)
            bias_part_v4_kernel<<<(unsigned)std::min<int64_t>((s.C_out * s.N + 7) / 8, 148 * 32), 256, 0, st>>>(
                go, bpart.f(), s);
        else
            bias_part_kernel<<<(unsigned)std::min<int64_t>(s.C_out * s.N, 148 * 16), 256, 0, st>>>(go, bpart.f(),
                                                                                                   s);
        count_launch();
        TLC_TRY(check_launch("conv bias grad"));
        TLC_TRY(launch_sum_dim(bpart.f(), d_b->data, s.C_out, s.N, 1, st));
    }
    return TLC_OK;
}

}  // namespace
}  // namespace tlc

using namespace tlc;

extern "C" int tlc_conv2d_shape(const tlc_tensor* input, const tlc_tensor* weight, int64_t stride,
                                int64_t padding, int64_t groups, int64_t* out_sizes) {
    clear_error();
    ConvShape s;
    TLC_TRY(conv_shape(input, weight, stride, padding, groups, s));
    if (out_sizes) {
        out_sizes[0] = s.N;
        out_sizes[1] = s.C_out;
        out_sizes[2] = s.H_out;
        out_sizes[3] = s.W_out;
    }
    return TLC_OK;
}

extern "C" int tlc_conv2d(const tlc_tensor* input, const tlc_tensor* weight, const tlc_tensor* bias,
                          int64_t stride, int64_t padding, int64_t groups, tlc_tensor* out, int mode,
                          void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve(mode, m));
    return forward(input, weight, bias, stride, padding, groups, out, m, static_cast<cudaStream_t>(stream));
}

extern "C" int tlc_conv2d_backward(const tlc_tensor* grad_output, const tlc_tensor* input,
                                   const tlc_tensor* weight, int64_t stride, int64_t padding,
                                   int64_t groups, tlc_tensor* d_input, tlc_tensor* d_weight,
                                   tlc_tensor* d_bias, int mode, void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve(mode, m));
    return backward(grad_output, input, weight, stride, padding, groups, d_input, d_weight, d_bias, m,
                    static_cast<cudaStream_t>(stream));
}
