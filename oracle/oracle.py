"""CPU oracle for torchlite-cpp's tl::matmul and MatmulBackward.

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and the CPU
baseline leg of bench.py, always as the checker, never as the product.

The shape logic is a restatement of the reference front end in Python; the
arithmetic runs in the C restatement (oracle/tl_oracle.c -> liboracle.so):

  matmul            src/ops.cpp:605-699  (contiguous, 1-D squeeze, shape checks,
                                          batch broadcast, per-batch GEMM,
                                          unsqueeze of the result)
  broadcast_shape   src/ops.cpp:55-72    (compute_broadcast_shape)
  broadcast_offset  src/ops.cpp:32-52    (get_broadcast_index)
  matmul_backward   src/autograd.cpp:341-384 (MatmulBackward::backward)
  sum_to            src/autograd.cpp:24-36
  sum_dim           src/ops.cpp:1181-1233
  accumulate_grad   src/autograd.cpp:16-22

``tlref`` gives the reference library itself (compiled from its sources into
oracle/_ref by oracle/Makefile) for pinning this restatement.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle)")
        L = ctypes.CDLL(path)
        args = [_f32p, _i64, _i64, _f32p, _i64, _i64, _f32p, _i64, _i64, _i64, _i64, ctypes.c_int]
        L.orc_gemm_chain.argtypes = args
        L.orc_gemm_chain.restype = None
        a64 = list(args)
        a64[6] = _f64p
        L.orc_gemm_f64.argtypes = a64
        L.orc_gemm_f64.restype = None
        L.orc_sum_dim.argtypes = [_f32p, _f32p, _i64, _i64, _i64]
        L.orc_sum_dim.restype = None
        L.orc_add.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.orc_add.restype = None
        L.orc_softmax.argtypes = [_f32p, _f32p, _i64, _i64]
        L.orc_softmax.restype = None
        L.orc_softmax_backward.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64]
        L.orc_softmax_backward.restype = None
        L.orc_flash_attention.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p,
                                          _f32p, _i64]
        L.orc_flash_attention.restype = None
        L.orc_flash_attention_backward.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i64,
                                                   _i64, ctypes.c_float, _f32p, _f32p, _f32p, _i64]
        L.orc_flash_attention_backward.restype = None
        _lib = L
    return _lib


def _fp(x: np.ndarray):
    return x.ctypes.data_as(_f32p)


def default_threads() -> int:
    return max(1, min(64, os.cpu_count() or 1))


def gemm2d(a: np.ndarray, b: np.ndarray, nthreads: int | None = None) -> np.ndarray:
    """One 2-D product C = A.B as the per-element fmaf chain of gemm_blocked
    (src/ops.cpp:242-268).  A and B may be any strided float32 views."""
    assert a.dtype == np.float32 and b.dtype == np.float32 and a.ndim == 2 and b.ndim == 2
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    c = np.empty((M, N), np.float32)
    isz = 4
    lib().orc_gemm_chain(_fp(a), a.strides[0] // isz, a.strides[1] // isz, _fp(b),
                         b.strides[0] // isz, b.strides[1] // isz, _fp(c), N, M, N, K,
                         nthreads or default_threads())
    return c


def gemm2d_f64(a: np.ndarray, b: np.ndarray, nthreads: int | None = None) -> np.ndarray:
    """Double-precision product of float32 operands (error measurement only)."""
    M, K = a.shape
    _, N = b.shape
    c = np.empty((M, N), np.float64)
    isz = 4
    lib().orc_gemm_f64(_fp(a), a.strides[0] // isz, a.strides[1] // isz, _fp(b),
                       b.strides[0] // isz, b.strides[1] // isz,
                       c.ctypes.data_as(_f64p), N, M, N, K, nthreads or default_threads())
    return c


def broadcast_shape(a, b):
    """compute_broadcast_shape, src/ops.cpp:55-72, except that a size-0 dim
    against a size-1 dim gives 0 (NumPy's rule; the reference takes the max, 1,
    and then reads the empty operand out of bounds)."""
    nd = max(len(a), len(b))
    out = []
    for i in range(nd):
        sa = 1 if i < nd - len(a) else a[i - (nd - len(a))]
        sb = 1 if i < nd - len(b) else b[i - (nd - len(b))]
        if sa != sb and sa != 1 and sb != 1:
            raise ValueError("Incompatible dimensions for broadcasting")
        out.append(sb if sa == 1 else sa)
    return out


def _batch_views(x: np.ndarray, batch_out):
    """Yield the 2-D matrix of x used for each flat output batch index, in order
    (get_broadcast_index, src/ops.cpp:32-52: size-1 and missing dims repeat)."""
    bx = list(x.shape[:-2])
    nd = len(batch_out)
    full = [1] * (nd - len(bx)) + bx
    xr = x.reshape(full + list(x.shape[-2:]))
    idx = tuple(np.arange(s) if f != 1 else np.zeros(s, np.int64) for s, f in zip(batch_out, full))
    if nd == 0:
        yield xr
        return
    grid = np.stack(np.meshgrid(*idx, indexing="ij"), -1).reshape(-1, nd)
    for g in grid:
        yield xr[tuple(g)]


def matmul(a: np.ndarray, b: np.ndarray, nthreads: int | None = None) -> np.ndarray:
    """tl::matmul, src/ops.cpp:605-699."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    sq_a = sq_b = False
    if a.ndim == 1:
        a = a.reshape(1, a.shape[0])
        sq_a = True
    if b.ndim == 1:
        b = b.reshape(b.shape[0], 1)
        sq_b = True
    if a.ndim < 2 or b.ndim < 2:
        raise ValueError("matmul: requires at least 1D tensors")
    M, K = a.shape[-2:]
    K2, N = b.shape[-2:]
    if K != K2:
        raise ValueError("Incompatible dimensions for matmul")
    batch_out = broadcast_shape(list(a.shape[:-2]), list(b.shape[:-2]))
    out = np.empty(batch_out + [M, N], np.float32)
    flat = out.reshape(int(np.prod(batch_out, dtype=np.int64)), M, N)
    for i, (av, bv) in enumerate(zip(_batch_views(a, batch_out), _batch_views(b, batch_out))):
        flat[i] = gemm2d(av, bv, nthreads)
    if sq_a and sq_b:
        return out.reshape(())
    if sq_a:
        return out.reshape(batch_out + [N])
    if sq_b:
        return out.reshape(batch_out + [M])
    return out


def sum_dim(x: np.ndarray, dim: int, keepdim: bool) -> np.ndarray:
    """sum(input, dim, keepdim), src/ops.cpp:1181-1233 (sequential, from 0.0f)."""
    x = np.ascontiguousarray(x, np.float32)
    nd = x.ndim
    if dim < 0:
        dim += nd
    if dim < 0 or dim >= nd:
        raise ValueError("sum: dimension out of range")
    outer = int(np.prod(x.shape[:dim], dtype=np.int64))
    D = x.shape[dim]
    inner = int(np.prod(x.shape[dim + 1:], dtype=np.int64))
    shape = [s for i, s in enumerate(x.shape) if i != dim] if not keepdim else \
        [1 if i == dim else s for i, s in enumerate(x.shape)]
    out = np.empty(shape, np.float32)
    lib().orc_sum_dim(_fp(x), _fp(out), outer, D, inner)
    return out


def sum_to(g: np.ndarray, target) -> np.ndarray:
    """sum_to, src/autograd.cpp:24-36."""
    while g.ndim > len(target):
        g = sum_dim(g, 0, False)
    for i, t in enumerate(target):
        if t == 1 and g.shape[i] != 1:
            g = sum_dim(g, i, True)
    return g


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Same-shape add (src/ops.cpp:75-103 without broadcasting)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.empty_like(a)
    lib().orc_add(_fp(a), _fp(b), _fp(out), a.size)
    return out


def add_bcast(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """tl::add with NumPy broadcasting (src/ops.cpp:74-103): one fp32 add per
    output element, operands picked by get_broadcast_index (src/ops.cpp:32-52).
    numpy's float32 add is the same correctly rounded addition."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    broadcast_shape(a.shape, b.shape)  # the reference's error for incompatible shapes
    return np.add(a, b, dtype=np.float32)


def scale(x: np.ndarray, s: float) -> np.ndarray:
    """tl::scale (src/ops.cpp:963-983): out = x * s in fp32."""
    return np.multiply(np.asarray(x, np.float32), np.float32(s), dtype=np.float32)


def softmax(x: np.ndarray) -> np.ndarray:
    """tl::softmax over the last dim (src/ops.cpp:985-1037)."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 0:
        raise ValueError("Softmax requires at least 1D tensor")
    out = np.empty_like(x)
    D = x.shape[-1]
    if D == 0 or x.size == 0:
        return out
    lib().orc_softmax(_fp(x), _fp(out), x.size // D, D)
    return out


def _conv_out(H, W, kH, kW, stride, padding):
    # (H + 2p - kH) / stride + 1 with C++'s truncating division
    def tdiv(a, b):
        return -((-a) // b) if a < 0 else a // b
    return tdiv(H + 2 * padding - kH, stride) + 1, tdiv(W + 2 * padding - kW, stride) + 1


def _im2col(x_n, c0, C_in_g, kH, kW, stride, padding, H_out, W_out):
    """col [C_in_g*kH*kW, H_out*W_out] of image x_n [C_in, H, W], channels
    c0.. (src/ops.cpp:1479-1511): zero outside the image."""
    _, H, W = x_n.shape
    col = np.zeros((C_in_g * kH * kW, H_out * W_out), np.float32)
    oh = np.arange(H_out)[:, None]
    ow = np.arange(W_out)[None, :]
    for c in range(C_in_g):
        for kh in range(kH):
            for kw in range(kW):
                ih = oh * stride - padding + kh
                iw = ow * stride - padding + kw
                ok = (ih >= 0) & (ih < H) & (iw >= 0) & (iw < W)
                v = np.zeros((H_out, W_out), np.float32)
                v[ok] = x_n[c0 + c][np.broadcast_to(ih, ok.shape)[ok], np.broadcast_to(iw, ok.shape)[ok]]
                col[c * kH * kW + kh * kW + kw] = v.reshape(-1)
    return col


def conv2d(x, w, b, stride=1, padding=0, groups=1):
    """conv2d, src/ops.cpp:1443-1548: per image and group, W_g . im2col
    (gemm_blocked's chain), then add(result, bias[1, C_out, 1, 1])."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    N, C_in, H, W = x.shape
    C_out, C_in_g, kH, kW = w.shape
    C_out_g = C_out // groups
    H_out, W_out = _conv_out(H, W, kH, kW, stride, padding)
    wr = np.ascontiguousarray(w.reshape(C_out, -1))
    out = np.zeros((N, C_out, H_out * W_out), np.float32)
    for n in range(N):
        for g in range(groups):
            col = _im2col(x[n], g * C_in_g, C_in_g, kH, kW, stride, padding, H_out, W_out)
            out[n, g * C_out_g:(g + 1) * C_out_g] = gemm2d(wr[g * C_out_g:(g + 1) * C_out_g], col)
    out = out.reshape(N, C_out, H_out, W_out)
    if b is not None and np.asarray(b).size:
        out = np.add(out, np.asarray(b, np.float32).reshape(1, C_out, 1, 1), dtype=np.float32)
    return out


def conv2d_backward(go, x, w, stride=1, padding=0, groups=1):
    """Conv2dBackward, src/autograd.cpp:386-517, then accumulate_grad (0 + d):
    (d_input, d_weight, d_bias)."""
    go = np.asarray(go, np.float32)
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    N, C_in, H, W = x.shape
    C_out, C_in_g, kH, kW = w.shape
    C_out_g = C_out // groups
    H_out, W_out = go.shape[2], go.shape[3]
    patch = C_in_g * kH * kW
    wr = np.ascontiguousarray(w.reshape(C_out, patch))
    gw = np.zeros((C_out, patch), np.float32)
    gi = np.zeros((N, C_in, H, W), np.float32)
    gb = np.zeros((C_out,), np.float32)
    oh = np.arange(H_out)[:, None]
    ow = np.arange(W_out)[None, :]
    for n in range(N):
        go_n = go[n].reshape(C_out, H_out * W_out)
        for g in range(groups):
            go_ng = np.ascontiguousarray(go_n[g * C_out_g:(g + 1) * C_out_g])
            col = _im2col(x[n], g * C_in_g, C_in_g, kH, kW, stride, padding, H_out, W_out)
            band = slice(g * C_out_g, (g + 1) * C_out_g)
            gw[band] = np.add(gw[band], gemm2d(go_ng, np.ascontiguousarray(col.T)), dtype=np.float32)
            gcol = gemm2d(np.ascontiguousarray(wr[band].T), go_ng)
            # col2im in the reference's loop order: per pixel, (kh, kw) ascending
            for kh in range(kH):
                for kw in range(kW):
                    ih = np.broadcast_to(oh * stride - padding + kh, (H_out, W_out))
                    iw = np.broadcast_to(ow * stride - padding + kw, (H_out, W_out))
                    ok = (ih >= 0) & (ih < H) & (iw >= 0) & (iw < W)
                    for c in range(C_in_g):
                        vals = gcol[c * kH * kW + kh * kW + kw].reshape(H_out, W_out)
                        ch = gi[n, g * C_in_g + c]
                        ch[ih[ok], iw[ok]] = np.add(ch[ih[ok], iw[ok]], vals[ok], dtype=np.float32)
    flat = go.reshape(N, C_out, H_out * W_out)
    for n in range(N):
        for hw in range(H_out * W_out):
            gb = np.add(gb, flat[n, :, hw], dtype=np.float32)
    z = np.float32(0.0)
    return gi + z, gw.reshape(w.shape) + z, gb + z


# SoftmaxBackward's row dot as the reference's Release build rounds it: blocks
# of SOFTMAX_BWD_VEC products rounded then added, the D mod SOFTMAX_BWD_VEC tail
# fused (8: the x86-64-v4 / AVX-512 build, the ISA of the GPU hosts).
SOFTMAX_BWD_VEC = 8


def softmax_backward(grad: np.ndarray, y: np.ndarray, vec: int = SOFTMAX_BWD_VEC) -> np.ndarray:
    """SoftmaxBackward (src/autograd.cpp:228-256) given the forward output y."""
    g = np.ascontiguousarray(grad, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    out = np.empty_like(y)
    D = y.shape[-1] if y.ndim else 1
    if y.size:
        lib().orc_softmax_backward(_fp(g), _fp(y), _fp(out), y.size // D, D, vec)
    return out


# The dots over the head dimension in flash_attention / FlashAttentionBackward
# round like SoftmaxBackward's (same loop shape, same vectorisation).
FLASH_VEC = SOFTMAX_BWD_VEC


def _heads(x):
    x = np.ascontiguousarray(x, np.float32)
    S, d = x.shape[-2], x.shape[-1]
    return x.reshape(-1, S, d), S, d


def flash_attention(q, k, v, scale, vec: int = FLASH_VEC):
    """flash_attention (src/ops.cpp:1040-1137) per head of [..., S, d]:
    returns (O, L) with L = m + log(l), the reference's L_cache."""
    shape = np.shape(q)
    (qh, S, d), (kh, _, _), (vh, _, _) = _heads(q), _heads(k), _heads(v)
    o = np.empty_like(qh)
    lse = np.empty(qh.shape[:2], np.float32)
    for h in range(qh.shape[0]):
        lib().orc_flash_attention(_fp(qh[h]), _fp(kh[h]), _fp(vh[h]), S, d, float(scale),
                                  _fp(o[h]), _fp(lse[h]), vec)
    return o.reshape(shape), lse.reshape(shape[:-1])


def flash_attention_backward(dout, q, k, v, o, lse, scale, vec: int = FLASH_VEC):
    """FlashAttentionBackward (src/autograd.cpp:575-669) per head: (dQ, dK, dV)."""
    shape = np.shape(q)
    (gh, S, d) = _heads(dout)
    qh, kh, vh, oh = (_heads(t)[0] for t in (q, k, v, o))
    lh = np.ascontiguousarray(lse, np.float32).reshape(-1, S)
    dq, dk, dv = (np.empty_like(qh) for _ in range(3))
    for h in range(qh.shape[0]):
        lib().orc_flash_attention_backward(_fp(gh[h]), _fp(qh[h]), _fp(kh[h]), _fp(vh[h]),
                                           _fp(oh[h]), _fp(lh[h]), S, d, float(scale),
                                           _fp(dq[h]), _fp(dk[h]), _fp(dv[h]), vec)
    return dq.reshape(shape), dk.reshape(shape), dv.reshape(shape)


def matmul_backward(grad: np.ndarray, a: np.ndarray, b: np.ndarray, nthreads: int | None = None):
    """MatmulBackward::backward, src/autograd.cpp:341-384, followed by
    accumulate_grad into empty grads (src/autograd.cpp:16-22: zeros + d).

    a, b are the inputs as given to matmul (any strided views); returns
    (dA, dB) with the shapes of a and b."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    sq_a, sq_b = a.ndim == 1, b.ndim == 1
    g = np.asarray(grad, np.float32)
    if sq_a:
        # (..., N) -> (..., 1, N); a 0-D grad (vector . vector) becomes [1]
        g = g.reshape(g.shape[:-1] + (1, g.shape[-1])) if g.ndim else g.reshape(1)
    if sq_b:
        g = g.reshape(g.shape + (1,))
    A = a.reshape(1, a.shape[0]) if sq_a else a
    B = b.reshape(b.shape[0], 1) if sq_b else b
    At = np.swapaxes(A, -2, -1)
    Bt = np.swapaxes(B, -2, -1)
    da = sum_to(matmul(g, Bt, nthreads), list(A.shape))
    db = sum_to(matmul(At, g, nthreads), list(B.shape))
    if sq_a:
        da = da.reshape(a.shape)
    if sq_b:
        db = db.reshape(b.shape)
    da = add(np.zeros(a.shape, np.float32), da)
    db = add(np.zeros(b.shape, np.float32), db)
    return da, db


# ---------------------------------------------------------------------------
# The reference library itself (oracle/_ref), for pinning the restatement.
# ---------------------------------------------------------------------------

def _cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


class TLRef:
    """ctypes view of oracle/_ref/libtlref_{v3,v4}.so (reference sources + ref_shim.cpp)."""

    def __init__(self, path: str | None = None):
        if path is None:
            flags = _cpu_flags()
            v4 = {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags
            path = os.path.join(HERE, "_ref", "libtlref_v4.so" if v4 else "libtlref_v3.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        L = ctypes.CDLL(path)
        i64p = ctypes.POINTER(_i64)
        L.tlref_hardware_threads.restype = ctypes.c_int
        L.tlref_matmul.argtypes = [_f32p, ctypes.c_int, i64p, ctypes.c_int, _f32p, ctypes.c_int,
                                   i64p, ctypes.c_int, _f32p, _i64, ctypes.POINTER(ctypes.c_int),
                                   i64p, ctypes.c_char_p, ctypes.c_int]
        L.tlref_matmul.restype = ctypes.c_int
        L.tlref_matmul_timed.argtypes = [_f32p, ctypes.c_int, i64p, _f32p, ctypes.c_int, i64p,
                                         ctypes.c_int, ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_double), ctypes.c_char_p,
                                         ctypes.c_int]
        L.tlref_matmul_timed.restype = ctypes.c_int
        L.tlref_matmul_backward.argtypes = [_f32p, ctypes.c_int, i64p, ctypes.c_int, _f32p,
                                            ctypes.c_int, i64p, ctypes.c_int, _f32p, ctypes.c_int,
                                            i64p, _f32p, _i64, _f32p, _i64, ctypes.c_char_p,
                                            ctypes.c_int]
        L.tlref_matmul_backward.restype = ctypes.c_int
        L.tlref_add.argtypes = [_f32p, ctypes.c_int, i64p, _f32p, ctypes.c_int, i64p, _f32p,
                                _i64, ctypes.POINTER(ctypes.c_int), i64p, ctypes.c_char_p,
                                ctypes.c_int]
        L.tlref_add.restype = ctypes.c_int
        L.tlref_scale.argtypes = [_f32p, ctypes.c_int, i64p, ctypes.c_float, _f32p, _i64,
                                  ctypes.c_char_p, ctypes.c_int]
        L.tlref_scale.restype = ctypes.c_int
        L.tlref_softmax.argtypes = [_f32p, ctypes.c_int, i64p, _f32p, _f32p, _f32p, _i64,
                                    ctypes.c_char_p, ctypes.c_int]
        L.tlref_softmax.restype = ctypes.c_int
        L.tlref_save_model.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                       i64p, _f32p, ctypes.c_char_p, ctypes.c_int]
        L.tlref_save_model.restype = ctypes.c_int
        L.tlref_load_model.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                       i64p, _f32p, ctypes.c_char_p, ctypes.c_int]
        L.tlref_load_model.restype = ctypes.c_int
        L.tlref_conv2d.argtypes = [_f32p, i64p, _f32p, i64p, _f32p, _i64, _i64, _i64, _f32p, _f32p,
                                   _f32p, _f32p, _f32p, ctypes.c_char_p, ctypes.c_int]
        L.tlref_conv2d.restype = ctypes.c_int
        L.tlref_flash_attention.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p,
                                            _f32p, _f32p, _f32p, _f32p, ctypes.c_char_p,
                                            ctypes.c_int]
        L.tlref_flash_attention.restype = ctypes.c_int
        self.L = L

    def hardware_threads(self) -> int:
        return int(self.L.tlref_hardware_threads())

    @staticmethod
    def _shape(x):
        return (_i64 * max(1, x.ndim))(*x.shape)

    def matmul(self, a, b, trans_a=False, trans_b=False, out_cap=None):
        """tl::matmul(A', B'); A', B' = transpose(-2,-1) views when trans_* is set."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        if out_cap is None:
            out_cap = max(1, _guess_numel(a, b, trans_a, trans_b))
        out = np.empty(out_cap, np.float32)
        nd = ctypes.c_int(0)
        sz = (_i64 * 16)()
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_matmul(_fp(a), a.ndim, self._shape(a), int(trans_a), _fp(b), b.ndim,
                                 self._shape(b), int(trans_b), _fp(out), out_cap,
                                 ctypes.byref(nd), sz, err, 256)
        if rc == 1:
            raise ValueError(err.value.decode())
        if rc != 0:
            raise RuntimeError(f"tlref_matmul rc={rc}")
        shape = tuple(sz[i] for i in range(nd.value))
        n = int(np.prod(shape, dtype=np.int64)) if shape else 1
        return out[:n].reshape(shape)

    def matmul_timed(self, a, b, warmup, steps):
        """Mean seconds per tl::matmul(A, B) call over `steps` calls after
        `warmup` (tensors built once; the timed region holds only the calls)."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        sec = ctypes.c_double(0.0)
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_matmul_timed(_fp(a), a.ndim, self._shape(a), _fp(b), b.ndim,
                                       self._shape(b), int(warmup), int(steps),
                                       ctypes.byref(sec), err, 256)
        if rc != 0:
            raise RuntimeError(f"tlref_matmul_timed: {err.value.decode()}")
        return sec.value

    def matmul_backward(self, a, b, grad, trans_a=False, trans_b=False):
        """Gradients of the stored leaves a, b for C = matmul(a', b'), dC = grad."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        g = np.ascontiguousarray(grad, np.float32)
        da = np.empty(a.shape, np.float32)
        db = np.empty(b.shape, np.float32)
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_matmul_backward(_fp(a), a.ndim, self._shape(a), int(trans_a), _fp(b),
                                          b.ndim, self._shape(b), int(trans_b), _fp(g), g.ndim,
                                          self._shape(g), _fp(da), max(1, da.size), _fp(db),
                                          max(1, db.size), err, 256)
        if rc == 1:
            raise ValueError(err.value.decode())
        if rc != 0:
            raise RuntimeError(f"tlref_matmul_backward rc={rc}")
        return da, db

    def add(self, a, b):
        """tl::add(a, b) with broadcasting."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        cap = max(1, a.size * max(1, b.size))
        out = np.empty(cap, np.float32)
        nd = ctypes.c_int(0)
        sz = (_i64 * 16)()
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_add(_fp(a), a.ndim, self._shape(a), _fp(b), b.ndim, self._shape(b),
                              _fp(out), cap, ctypes.byref(nd), sz, err, 256)
        if rc == 1:
            raise ValueError(err.value.decode())
        if rc != 0:
            raise RuntimeError(f"tlref_add rc={rc}")
        shape = tuple(sz[i] for i in range(nd.value))
        n = int(np.prod(shape, dtype=np.int64)) if shape else 1
        return out[:n].reshape(shape)

    def scale(self, x, s):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.shape, np.float32)
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_scale(_fp(x), x.ndim, self._shape(x), float(s), _fp(out),
                                max(1, out.size), err, 256)
        if rc != 0:
            raise RuntimeError(f"tlref_scale rc={rc}: {err.value.decode()}")
        return out

    @staticmethod
    def _pack(shapes):
        nd = (ctypes.c_int * max(1, len(shapes)))(*[len(s) for s in shapes])
        flat = [d for s in shapes for d in s]
        return nd, (_i64 * max(1, len(flat)))(*flat)

    def save_model(self, path, tensors):
        """tl::save_model of the given arrays (in order)."""
        ts = [np.array(t, dtype=np.float32, order="C", copy=True) for t in tensors]  # keeps 0-D
        nd, sh = self._pack([t.shape for t in ts])
        data = np.concatenate([t.reshape(-1) for t in ts]) if ts else np.zeros(1, np.float32)
        data = np.ascontiguousarray(data if data.size else np.zeros(1, np.float32))
        err = ctypes.create_string_buffer(512)
        if self.L.tlref_save_model(str(path).encode(), len(ts), nd, sh, _fp(data), err, 512):
            raise RuntimeError(err.value.decode())

    def load_model(self, path, shapes):
        """tl::load_model into fresh tensors of these shapes; returns the arrays."""
        nd, sh = self._pack(shapes)
        sizes = [int(np.prod(s, dtype=np.int64)) for s in shapes]
        data = np.zeros(max(1, sum(sizes)), np.float32)
        err = ctypes.create_string_buffer(512)
        if self.L.tlref_load_model(str(path).encode(), len(shapes), nd, sh, _fp(data), err, 512):
            raise RuntimeError(err.value.decode())
        out, off = [], 0
        for s, n in zip(shapes, sizes):
            out.append(data[off:off + n].reshape(s))
            off += n
        return out

    def conv2d(self, x, w, b, stride=1, padding=0, groups=1, grad=None):
        """tl::conv2d; with grad also (x.grad, w.grad, b.grad) after backward."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        bb = None if b is None else np.ascontiguousarray(b, np.float32)
        N, C_in, H, W = x.shape
        C_out, _, kH, kW = w.shape
        H_out, W_out = _conv_out(H, W, kH, kW, stride, padding)
        out = np.empty((N, C_out, max(H_out, 0), max(W_out, 0)), np.float32)
        g = None if grad is None else np.ascontiguousarray(grad, np.float32)
        dx = np.empty_like(x)
        dw = np.empty_like(w)
        db = np.empty((C_out,), np.float32)
        err = ctypes.create_string_buffer(512)
        rc = self.L.tlref_conv2d(_fp(x), (_i64 * 4)(*x.shape), _fp(w), (_i64 * 4)(*w.shape),
                                 None if bb is None else _fp(bb), stride, padding, groups,
                                 None if g is None else _fp(g), _fp(out), _fp(dx), _fp(dw), _fp(db),
                                 err, 512)
        if rc:
            raise ValueError(err.value.decode())
        return out if g is None else (out, dx, dw, db)

    def flash_attention(self, q, k, v, scale, grad=None):
        """O = tl::flash_attention(Q, K, V, scale) on [S, d]; with grad also
        (Q.grad, K.grad, V.grad) after O.backward()."""
        q, k, v = (np.ascontiguousarray(t, np.float32) for t in (q, k, v))
        S, d = q.shape
        out = np.empty_like(q)
        dq, dk, dv = (np.empty_like(q) for _ in range(3))
        g = None if grad is None else np.ascontiguousarray(grad, np.float32)
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_flash_attention(_fp(q), _fp(k), _fp(v), S, d, float(scale),
                                          None if g is None else _fp(g), _fp(out), _fp(dq),
                                          _fp(dk), _fp(dv), err, 256)
        if rc:
            raise RuntimeError(f"tlref_flash_attention rc={rc}: {err.value.decode()}")
        return out if g is None else (out, dq, dk, dv)

    def softmax(self, x, grad=None):
        """y = tl::softmax(x); with grad, also x.grad after y.backward() (SoftmaxBackward
        followed by accumulate_grad, i.e. 0 + dx)."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(x.shape, np.float32)
        dx = np.empty(x.shape, np.float32)
        g = None if grad is None else np.ascontiguousarray(grad, np.float32)
        err = ctypes.create_string_buffer(256)
        rc = self.L.tlref_softmax(_fp(x), x.ndim, self._shape(x), None if g is None else _fp(g),
                                  _fp(y), _fp(dx), max(1, x.size), err, 256)
        if rc != 0:
            raise RuntimeError(f"tlref_softmax rc={rc}: {err.value.decode()}")
        return y if g is None else (y, dx)


def _guess_numel(a, b, ta, tb):
    sa = list(a.shape)
    sb = list(b.shape)
    if ta and len(sa) >= 2:
        sa[-1], sa[-2] = sa[-2], sa[-1]
    if tb and len(sb) >= 2:
        sb[-1], sb[-2] = sb[-2], sb[-1]
    M = sa[-2] if len(sa) >= 2 else 1
    N = sb[-1] if len(sb) >= 2 else 1
    try:
        bo = broadcast_shape(sa[:-2], sb[:-2])
    except ValueError:
        bo = []
    return int(np.prod(bo, dtype=np.int64)) * M * N


def tlref(path: str | None = None) -> TLRef:
    return TLRef(path)
