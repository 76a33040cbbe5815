"""Python binding of libtl_cuda (include/tlc.h) over ctypes.

Device memory and streams come from PyTorch (plumbing only); every kernel
that runs is one of libtl_cuda's.  If the library is missing, importing the
binding works but every call raises: there is no fallback path.

    import tlcuda
    c = tlcuda.matmul(a, b, mode="tf32")          # a, b: CUDA float32 tensors, any strides
    da, db = tlcuda.matmul_backward(dc, a, b)      # MatmulBackward
    c = tlcuda.matmul_host(a_np, b_np)             # host buffers in, host buffer out
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libtl_cuda.so")
MAX_DIMS = 8

MODES = {"exact": 0, "fp32": 0, "tf32": 1, "3xtf32": 2, "default": -1}
STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "CUDA error",
          4: "out of memory", 5: "kernel wait timed out", 6: "I/O error"}


class TLCError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status
        self.msg = msg


class TLCInvalidArgument(TLCError, ValueError):
    """TLC_ERR_INVALID_ARGUMENT: the reference throws std::invalid_argument."""


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("ndim", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * MAX_DIMS), ("strides", ctypes.c_int64 * MAX_DIMS)]


class GemmDesc(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("A", ctypes.c_void_p), ("a_rs", ctypes.c_int64), ("a_cs", ctypes.c_int64),
                ("B", ctypes.c_void_p), ("b_rs", ctypes.c_int64), ("b_cs", ctypes.c_int64),
                ("C", ctypes.c_void_p), ("c_rs", ctypes.c_int64),
                ("batch_ndim", ctypes.c_int32), ("batch_sizes", ctypes.c_int64 * 3),
                ("a_bstride", ctypes.c_int64 * 3), ("b_bstride", ctypes.c_int64 * 3),
                ("c_bstride", ctypes.c_int64 * 3)]


# Every symbol include/tlc.h declares, with its ctypes signature.
_P = ctypes.POINTER
_T = _P(Tensor)
_v, _i, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "tlc_version": ([], _i),
    "tlc_status_string": ([_i], ctypes.c_char_p),
    "tlc_last_error": ([], ctypes.c_char_p),
    "tlc_launch_count": ([], ctypes.c_uint64),
    "tlc_mode_from_string": ([ctypes.c_char_p], _i),
    "tlc_default_mode": ([], _i),
    "tlc_device_count": ([_P(_i)], _i),
    "tlc_set_device": ([_i], _i),
    "tlc_get_device": ([_P(_i)], _i),
    "tlc_malloc": ([_P(_v), _sz], _i),
    "tlc_free": ([_v], _i),
    "tlc_malloc_host": ([_P(_v), _sz], _i),
    "tlc_free_host": ([_v], _i),
    "tlc_memcpy": ([_v, _v, _sz, _i, _v], _i),
    "tlc_memset_zero": ([_v, _sz, _v], _i),
    "tlc_stream_synchronize": ([_v], _i),
    "tlc_check_device_errors": ([], _i),
    "tlc_selftest_bounded_wait": ([ctypes.c_uint64], _i),
    "tlc_matmul_shape": ([_T, _T, _P(ctypes.c_int32), _P(_i64)], _i),
    "tlc_matmul": ([_T, _T, _T, _i, _v], _i),
    "tlc_matmul_backward": ([_T, _T, _T, _T, _T, _i, _i, _v], _i),
    "tlc_matmul_host": ([_T, _T, _T, _i, _v], _i),
    "tlc_matmul_backward_host": ([_T, _T, _T, _T, _T, _i, _i, _v], _i),
    "tlc_gemm": ([_P(GemmDesc), _i, _v], _i),
    "tlc_gemm_3xtf32_noalloc": ([_P(GemmDesc), _v], _i),
    "tlc_sum_dim": ([_v, _v, _i64, _i64, _i64, _v], _i),
    "tlc_sum_dim_from": ([_v, _v, _v, _i64, _i64, _i64, _v], _i),
    "tlc_add": ([_v, _v, _v, _i64, _v], _i),
    "tlc_contiguous": ([_T, _v, _v], _i),
    "tlc_matmul_fused": ([_T, _T, ctypes.c_float, _T, _T, _i, _v], _i),
    "tlc_add_tensors": ([_T, _T, _T, _v], _i),
    "tlc_scale": ([_T, ctypes.c_float, _T, _v], _i),
    "tlc_softmax": ([_T, _T, _v], _i),
    "tlc_softmax_backward": ([_T, _T, _T, _v], _i),
    "tlc_sum_to": ([_T, _T, _v], _i),
    "tlc_conv2d_shape": ([_T, _T, _i64, _i64, _i64, _P(_i64)], _i),
    "tlc_conv2d": ([_T, _T, _T, _i64, _i64, _i64, _T, _i, _v], _i),
    "tlc_conv2d_backward": ([_T, _T, _T, _i64, _i64, _i64, _T, _T, _T, _i, _v], _i),
    "tlc_flash_attention": ([_T, _T, _T, ctypes.c_float, _T, _T, _i, _v], _i),
    "tlc_flash_attention_backward": ([_T, _T, _T, _T, _T, _T, ctypes.c_float, _T, _T, _T, _i, _v],
                                     _i),
    "tlc_load_tlmd": ([ctypes.c_char_p, ctypes.c_int32, _T, _v], _i),
    "tlc_save_tlmd": ([ctypes.c_char_p, ctypes.c_int32, _T, _v], _i),
    "tlc_shard_range": ([_i64, _i, _i, _P(_i64), _P(_i64)], _i),
    "tlc_shard_cols": ([_i64, _i, _i, _i64, _P(_i64), _P(_i64)], _i),
    "tlc_gather_colblocks": ([_v, _v, _i64, _i64, _i, _P(_i64), _v], _i),
    "tlc_group_create": ([_P(ctypes.c_int), _i, _P(_v)], _i),
    "tlc_group_destroy": ([_v], _i),
    "tlc_group_size": ([_v, _P(_i), _P(_i)], _i),
    "tlc_group_matmul_host": ([_v, _T, _T, _T, _i], _i),
    "tlc_group_matmul_backward_host": ([_v, _T, _T, _T, _T, _T, _i, _i], _i),
    "tlc_group_matmul": ([_v, _T, _T, _T, _i, _v], _i),
}

_lib = None


def lib():
    """The loaded libtl_cuda; raises if it was not built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libtl_cuda is not built: {LIB_PATH} missing "
                               "(run python torchlite-cpp_b200/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _check(status: int):
    if status != 0:
        msg = lib().tlc_last_error().decode()
        if status == 1:
            raise TLCInvalidArgument(status, msg)
        raise TLCError(status, msg)


def mode_id(mode) -> int:
    if isinstance(mode, int):
        return mode
    m = MODES.get(str(mode).lower())
    if m is None:
        raise ValueError(f"unknown mode {mode!r}; use exact, tf32 or 3xtf32")
    return m


def launch_count() -> int:
    return int(lib().tlc_launch_count())


def check_device_errors():
    """Synchronise the current device; raise if a kernel recorded a timeout."""
    _check(lib().tlc_check_device_errors())


def selftest_bounded_wait(timeout_ns: int) -> int:
    """Status of the bounded-wait self test (TLC_ERR_TIMEOUT == 5 when it works)."""
    return int(lib().tlc_selftest_bounded_wait(int(timeout_ns)))


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def view_of(t) -> Tensor:
    """tlc_tensor for a torch tensor (device or host) or a numpy array."""
    v = Tensor()
    if isinstance(t, np.ndarray):
        assert t.dtype == np.float32
        v.data = t.ctypes.data
        v.ndim = t.ndim
        for i in range(t.ndim):
            v.sizes[i] = t.shape[i]
            v.strides[i] = t.strides[i] // 4
    else:
        import torch
        assert t.dtype == torch.float32, "libtl_cuda computes in float32"
        v.data = t.data_ptr()
        v.ndim = t.dim()
        for i in range(t.dim()):
            v.sizes[i] = t.size(i)
            v.strides[i] = t.stride(i)
    if v.ndim > MAX_DIMS:
        raise ValueError(f"at most {MAX_DIMS} dims")
    return v


def matmul_shape(a, b):
    nd = ctypes.c_int32(0)
    sz = (ctypes.c_int64 * MAX_DIMS)()
    va, vb = view_of(a), view_of(b)
    _check(lib().tlc_matmul_shape(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(nd), sz))
    return tuple(sz[i] for i in range(nd.value))


def matmul(a, b, mode="exact", out=None, stream=None):
    """tl::matmul on CUDA float32 tensors (any strides)."""
    import torch
    shape = matmul_shape(a, b)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=a.device)
    va, vb, vo = view_of(a), view_of(b), view_of(out)
    _check(lib().tlc_matmul(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vo), mode_id(mode),
                            _stream_ptr(stream)))
    return out


def matmul_backward(grad, a, b, mode="exact", da=None, db=None, accumulate=False, stream=None,
                    need_a=True, need_b=True):
    """MatmulBackward on CUDA tensors: returns (dA, dB) with the shapes of a and b."""
    import torch
    if need_a and da is None:
        da = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    if need_b and db is None:
        db = torch.empty(b.shape, dtype=torch.float32, device=b.device)
    vg, va, vb = view_of(grad), view_of(a), view_of(b)
    vda = view_of(da) if need_a else Tensor()
    vdb = view_of(db) if need_b else Tensor()
    _check(lib().tlc_matmul_backward(ctypes.byref(vg), ctypes.byref(va), ctypes.byref(vb),
                                     ctypes.byref(vda), ctypes.byref(vdb), int(accumulate),
                                     mode_id(mode), _stream_ptr(stream)))
    return da, db


def matmul_host(a, b, mode="exact", out=None, stream=None):
    """tl::matmul on host buffers (numpy arrays or CPU torch tensors, pinned or
    not); copies in and out inside the call.  `stream`: a torch CUDA stream to
    run on (None = the library's own)."""
    shape = matmul_shape(a, b)
    if out is None:
        out = np.empty(shape, np.float32)
    va, vb, vo = view_of(a), view_of(b), view_of(out)
    sp = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
    _check(lib().tlc_matmul_host(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vo),
                                 mode_id(mode), sp))
    return out


def matmul_backward_host(grad: np.ndarray, a: np.ndarray, b: np.ndarray, mode="exact"):
    da = np.empty(a.shape, np.float32)
    db = np.empty(b.shape, np.float32)
    vg, va, vb, vda, vdb = map(view_of, (grad, a, b, da, db))
    _check(lib().tlc_matmul_backward_host(ctypes.byref(vg), ctypes.byref(va), ctypes.byref(vb),
                                          ctypes.byref(vda), ctypes.byref(vdb), 0, mode_id(mode),
                                          None))
    return da, db


def gemm(A, B, C, M, N, K, a_rs, a_cs, b_rs, b_cs, c_rs, batch=(), a_bs=(), b_bs=(), c_bs=(),
         mode="exact", stream=None):
    """tlc_gemm on raw device addresses (element strides)."""
    d = GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.A, d.a_rs, d.a_cs = A, a_rs, a_cs
    d.B, d.b_rs, d.b_cs = B, b_rs, b_cs
    d.C, d.c_rs = C, c_rs
    d.batch_ndim = len(batch)
    for i, s in enumerate(batch):
        d.batch_sizes[i] = s
        d.a_bstride[i] = a_bs[i]
        d.b_bstride[i] = b_bs[i]
        d.c_bstride[i] = c_bs[i]
    _check(lib().tlc_gemm(ctypes.byref(d), mode_id(mode), _stream_ptr(stream)))


def sum_dim0(stack, out=None, stream=None, init=None):
    """sum over dim 0 of a contiguous CUDA tensor, ascending from 0.0f
    (tlc_sum_dim with outer = 1): the reference's sum(x, 0) order.  With
    `init` (the shape of one entry) the sum continues from it:
    init + stack[0] + stack[1] + ... (tlc_sum_dim_from)."""
    import torch
    assert stack.is_contiguous()
    if out is None:
        out = torch.empty(stack.shape[1:], dtype=torch.float32, device=stack.device)
    inner = out.numel()
    if init is not None:
        assert init.is_contiguous() and init.numel() == inner
    _check(lib().tlc_sum_dim_from(ctypes.c_void_p(stack.data_ptr()),
                                  ctypes.c_void_p(init.data_ptr() if init is not None else None),
                                  ctypes.c_void_p(out.data_ptr()), 1, stack.shape[0], inner,
                                  _stream_ptr(stream)))
    return out


def matmul_fused(a, b, scale=1.0, bias=None, mode="exact", out=None, stream=None):
    """scale * (a . b) + bias (bias: 1-D of length N, or None), fused into the GEMM."""
    import torch
    shape = matmul_shape(a, b)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=a.device)
    va, vb, vo = view_of(a), view_of(b), view_of(out)
    vbias = view_of(bias) if bias is not None else None
    _check(lib().tlc_matmul_fused(ctypes.byref(va), ctypes.byref(vb), float(scale),
                                  ctypes.byref(vbias) if vbias is not None else None,
                                  ctypes.byref(vo), mode_id(mode), _stream_ptr(stream)))
    return out


def _broadcast(sa, sb):
    nd = max(len(sa), len(sb))
    out = []
    for i in range(nd):
        x = sa[i - (nd - len(sa))] if i >= nd - len(sa) else 1
        y = sb[i - (nd - len(sb))] if i >= nd - len(sb) else 1
        out.append(y if x == 1 else x)  # size 0 against 1 gives 0
    return tuple(out)


def add_tensors(a, b, out=None, stream=None):
    """tl::add with broadcasting on CUDA tensors."""
    import torch
    if out is None:
        out = torch.empty(_broadcast(tuple(a.shape), tuple(b.shape)), dtype=torch.float32,
                          device=a.device)
    va, vb, vo = view_of(a), view_of(b), view_of(out)
    _check(lib().tlc_add_tensors(ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vo),
                                 _stream_ptr(stream)))
    return out


def scale(x, s, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty(tuple(x.shape), dtype=torch.float32, device=x.device)
    vx, vo = view_of(x), view_of(out)
    _check(lib().tlc_scale(ctypes.byref(vx), float(s), ctypes.byref(vo), _stream_ptr(stream)))
    return out


def softmax(x, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty(tuple(x.shape), dtype=torch.float32, device=x.device)
    vx, vo = view_of(x), view_of(out)
    _check(lib().tlc_softmax(ctypes.byref(vx), ctypes.byref(vo), _stream_ptr(stream)))
    return out


def softmax_backward(grad, y, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty(tuple(y.shape), dtype=torch.float32, device=y.device)
    vg, vy, vo = view_of(grad), view_of(y), view_of(out)
    _check(lib().tlc_softmax_backward(ctypes.byref(vg), ctypes.byref(vy), ctypes.byref(vo),
                                      _stream_ptr(stream)))
    return out


def sum_to(x, target, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty(tuple(target), dtype=torch.float32, device=x.device)
    vx, vo = view_of(x), view_of(out)
    _check(lib().tlc_sum_to(ctypes.byref(vx), ctypes.byref(vo), _stream_ptr(stream)))
    return out


def conv2d(x, w, bias=None, stride=1, padding=0, groups=1, mode="exact", out=None, stream=None):
    """tl::conv2d on CUDA NCHW tensors."""
    import torch
    vx, vw = view_of(x), view_of(w)
    sz = (ctypes.c_int64 * 4)()
    _check(lib().tlc_conv2d_shape(ctypes.byref(vx), ctypes.byref(vw), stride, padding, groups, sz))
    if out is None:
        out = torch.empty(tuple(sz), dtype=torch.float32, device=x.device)
    vb = view_of(bias) if bias is not None else None
    vo = view_of(out)
    _check(lib().tlc_conv2d(ctypes.byref(vx), ctypes.byref(vw), ctypes.byref(vb) if vb else None,
                            stride, padding, groups, ctypes.byref(vo), mode_id(mode),
                            _stream_ptr(stream)))
    return out


def conv2d_backward(grad, x, w, stride=1, padding=0, groups=1, mode="exact", need=(True, True, True),
                    stream=None):
    """Conv2dBackward: (d_input, d_weight, d_bias), None where not requested."""
    import torch
    outs = [torch.empty(tuple(x.shape), device=x.device) if need[0] else None,
            torch.empty(tuple(w.shape), device=x.device) if need[1] else None,
            torch.empty((w.shape[0],), device=x.device) if need[2] else None]
    views = [view_of(o) if o is not None else None for o in outs]
    vg, vx, vw = view_of(grad), view_of(x), view_of(w)
    _check(lib().tlc_conv2d_backward(ctypes.byref(vg), ctypes.byref(vx), ctypes.byref(vw), stride,
                                     padding, groups,
                                     *[ctypes.byref(v) if v else None for v in views],
                                     mode_id(mode), _stream_ptr(stream)))
    return tuple(outs)


def flash_attention(q, k, v, sm_scale, out=None, lse=None, mode="exact", stream=None):
    """tl::flash_attention on CUDA [..., S, d] tensors (every leading index a
    head): returns (out, lse), lse = m + log(l) per row, what the backward needs.
    mode "tf32" runs the tensor-core kernel where it applies (32 <= d <= 64)."""
    import torch
    if out is None:
        out = torch.empty(tuple(q.shape), dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty(tuple(q.shape[:-1]), dtype=torch.float32, device=q.device)
    vq, vk, vv, vo, vl = (view_of(t) for t in (q, k, v, out, lse))
    _check(lib().tlc_flash_attention(ctypes.byref(vq), ctypes.byref(vk), ctypes.byref(vv),
                                     float(sm_scale), ctypes.byref(vo), ctypes.byref(vl),
                                     mode_id(mode), _stream_ptr(stream)))
    return out, lse


def flash_attention_backward(grad, q, k, v, out, lse, sm_scale, mode="exact", dq=None, dk=None,
                             dv=None, stream=None):
    """FlashAttentionBackward: (dq, dk, dv)."""
    import torch
    dq, dk, dv = (t if t is not None else torch.empty(tuple(q.shape), device=q.device)
                  for t in (dq, dk, dv))
    vs = [view_of(t) for t in (grad, q, k, v, out, lse)]
    vd = [view_of(t) for t in (dq, dk, dv)]
    _check(lib().tlc_flash_attention_backward(*[ctypes.byref(x) for x in vs], float(sm_scale),
                                              *[ctypes.byref(x) for x in vd], mode_id(mode),
                                              _stream_ptr(stream)))
    return dq, dk, dv


def _views(tensors):
    arr = (Tensor * max(1, len(tensors)))()
    for i, t in enumerate(tensors):
        arr[i] = view_of(t)
    return arr


def _io_stream(stream):
    # torch's current stream when a GPU is there; otherwise the legacy stream
    # (the file checks that fail before any copy need no device)
    import torch
    return _stream_ptr(stream) if torch.cuda.is_available() else None


def load_tlmd(path, tensors, stream=None):
    """load_model into CUDA tensors (contiguous, shapes as stored)."""
    _check(lib().tlc_load_tlmd(str(path).encode(), len(tensors), _views(tensors),
                               _io_stream(stream)))
    return tensors


def save_tlmd(path, tensors, stream=None):
    """save_model from CUDA tensors."""
    _check(lib().tlc_save_tlmd(str(path).encode(), len(tensors), _views(tensors),
                               _io_stream(stream)))


def shard_range(count, world, rank):
    b, e = ctypes.c_int64(), ctypes.c_int64()
    _check(lib().tlc_shard_range(count, world, rank, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


def shard_cols(N, world, rank, align=1):
    b, e = ctypes.c_int64(), ctypes.c_int64()
    _check(lib().tlc_shard_cols(N, world, rank, align, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


def gather_colblocks(gathered, out, M, N, col_begin, stream=None):
    world = len(col_begin) - 1
    cb = (ctypes.c_int64 * len(col_begin))(*col_begin)
    _check(lib().tlc_gather_colblocks(ctypes.c_void_p(gathered.data_ptr()),
                                      ctypes.c_void_p(out.data_ptr()), M, N, world, cb,
                                      _stream_ptr(stream)))
    return out


class Group:
    """A device group (tlc_group_*): one tl::matmul over several GPUs of the
    box from this process.  `devices` may repeat a device."""

    def __init__(self, devices):
        self.devices = list(devices)
        arr = (ctypes.c_int * len(self.devices))(*self.devices)
        self._g = ctypes.c_void_p()
        _check(lib().tlc_group_create(arr, len(self.devices), ctypes.byref(self._g)))

    def size(self):
        n, nc = ctypes.c_int(0), ctypes.c_int(0)
        _check(lib().tlc_group_size(self._g, ctypes.byref(n), ctypes.byref(nc)))
        return n.value, bool(nc.value)

    def matmul_host(self, a, b, mode="exact", out=None):
        shape = matmul_shape(a, b)
        if out is None:
            out = np.empty(shape, np.float32)
        va, vb, vo = view_of(a), view_of(b), view_of(out)
        _check(lib().tlc_group_matmul_host(self._g, ctypes.byref(va), ctypes.byref(vb),
                                           ctypes.byref(vo), mode_id(mode)))
        return out

    def matmul_backward_host(self, grad, a, b, mode="exact", da=None, db=None, accumulate=False,
                             need_a=True, need_b=True):
        if need_a and da is None:
            da = np.empty(a.shape, np.float32)
        if need_b and db is None:
            db = np.empty(b.shape, np.float32)
        vg, va, vb = view_of(grad), view_of(a), view_of(b)
        vda = view_of(da) if need_a else Tensor()
        vdb = view_of(db) if need_b else Tensor()
        _check(lib().tlc_group_matmul_backward_host(self._g, ctypes.byref(vg), ctypes.byref(va),
                                                    ctypes.byref(vb), ctypes.byref(vda),
                                                    ctypes.byref(vdb), int(accumulate),
                                                    mode_id(mode)))
        return da, db

    def matmul(self, a, b, mode="exact", out=None, stream=None):
        """a, b, out: CUDA tensors on the group's first device."""
        import torch
        shape = matmul_shape(a, b)
        if out is None:
            out = torch.empty(shape, dtype=torch.float32, device=a.device)
        va, vb, vo = view_of(a), view_of(b), view_of(out)
        _check(lib().tlc_group_matmul(self._g, ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vo),
                                      mode_id(mode), _stream_ptr(stream)))
        return out

    def close(self):
        if self._g:
            _check(lib().tlc_group_destroy(self._g))
            self._g = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
