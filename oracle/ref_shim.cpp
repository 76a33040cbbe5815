// C entry points over the reference library itself, compiled from the
// reference's own sources (see oracle/Makefile) into oracle/_ref/.
//
// TEST INFRASTRUCTURE ONLY: the tests use it to pin the C oracle
// (oracle/tl_oracle.c) against the real tl::matmul / MatmulBackward, and the
// CPU-baseline leg of bench.py times it.  The product never loads it.
//
// Every function builds reference tl::Tensor objects from flat host buffers,
// runs the reference code path unchanged, and copies results out.
#include <tl/autograd.h>
#include <tl/model_io.h>
#include <tl/ops.h>
#include <tl/tensor.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <thread>
#include <vector>

namespace {

tl::Tensor make(const float* p, int nd, const int64_t* sz) {
    std::vector<int64_t> s(sz, sz + nd);
    tl::Tensor t(s);
    if (t.numel() > 0) std::memcpy(t.data(), p, sizeof(float) * t.numel());
    return t;
}

// Optionally view the last two dims transposed (tl::transpose, src/ops.cpp:702).
tl::Tensor maybe_t(const tl::Tensor& t, int trans) {
    return trans ? tl::transpose(t, -2, -1) : t;
}

int fail(const std::exception& e, char* err, int errlen) {
    if (err && errlen > 0) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = 0;
    }
    return 1;
}

int copy_out(const tl::Tensor& t, float* out, int64_t cap, int* out_nd, int64_t* out_sz) {
    tl::Tensor c = t.contiguous();
    if (out_nd) *out_nd = (int)c.sizes().size();
    if (out_sz)
        for (size_t i = 0; i < c.sizes().size(); ++i) out_sz[i] = c.sizes()[i];
    if (c.numel() > cap) return 2;
    if (c.numel() > 0) std::memcpy(out, c.data(), sizeof(float) * c.numel());
    return 0;
}

}  // namespace

extern "C" {

int tlref_hardware_threads() { return (int)std::thread::hardware_concurrency(); }

// out = tl::matmul(A', B') where A' / B' are A / B with their last two dims
// transposed when trans_a / trans_b is set (the storage is given untransposed).
int tlref_matmul(const float* a, int a_nd, const int64_t* a_sz, int trans_a, const float* b,
                 int b_nd, const int64_t* b_sz, int trans_b, float* out, int64_t out_cap,
                 int* out_nd, int64_t* out_sz, char* err, int errlen) {
    try {
        tl::Tensor A = maybe_t(make(a, a_nd, a_sz), trans_a);
        tl::Tensor B = maybe_t(make(b, b_nd, b_sz), trans_b);
        tl::Tensor C = tl::matmul(A, B);
        return copy_out(C, out, out_cap, out_nd, out_sz);
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// Times tl::matmul(A, B) on tensors built once from A and B: `warmup` untimed
// calls, then `steps` calls between two steady_clock reads (each call
// allocates and zero-fills its result, as the reference's matmul does,
// src/ops.cpp:652).  *seconds = the mean per call.  The CPU arm of the
// benchmark: the reference's own batch loop and gemm_mt threads over the
// whole workload, without the shim's copies in the timed region.
int tlref_matmul_timed(const float* a, int a_nd, const int64_t* a_sz, const float* b, int b_nd,
                       const int64_t* b_sz, int warmup, int steps, double* seconds, char* err,
                       int errlen) {
    try {
        tl::Tensor A = make(a, a_nd, a_sz);
        tl::Tensor B = make(b, b_nd, b_sz);
        for (int i = 0; i < warmup; ++i) tl::matmul(A, B);
        const auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < steps; ++i) tl::matmul(A, B);
        const auto t1 = std::chrono::steady_clock::now();
        *seconds = std::chrono::duration<double>(t1 - t0).count() / (steps > 0 ? steps : 1);
        return 0;
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// C = tl::matmul(A', B'); C.grad() = dC; C.backward(); returns A.grad, B.grad
// (gradients of the stored, untransposed leaves; a transposed view's grad
// flows back through TransposeBackward exactly as in the reference).
int tlref_matmul_backward(const float* a, int a_nd, const int64_t* a_sz, int trans_a,
                          const float* b, int b_nd, const int64_t* b_sz, int trans_b,
                          const float* grad, int g_nd, const int64_t* g_sz, float* da,
                          int64_t da_cap, float* db, int64_t db_cap, char* err, int errlen) {
    try {
        tl::Tensor A = make(a, a_nd, a_sz);
        tl::Tensor B = make(b, b_nd, b_sz);
        A.set_requires_grad(true);
        B.set_requires_grad(true);
        tl::Tensor C = tl::matmul(maybe_t(A, trans_a), maybe_t(B, trans_b));
        C.grad() = make(grad, g_nd, g_sz);
        C.backward();
        int rc = copy_out(A.grad(), da, da_cap, nullptr, nullptr);
        if (rc) return rc;
        return copy_out(B.grad(), db, db_cap, nullptr, nullptr);
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// out = tl::add(A, B) (broadcasting).
int tlref_add(const float* a, int a_nd, const int64_t* a_sz, const float* b, int b_nd,
              const int64_t* b_sz, float* out, int64_t out_cap, int* out_nd, int64_t* out_sz,
              char* err, int errlen) {
    try {
        return copy_out(tl::add(make(a, a_nd, a_sz), make(b, b_nd, b_sz)), out, out_cap, out_nd,
                        out_sz);
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// out = tl::scale(X, s).
int tlref_scale(const float* x, int nd, const int64_t* sz, float s, float* out, int64_t out_cap,
                char* err, int errlen) {
    try {
        return copy_out(tl::scale(make(x, nd, sz), s), out, out_cap, nullptr, nullptr);
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// y = tl::softmax(X); if grad: y.grad() = grad; y.backward(); dx = X.grad
// (SoftmaxBackward, then accumulate_grad: 0 + d).
int tlref_softmax(const float* x, int nd, const int64_t* sz, const float* grad, float* y,
                  float* dx, int64_t cap, char* err, int errlen) {
    try {
        tl::Tensor X = make(x, nd, sz);
        if (grad) X.set_requires_grad(true);
        tl::Tensor Y = tl::softmax(X);
        int rc = copy_out(Y, y, cap, nullptr, nullptr);
        if (rc || !grad) return rc;
        Y.grad() = make(grad, nd, sz);
        Y.backward();
        return copy_out(X.grad(), dx, cap, nullptr, nullptr);
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// tl::save_model of `count` tensors (shapes flattened in `shapes`, data in
// `data`, both in order); tl::load_model of a file into tensors of the given
// shapes, data out in `data`.  Errors (std::runtime_error) as text in err.
int tlref_save_model(const char* path, int count, const int* ndims, const int64_t* shapes,
                     const float* data, char* err, int errlen) {
    try {
        std::vector<tl::Tensor> ts;
        for (int i = 0; i < count; ++i) {
            ts.push_back(make(data, ndims[i], shapes));
            data += ts.back().numel();
            shapes += ndims[i];
        }
        std::vector<tl::Tensor*> ps;
        for (auto& t : ts) ps.push_back(&t);
        tl::save_model(path, ps);
        return 0;
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

int tlref_load_model(const char* path, int count, const int* ndims, const int64_t* shapes,
                     float* data, char* err, int errlen) {
    try {
        std::vector<tl::Tensor> ts;
        for (int i = 0; i < count; ++i) {
            ts.push_back(tl::Tensor(std::vector<int64_t>(shapes, shapes + ndims[i])));
            shapes += ndims[i];
        }
        std::vector<tl::Tensor*> ps;
        for (auto& t : ts) ps.push_back(&t);
        tl::load_model(path, ps);
        for (auto& t : ts) {
            if (t.numel()) std::memcpy(data, t.data(), sizeof(float) * t.numel());
            data += t.numel();
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// out = tl::conv2d(X, W, b, stride, padding, groups); with grad: out.grad() =
// grad, out.backward(), then X.grad, W.grad, b.grad.  b may be NULL (empty).
int tlref_conv2d(const float* x, const int64_t* xs, const float* w, const int64_t* ws,
                 const float* b, int64_t stride, int64_t padding, int64_t groups,
                 const float* grad, float* out, float* dx, float* dw, float* db, char* err,
                 int errlen) {
    try {
        tl::Tensor X = make(x, 4, xs), W = make(w, 4, ws);
        const int64_t cout[1] = {ws[0]};
        tl::Tensor B = b ? make(b, 1, cout) : tl::Tensor();
        if (grad) {
            X.set_requires_grad(true);
            W.set_requires_grad(true);
            if (b) B.set_requires_grad(true);
        }
        tl::Tensor Y = tl::conv2d(X, W, B, stride, padding, groups);
        int rc = copy_out(Y, out, Y.numel() ? Y.numel() : 1, nullptr, nullptr);
        if (rc || !grad) return rc;
        Y.grad() = make(grad, 4, Y.sizes().data());
        Y.backward();
        rc = copy_out(X.grad(), dx, X.numel(), nullptr, nullptr);
        if (!rc) rc = copy_out(W.grad(), dw, W.numel(), nullptr, nullptr);
        if (!rc && b) rc = copy_out(B.grad(), db, B.numel(), nullptr, nullptr);
        return rc;
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

// O = tl::flash_attention(Q, K, V, scale) on [S, d]; with grad: O.grad() =
// grad, O.backward() (FlashAttentionBackward, then accumulate_grad), then
// Q.grad, K.grad, V.grad.
int tlref_flash_attention(const float* q, const float* k, const float* v, int64_t S, int64_t d,
                          float scale, const float* grad, float* out, float* dq, float* dk,
                          float* dv, char* err, int errlen) {
    try {
        const int64_t sz[2] = {S, d};
        tl::Tensor Q = make(q, 2, sz), K = make(k, 2, sz), V = make(v, 2, sz);
        if (grad) {
            Q.set_requires_grad(true);
            K.set_requires_grad(true);
            V.set_requires_grad(true);
        }
        tl::Tensor O = tl::flash_attention(Q, K, V, scale);
        int rc = copy_out(O, out, S * d, nullptr, nullptr);
        if (rc || !grad) return rc;
        O.grad() = make(grad, 2, sz);
        O.backward();
        rc = copy_out(Q.grad(), dq, S * d, nullptr, nullptr);
        if (!rc) rc = copy_out(K.grad(), dk, S * d, nullptr, nullptr);
        if (!rc) rc = copy_out(V.grad(), dv, S * d, nullptr, nullptr);
        return rc;
    } catch (const std::exception& e) {
        return fail(e, err, errlen);
    }
}

}  // extern "C"
