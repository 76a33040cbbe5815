// The C ABI of libtl_cuda (include/tlc.h): the tl::matmul front end
// (src/ops.cpp:605-699), MatmulBackward (src/autograd.cpp:341-384) with
// sum_to / accumulate_grad (src/autograd.cpp:16-36), the host-buffer forms,
// device memory, and the multi-GPU partition helpers.
//
// The front end turns two strided tensor views into one normalised batched
// GEMM (common.cuh: Gemm): it squeezes 1-D operands, broadcasts the batch
// dims (stride 0 for broadcast dims, as get_broadcast_index does), merges
// batch dims that are laid out as one, and reads transposed views in place.
// Only a view with no unit stride in its last two dims is copied first (the
// reference copies every non-contiguous view, src/ops.cpp:606-607).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace tlc {

std::atomic<uint64_t> g_launches{0};

namespace {
thread_local std::string t_last_error;
}

int set_error(int status, const std::string& msg) {
    t_last_error = msg;
    return status;
}
void clear_error() { t_last_error.clear(); }

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(TLC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return TLC_OK;
}

void* current_context() {
    using GetCurrent = int (*)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)
    static GetCurrent fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<GetCurrent>(f);
    }();
    void* c = nullptr;
    if (!fn || fn(&c) != 0) return nullptr;
    return c;
}

int scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
    *p = nullptr;
    if (bytes == 0) return TLC_OK;
    static DeviceOnce once;
    // Keep freed pool memory instead of returning it to the driver, so
    // repeated calls do not pay for fresh allocations.
    TLC_TRY(device_once(once, [](int dev) -> int {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            uint64_t thr = ~0ull;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
        return TLC_OK;
    }));
    TLC_CUDA_TRY(cudaMallocAsync(p, bytes, s));
    return TLC_OK;
}

void scratch_free(void* p, cudaStream_t s) {
    if (p) cudaFreeAsync(p, s);
}

namespace {

// RAII holder for stream-ordered scratch.
struct Scratch {
    void* p = nullptr;
    cudaStream_t s = nullptr;
    explicit Scratch(cudaStream_t st) : s(st) {}
    int alloc(size_t bytes) {
        scratch_free(p, s);
        p = nullptr;
        return scratch_alloc(&p, bytes, s);
    }
    float* f() const { return static_cast<float*>(p); }
    ~Scratch() { scratch_free(p, s); }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
};

// ---- views -------------------------------------------------------------------------

struct View {
    const float* data = nullptr;
    int nd = 0;
    int64_t sz[TLC_MAX_DIMS + 1] = {};
    int64_t st[TLC_MAX_DIMS + 1] = {};
    int64_t numel() const {
        int64_t n = 1;
        for (int i = 0; i < nd; ++i) n *= sz[i];
        return n;
    }
    bool contiguous() const {
        int64_t e = 1;
        for (int i = nd - 1; i >= 0; --i) {
            if (sz[i] != 1 && st[i] != e) return false;
            e *= sz[i];
        }
        return true;
    }
};

int to_view(const tlc_tensor* t, View& v, const char* name) {
    if (!t) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + " is NULL");
    if (t->ndim < 0 || t->ndim > TLC_MAX_DIMS)
        return set_error(TLC_ERR_INVALID_ARGUMENT,
                         std::string(name) + ": ndim must be 0.." + std::to_string(TLC_MAX_DIMS));
    v.data = t->data;
    v.nd = t->ndim;
    for (int i = 0; i < v.nd; ++i) {
        if (t->sizes[i] < 0)
            return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": negative size");
        if (t->strides[i] < 0)
            return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": negative stride");
        v.sz[i] = t->sizes[i];
        v.st[i] = t->strides[i];
    }
    return TLC_OK;
}

View contiguous_view(const float* data, const std::vector<int64_t>& sizes) {
    View v;
    v.data = data;
    v.nd = (int)sizes.size();
    int64_t e = 1;
    for (int i = v.nd - 1; i >= 0; --i) {
        v.sz[i] = sizes[i];
        v.st[i] = e;
        e *= sizes[i];
    }
    return v;
}

// ---- shape logic of tl::matmul ------------------------------------------------------

struct Plan {
    View a, b;  // after the 1-D squeeze (>= 2-D)
    bool sq_a = false, sq_b = false;
    int64_t M = 0, N = 0, K = 0;
    std::vector<int64_t> batch_out;   // broadcast batch shape
    std::vector<int64_t> full_out;    // batch_out + [M, N]
    std::vector<int64_t> result;      // after dropping squeezed dims
};

// compute_broadcast_shape, src/ops.cpp:55-72, with one deliberate difference:
// a size-0 dim against a size-1 dim gives 0 (NumPy's rule).  The reference
// takes std::max and gets 1, then indexes the empty operand (an out-of-bounds
// read); here that case yields an empty result instead.
int broadcast_shape(const std::vector<int64_t>& a, const std::vector<int64_t>& b,
                    std::vector<int64_t>& out) {
    const size_t nd = std::max(a.size(), b.size());
    out.assign(nd, 1);
    for (size_t i = 0; i < nd; ++i) {
        const int64_t sa = i < nd - a.size() ? 1 : a[i - (nd - a.size())];
        const int64_t sb = i < nd - b.size() ? 1 : b[i - (nd - b.size())];
        if (sa != sb && sa != 1 && sb != 1)
            return set_error(TLC_ERR_INVALID_ARGUMENT, "Incompatible dimensions for broadcasting");
        out[i] = sa == 1 ? sb : sa;
    }
    return TLC_OK;
}

// The checks and shapes of src/ops.cpp:605-652 and :676-687.
int plan_matmul(const View& a_in, const View& b_in, Plan& p) {
    p.a = a_in;
    p.b = b_in;
    if (p.a.nd == 1) {  // [K] -> [1, K]
        p.a.sz[1] = p.a.sz[0];
        p.a.st[1] = p.a.st[0];
        p.a.sz[0] = 1;
        p.a.st[0] = p.a.sz[1] * p.a.st[1];
        p.a.nd = 2;
        p.sq_a = true;
    }
    if (p.b.nd == 1) {  // [K] -> [K, 1]
        p.b.sz[1] = 1;
        p.b.st[1] = 1;
        p.b.nd = 2;
        p.sq_b = true;
    }
    if (p.a.nd < 2 || p.b.nd < 2)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "matmul: requires at least 1D tensors");
    p.M = p.a.sz[p.a.nd - 2];
    p.K = p.a.sz[p.a.nd - 1];
    const int64_t K2 = p.b.sz[p.b.nd - 2];
    p.N = p.b.sz[p.b.nd - 1];
    if (p.K != K2) return set_error(TLC_ERR_INVALID_ARGUMENT, "Incompatible dimensions for matmul");
    std::vector<int64_t> ba(p.a.sz, p.a.sz + p.a.nd - 2), bb(p.b.sz, p.b.sz + p.b.nd - 2);
    TLC_TRY(broadcast_shape(ba, bb, p.batch_out));
    if (p.batch_out.size() + 2 > TLC_MAX_DIMS)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "matmul: result has too many dims");
    p.full_out = p.batch_out;
    p.full_out.push_back(p.M);
    p.full_out.push_back(p.N);
    p.result = p.full_out;
    if (p.sq_a && p.sq_b) {
        p.result.clear();
    } else if (p.sq_a) {
        p.result.erase(p.result.end() - 2);
    } else if (p.sq_b) {
        p.result.erase(p.result.end() - 1);
    }
    return TLC_OK;
}

// ---- building the normalised GEMM -------------------------------------------------

int64_t round4(int64_t v) { return (v + 3) & ~int64_t(3); }

// Chooses (row stride, col stride) of a 2-D matrix view so that one of them
// is 1, if the view allows it; size-1 dims take whatever stride suits.
bool unit_stride_2d(int64_t rows, int64_t cols, int64_t rs, int64_t cs, int64_t& ors,
                    int64_t& ocs) {
    if (cols == 1) cs = 1;
    if (rows == 1 && cs != 1) rs = 1;
    if (cs == 1) {
        ors = rows == 1 ? round4(cols) : rs;
        ocs = 1;
        return true;
    }
    if (rs == 1) {
        ors = 1;
        ocs = cols == 1 ? round4(rows) : cs;
        return true;
    }
    return false;
}

struct BatchDim {
    int64_t size, sa, sb, sc;
};

// One GEMM call per index of the batch dims that do not fit in Gemm (rare:
// more than three unmergeable batch dims).
int run_gemm(Gemm g, const std::vector<BatchDim>& outer, int mode, cudaStream_t s) {
    if (outer.empty()) {
        if (mode == TLC_MODE_EXACT) return gemm_exact(g, s);
        return gemm_tc(g, mode, s);
    }
    const BatchDim d = outer.front();
    std::vector<BatchDim> rest(outer.begin() + 1, outer.end());
    for (int64_t i = 0; i < d.size; ++i) {
        Gemm h = g;
        h.A = g.A + i * d.sa;
        h.B = g.B + i * d.sb;
        h.C = g.C + i * d.sc;
        TLC_TRY(run_gemm(h, rest, mode, s));
    }
    return TLC_OK;
}

int resolve_mode(int mode, int& out) {
    if (mode == TLC_MODE_DEFAULT) mode = tlc_default_mode();
    if (mode != TLC_MODE_EXACT && mode != TLC_MODE_TF32 && mode != TLC_MODE_3XTF32)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "unknown GEMM mode " + std::to_string(mode));
    out = mode;
    return TLC_OK;
}

// Per-element epilogue of a fused GEMM (see Gemm): c * scale, then + bias[n].
struct Epilogue {
    const float* bias = nullptr;  // [N], contiguous, device
    float scale = 1.0f;
    int apply_scale = 0;
};

// C (contiguous, shape p.full_out) = A . B for a planned matmul, followed by
// the epilogue `ep`.
int matmul_planned(const Plan& p, float* C, int mode, cudaStream_t s, const Epilogue& ep = Epilogue()) {
    const int64_t total = [&] {
        int64_t n = 1;
        for (int64_t v : p.full_out) n *= v;
        return n;
    }();
    if (total == 0) return TLC_OK;
    if (p.K == 0) {
        TLC_TRY(launch_fill_zero(C, total, s));
        return launch_epilogue(C, total / p.N, p.N, ep.scale, ep.apply_scale != 0, ep.bias, s);
    }

    Scratch sa(s), sb(s);
    View a = p.a, b = p.b;
    int64_t a_rs, a_cs, b_rs, b_cs;
    // Views with no unit stride in the matrix dims are made contiguous first.
    if (!unit_stride_2d(p.M, p.K, a.st[a.nd - 2], a.st[a.nd - 1], a_rs, a_cs)) {
        TLC_TRY(sa.alloc(sizeof(float) * a.numel()));
        TLC_TRY(launch_strided_copy(a.data, a.nd, a.sz, a.st, sa.f(), s));
        a = contiguous_view(sa.f(), std::vector<int64_t>(a.sz, a.sz + a.nd));
        unit_stride_2d(p.M, p.K, a.st[a.nd - 2], a.st[a.nd - 1], a_rs, a_cs);
    }
    if (!unit_stride_2d(p.K, p.N, b.st[b.nd - 2], b.st[b.nd - 1], b_rs, b_cs)) {
        TLC_TRY(sb.alloc(sizeof(float) * b.numel()));
        TLC_TRY(launch_strided_copy(b.data, b.nd, b.sz, b.st, sb.f(), s));
        b = contiguous_view(sb.f(), std::vector<int64_t>(b.sz, b.sz + b.nd));
        unit_stride_2d(p.K, p.N, b.st[b.nd - 2], b.st[b.nd - 1], b_rs, b_cs);
    }

    // Batch dims, outermost first, broadcast dims carrying stride 0
    // (get_broadcast_index, src/ops.cpp:32-52).
    const int nbo = (int)p.batch_out.size();
    std::vector<BatchDim> dims;
    int64_t cstride = p.M * p.N;
    std::vector<int64_t> cst(nbo);
    for (int i = nbo - 1; i >= 0; --i) {
        cst[i] = cstride;
        cstride *= p.batch_out[i];
    }
    for (int i = 0; i < nbo; ++i) {
        const int ia = i - (nbo - (a.nd - 2)), ib = i - (nbo - (b.nd - 2));
        BatchDim d;
        d.size = p.batch_out[i];
        d.sa = (ia >= 0 && a.sz[ia] != 1) ? a.st[ia] : 0;
        d.sb = (ib >= 0 && b.sz[ib] != 1) ? b.st[ib] : 0;
        d.sc = cst[i];
        if (d.size == 1) continue;
        // Merge into the previous (outer) dim when the two walk memory as one.
        if (!dims.empty()) {
            BatchDim& o = dims.back();
            if (o.sa == d.sa * d.size && o.sb == d.sb * d.size && o.sc == d.sc * d.size) {
                o.size *= d.size;
                o.sa = d.sa;
                o.sb = d.sb;
                o.sc = d.sc;
                continue;
            }
        }
        dims.push_back(d);
    }

    // Inner batch dims over which B is broadcast, and along which A's rows
    // (K-major) and C's rows run on contiguously, fold into M: one taller
    // GEMM instead of a batch of short ones (a [batch, 7, K] . [K, N] product
    // fills 128-row tiles instead of leaving 121 rows of each empty).  Every
    // output is still the same k-chain, so results do not change.
    int64_t M = p.M;
    while (!dims.empty()) {
        const BatchDim& d = dims.back();
        if (d.sb != 0 || a_cs != 1 || d.sa != M * a_rs || d.sc != M * p.N || M * d.size > INT32_MAX) break;
        M *= d.size;
        dims.pop_back();
    }

    Gemm g{};
    g.M = M;
    g.N = p.N;
    g.K = p.K;
    g.A = a.data;
    g.a_rs = a_rs;
    g.a_cs = a_cs;
    g.B = b.data;
    g.b_rs = b_rs;
    g.b_cs = b_cs;
    g.C = C;
    g.c_rs = p.N;
    g.bias = ep.bias;
    g.scale = ep.scale;
    g.apply_scale = ep.apply_scale;
    std::vector<BatchDim> outer;
    const int keep = std::min<int>((int)dims.size(), kMaxBatchDims);
    const int n_outer = (int)dims.size() - keep;
    for (int i = 0; i < n_outer; ++i) outer.push_back(dims[i]);
    g.nb = keep;
    for (int i = 0; i < keep; ++i) {
        const BatchDim& d = dims[n_outer + i];
        g.bsz[i] = d.size;
        g.abs_[i] = d.sa;
        g.bbs[i] = d.sb;
        g.cbs[i] = d.sc;
    }
    return run_gemm(g, outer, mode, s);
}

int check_out(const tlc_tensor* out, const std::vector<int64_t>& shape, const char* name) {
    if (!out) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + " is NULL");
    if (out->ndim != (int)shape.size())
        return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": wrong rank");
    const bool empty = std::find(shape.begin(), shape.end(), int64_t(0)) != shape.end();
    int64_t e = 1;
    for (int i = out->ndim - 1; i >= 0; --i) {
        if (out->sizes[i] != shape[i])
            return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": wrong shape");
        if (!empty && out->sizes[i] != 1 && out->strides[i] != e)  // strides of empty tensors vary
            return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + " must be contiguous");
        e *= shape[i];
    }
    if (e > 0 && !out->data) return set_error(TLC_ERR_INVALID_ARGUMENT, std::string(name) + ": NULL data");
    return TLC_OK;
}

int64_t prod(const std::vector<int64_t>& v) {
    int64_t n = 1;
    for (int64_t x : v) n *= x;
    return n;
}

// sum_to (src/autograd.cpp:24-36) of a contiguous tensor `src` of shape `s`
// into `dst` (shape `target`): repeated sum over dim 0 while it has more dims,
// then keepdim sums over dims that the target holds at size 1.
int sum_to(const float* src, std::vector<int64_t> s, const std::vector<int64_t>& target,
           float* dst, cudaStream_t st) {
    struct Step {
        int64_t outer, D, inner;
    };
    std::vector<Step> steps;
    std::vector<int64_t> cur = s;
    while (cur.size() > target.size()) {
        steps.push_back({1, cur[0], prod(std::vector<int64_t>(cur.begin() + 1, cur.end()))});
        cur.erase(cur.begin());
    }
    for (size_t i = 0; i < target.size(); ++i) {
        if (target[i] == 1 && cur[i] != 1) {
            steps.push_back({prod(std::vector<int64_t>(cur.begin(), cur.begin() + i)), cur[i],
                             prod(std::vector<int64_t>(cur.begin() + i + 1, cur.end()))});
            cur[i] = 1;
        }
    }
    if (steps.empty()) {
        const int64_t n = prod(cur);
        if (n && src != dst)
            TLC_CUDA_TRY(cudaMemcpyAsync(dst, src, sizeof(float) * n, cudaMemcpyDeviceToDevice, st));
        return TLC_OK;
    }
    Scratch ping(st), pong(st);
    const float* in = src;
    for (size_t i = 0; i < steps.size(); ++i) {
        float* out;
        const int64_t n = steps[i].outer * steps[i].inner;
        if (i + 1 == steps.size()) {
            out = dst;
        } else {
            Scratch& sc = (i & 1) ? pong : ping;
            TLC_TRY(sc.alloc(sizeof(float) * std::max<int64_t>(n, 1)));
            out = sc.f();
        }
        TLC_TRY(launch_sum_dim(in, out, steps[i].outer, steps[i].D, steps[i].inner, st));
        in = out;
    }
    return TLC_OK;
}

// One gradient of MatmulBackward: d = sum_to(L . R, target), then
// accumulate_grad into `out` (contiguous, shape = target).
int grad_product(const View& L, const View& R, const std::vector<int64_t>& target, float* out,
                 int accumulate, int mode, cudaStream_t s) {
    Plan p;
    TLC_TRY(plan_matmul(L, R, p));
    const int64_t n_out = prod(target);
    const bool direct = p.full_out == target && !accumulate;
    if (direct) return matmul_planned(p, out, mode, s);
    Scratch prodbuf(s), res(s);
    TLC_TRY(prodbuf.alloc(sizeof(float) * std::max<int64_t>(prod(p.full_out), 1)));
    TLC_TRY(matmul_planned(p, prodbuf.f(), mode, s));
    if (!accumulate) return sum_to(prodbuf.f(), p.full_out, target, out, s);
    TLC_TRY(res.alloc(sizeof(float) * std::max<int64_t>(n_out, 1)));
    TLC_TRY(sum_to(prodbuf.f(), p.full_out, target, res.f(), s));
    return launch_add(out, res.f(), out, n_out, s);  // grad = add(grad, d)
}

View transpose_last2(View v) {
    std::swap(v.sz[v.nd - 1], v.sz[v.nd - 2]);
    std::swap(v.st[v.nd - 1], v.st[v.nd - 2]);
    return v;
}

// Insert a size-1 dim before position `pos` (stride irrelevant).
View insert_unit(View v, int pos) {
    for (int i = v.nd; i > pos; --i) {
        v.sz[i] = v.sz[i - 1];
        v.st[i] = v.st[i - 1];
    }
    v.sz[pos] = 1;
    v.st[pos] = pos + 1 < v.nd + 1 ? v.sz[pos + 1] * v.st[pos + 1] : 1;
    v.nd += 1;
    return v;
}

int backward_impl(const tlc_tensor* grad, const tlc_tensor* a, const tlc_tensor* b,
                  tlc_tensor* da, tlc_tensor* db, int accumulate, int mode, cudaStream_t s) {
    View va, vb, vg;
    TLC_TRY(to_view(a, va, "a"));
    TLC_TRY(to_view(b, vb, "b"));
    TLC_TRY(to_view(grad, vg, "grad"));
    Plan p;
    TLC_TRY(plan_matmul(va, vb, p));
    if (vg.nd != (int)p.result.size())
        return set_error(TLC_ERR_INVALID_ARGUMENT, "matmul_backward: grad has the wrong rank");
    for (int i = 0; i < vg.nd; ++i)
        if (vg.sz[i] != p.result[i])
            return set_error(TLC_ERR_INVALID_ARGUMENT, "matmul_backward: grad has the wrong shape");
    // grad_output comes squeezed; unsqueeze it (src/autograd.cpp:351-362).
    if (p.sq_a) vg = insert_unit(vg, vg.nd > 0 ? vg.nd - 1 : 0);
    if (p.sq_b) vg = insert_unit(vg, vg.nd);
    std::vector<int64_t> ta(p.a.sz, p.a.sz + p.a.nd), tb(p.b.sz, p.b.sz + p.b.nd);
    const bool want_a = da && da->data, want_b = db && db->data;
    if (want_a) TLC_TRY(check_out(da, std::vector<int64_t>(va.sz, va.sz + va.nd), "da"));
    if (want_b) TLC_TRY(check_out(db, std::vector<int64_t>(vb.sz, vb.sz + vb.nd), "db"));
    // dA = sum_to(grad . B^T, A.shape); dB = sum_to(A^T . grad, B.shape)
    // (src/autograd.cpp:370-375); transposes are strided views, never copies.
    if (want_a) TLC_TRY(grad_product(vg, transpose_last2(p.b), ta, da->data, accumulate, mode, s));
    if (want_b) TLC_TRY(grad_product(transpose_last2(p.a), vg, tb, db->data, accumulate, mode, s));
    return TLC_OK;
}

// ---- host-buffer forms --------------------------------------------------------------

// Extent (in elements) of storage a strided view touches, from its first element.
int64_t span_of(const View& v) {
    if (v.numel() == 0) return 0;
    int64_t hi = 0;
    for (int i = 0; i < v.nd; ++i) hi += (v.sz[i] - 1) * v.st[i];
    return hi + 1;
}

struct DevCopy {
    Scratch buf;
    tlc_tensor t{};
    explicit DevCopy(cudaStream_t s) : buf(s) {}
    int up(const tlc_tensor* h, cudaStream_t s) {
        View v;
        TLC_TRY(to_view(h, v, "tensor"));
        t = *h;
        const int64_t n = span_of(v);
        TLC_TRY(buf.alloc(sizeof(float) * std::max<int64_t>(n, 1)));
        if (n) TLC_CUDA_TRY(cudaMemcpyAsync(buf.p, h->data, sizeof(float) * n, cudaMemcpyHostToDevice, s));
        t.data = buf.f();
        return TLC_OK;
    }
    int alloc_like(const tlc_tensor* h) {
        View v;
        TLC_TRY(to_view(h, v, "tensor"));
        t = *h;
        TLC_TRY(buf.alloc(sizeof(float) * std::max<int64_t>(span_of(v), 1)));
        t.data = buf.f();
        return TLC_OK;
    }
};

// Streams the library keeps per device (and context) for the host-buffer
// forms: [0] the work, [1] uploads and [2] downloads of the pipelined form.
cudaStream_t library_stream(int which) {
    static DeviceOnce once;
    static cudaStream_t streams[64][3] = {};
    int dev = 0;
    const int st = device_once(once, [](int d) -> int {
        for (int i = 0; i < 3; ++i) {
            streams[d][i] = nullptr;
            TLC_CUDA_TRY(cudaStreamCreateWithFlags(&streams[d][i], cudaStreamNonBlocking));
        }
        return TLC_OK;
    }, &dev);
    return st == TLC_OK ? streams[dev][which] : nullptr;
}

cudaStream_t host_stream() { return library_stream(0); }

// Upload and download streams per device for the pipelined host-buffer form.
void copy_streams(cudaStream_t& in, cudaStream_t& out) {
    in = library_stream(1);
    out = library_stream(2);
}

View dense_view(float* data, std::initializer_list<int64_t> sizes) {
    return contiguous_view(data, std::vector<int64_t>(sizes));
}

// Events of one pipelined call, destroyed with it.
struct Events {
    std::vector<cudaEvent_t> ev;
    cudaEvent_t make() {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        ev.push_back(e);
        return e;
    }
    ~Events() {
        for (auto e : ev) cudaEventDestroy(e);
    }
};

constexpr int64_t kPipeMinBytes = 64ll << 20;  // smaller problems: one upload, one download
constexpr int kPipeChunks = 32;

// Host-buffer matmul with the transfers pipelined against the GEMMs: the
// output is cut into chunks, along the flattened batch when every operand is
// either batched like the output or one shared matrix, else along the rows of
// A and C; chunk i's upload (stream `in`), GEMM (stream `s`) and download
// (stream `out`) overlap with its neighbours', so the host link's two
// directions and the GEMM run at once.  Operands and result must be dense
// host buffers; returns TLC_ERR_UNSUPPORTED otherwise (the caller then takes
// the sequential path).  Chunking does not change any element's arithmetic.
int matmul_host_pipelined(const Plan& p, const View& ha, const View& hb, float* out_host, int mode,
                          cudaStream_t s) {
    if (!ha.contiguous() || !hb.contiguous()) return TLC_ERR_UNSUPPORTED;
    const int64_t M = p.M, N = p.N, K = p.K;
    const int64_t nbatch = prod(p.batch_out);
    const int64_t bytes = 4 * (ha.numel() + hb.numel() + prod(p.full_out));
    if (bytes < kPipeMinBytes || K == 0 || M == 0 || N == 0) return TLC_ERR_UNSUPPORTED;
    auto batched_like_out = [&](const View& v) {
        if (v.nd - 2 != (int)p.batch_out.size()) return false;
        for (int i = 0; i < v.nd - 2; ++i)
            if (v.sz[i] != p.batch_out[i]) return false;
        return true;
    };
    auto plain = [&](const View& v) {
        int64_t bp = 1;
        for (int i = 0; i < v.nd - 2; ++i) bp *= v.sz[i];
        return bp == 1;
    };
    const bool by_batch = nbatch >= 2 && (batched_like_out(p.a) || plain(p.a)) &&
                          (batched_like_out(p.b) || plain(p.b));
    const bool by_rows = nbatch == 1 && M >= 2 * 256;
    if (!by_batch && !by_rows) return TLC_ERR_UNSUPPORTED;
    const bool a_batched = by_batch && !plain(p.a), b_batched = by_batch && !plain(p.b);

    cudaStream_t in = nullptr, out = nullptr;
    copy_streams(in, out);
    if (!in || !out) return TLC_ERR_UNSUPPORTED;
    Scratch dA(s), dB(s), dC(s);
    TLC_TRY(dA.alloc(sizeof(float) * ha.numel()));
    TLC_TRY(dB.alloc(sizeof(float) * hb.numel()));
    TLC_TRY(dC.alloc(sizeof(float) * prod(p.full_out)));
    Events E;
    cudaEvent_t ready = E.make();
    if (!ready) return set_error(TLC_ERR_CUDA, "cudaEventCreate failed");
    TLC_CUDA_TRY(cudaEventRecord(ready, s));  // the allocations precede every copy
    TLC_CUDA_TRY(cudaStreamWaitEvent(in, ready, 0));
    TLC_CUDA_TRY(cudaStreamWaitEvent(out, ready, 0));
    // shared operands go up whole, first
    if (!a_batched && !by_rows)
        TLC_CUDA_TRY(cudaMemcpyAsync(dA.p, ha.data, sizeof(float) * ha.numel(), cudaMemcpyHostToDevice, in));
    if (!b_batched)
        TLC_CUDA_TRY(cudaMemcpyAsync(dB.p, hb.data, sizeof(float) * hb.numel(), cudaMemcpyHostToDevice, in));

    const int64_t units = by_batch ? nbatch : (M + 255) / 256;  // batch entries or 256-row blocks
    const int64_t chunks = std::min<int64_t>(kPipeChunks, units);
    for (int64_t c = 0; c < chunks; ++c) {
        int64_t u0, u1;
        tlc_shard_range(units, (int)chunks, (int)c, &u0, &u1);
        if (u1 <= u0) continue;
        View a, b, o;
        int64_t a_off = 0, a_n = 0, b_off = 0, b_n = 0, o_off, o_n;
        if (by_batch) {
            const int64_t cnt = u1 - u0;
            if (a_batched) {
                a_off = u0 * M * K;
                a_n = cnt * M * K;
                a = dense_view(dA.f() + a_off, {cnt, M, K});
            } else {
                a = dense_view(dA.f(), {M, K});
            }
            if (b_batched) {
                b_off = u0 * K * N;
                b_n = cnt * K * N;
                b = dense_view(dB.f() + b_off, {cnt, K, N});
            } else {
                b = dense_view(dB.f(), {K, N});
            }
            o_off = u0 * M * N;
            o_n = cnt * M * N;
            o = dense_view(dC.f() + o_off, {cnt, M, N});
        } else {
            const int64_t r0 = u0 * 256, r1 = std::min(M, u1 * 256);
            a_off = r0 * K;
            a_n = (r1 - r0) * K;
            a = dense_view(dA.f() + a_off, {r1 - r0, K});
            b = dense_view(dB.f(), {K, N});
            o_off = r0 * N;
            o_n = (r1 - r0) * N;
            o = dense_view(dC.f() + o_off, {r1 - r0, N});
        }
        if (a_n)
            TLC_CUDA_TRY(cudaMemcpyAsync(dA.f() + a_off, ha.data + a_off, sizeof(float) * a_n,
                                         cudaMemcpyHostToDevice, in));
        if (b_n)
            TLC_CUDA_TRY(cudaMemcpyAsync(dB.f() + b_off, hb.data + b_off, sizeof(float) * b_n,
                                         cudaMemcpyHostToDevice, in));
        cudaEvent_t up = E.make(), done = E.make();
        if (!up || !done) return set_error(TLC_ERR_CUDA, "cudaEventCreate failed");
        TLC_CUDA_TRY(cudaEventRecord(up, in));
        TLC_CUDA_TRY(cudaStreamWaitEvent(s, up, 0));
        Plan q;
        TLC_TRY(plan_matmul(a, b, q));
        TLC_TRY(matmul_planned(q, const_cast<float*>(o.data), mode, s));
        TLC_CUDA_TRY(cudaEventRecord(done, s));
        TLC_CUDA_TRY(cudaStreamWaitEvent(out, done, 0));
        TLC_CUDA_TRY(cudaMemcpyAsync(out_host + o_off, o.data, sizeof(float) * o_n,
                                     cudaMemcpyDeviceToHost, out));
    }
    cudaEvent_t drained = E.make();
    if (!drained) return set_error(TLC_ERR_CUDA, "cudaEventCreate failed");
    TLC_CUDA_TRY(cudaEventRecord(drained, out));
    TLC_CUDA_TRY(cudaStreamWaitEvent(s, drained, 0));  // frees (on s) follow the downloads
    return TLC_OK;
}

}  // namespace
}  // namespace tlc

using namespace tlc;

extern "C" {

int tlc_version(void) { return 100; }

const char* tlc_status_string(int st) {
    switch (st) {
        case TLC_OK: return "ok";
        case TLC_ERR_INVALID_ARGUMENT: return "invalid argument";
        case TLC_ERR_UNSUPPORTED: return "unsupported";
        case TLC_ERR_CUDA: return "CUDA error";
        case TLC_ERR_OUT_OF_MEMORY: return "out of memory";
        case TLC_ERR_TIMEOUT: return "kernel wait timed out";
        case TLC_ERR_IO: return "I/O error";
        default: return "unknown status";
    }
}

const char* tlc_last_error(void) { return t_last_error.c_str(); }

uint64_t tlc_launch_count(void) { return g_launches.load(); }

int tlc_mode_from_string(const char* name) {
    if (!name) return -1;
    std::string s(name);
    for (auto& c : s) c = (char)std::tolower((unsigned char)c);
    if (s == "exact" || s == "fp32" || s == "fp32-exact") return TLC_MODE_EXACT;
    if (s == "tf32") return TLC_MODE_TF32;
    if (s == "3xtf32") return TLC_MODE_3XTF32;
    return -1;
}

int tlc_default_mode(void) {
    static int mode = [] {
        const char* e = std::getenv("TL_GEMM_MODE");
        int m = e ? tlc_mode_from_string(e) : TLC_MODE_EXACT;
        return m < 0 ? (int)TLC_MODE_EXACT : m;
    }();
    return mode;
}

int tlc_device_count(int* count) {
    clear_error();
    TLC_CUDA_TRY(cudaGetDeviceCount(count));
    return TLC_OK;
}
int tlc_set_device(int device) {
    clear_error();
    TLC_CUDA_TRY(cudaSetDevice(device));
    return TLC_OK;
}
int tlc_get_device(int* device) {
    clear_error();
    TLC_CUDA_TRY(cudaGetDevice(device));
    return TLC_OK;
}
int tlc_malloc(void** ptr, size_t bytes) {
    clear_error();
    *ptr = nullptr;
    if (bytes == 0) return TLC_OK;
    TLC_CUDA_TRY(cudaMalloc(ptr, bytes));
    return TLC_OK;
}
int tlc_free(void* ptr) {
    clear_error();
    if (ptr) TLC_CUDA_TRY(cudaFree(ptr));
    return TLC_OK;
}
int tlc_malloc_host(void** ptr, size_t bytes) {
    clear_error();
    *ptr = nullptr;
    if (bytes == 0) return TLC_OK;
    TLC_CUDA_TRY(cudaMallocHost(ptr, bytes));
    return TLC_OK;
}
int tlc_free_host(void* ptr) {
    clear_error();
    if (ptr) TLC_CUDA_TRY(cudaFreeHost(ptr));
    return TLC_OK;
}
int tlc_memcpy(void* dst, const void* src, size_t bytes, int kind, void* stream) {
    clear_error();
    cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice
                       : kind == 1 ? cudaMemcpyDeviceToHost
                                   : cudaMemcpyDeviceToDevice;
    if (kind < 0 || kind > 2) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_memcpy: bad kind");
    if (bytes) TLC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, (cudaStream_t)stream));
    return TLC_OK;
}
int tlc_memset_zero(void* dst, size_t bytes, void* stream) {
    clear_error();
    if (bytes) TLC_CUDA_TRY(cudaMemsetAsync(dst, 0, bytes, (cudaStream_t)stream));
    return TLC_OK;
}
namespace tlc {
namespace {
// Reads and clears the device error word of the current device.
int take_device_error() {
    int* w = nullptr;
    TLC_TRY(tc_error_word(&w));
    int v = 0;
    TLC_CUDA_TRY(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) {
        const int zero = 0;
        TLC_CUDA_TRY(cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice));
        return set_error(TLC_ERR_TIMEOUT,
                         "a bounded wait inside a tensor-core GEMM kernel timed out (site " +
                             std::to_string(v) + ")");
    }
    return TLC_OK;
}
}  // namespace
}  // namespace tlc

int tlc_stream_synchronize(void* stream) {
    clear_error();
    TLC_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    return take_device_error();
}

int tlc_check_device_errors(void) {
    clear_error();
    TLC_CUDA_TRY(cudaDeviceSynchronize());
    return take_device_error();
}

int tlc_selftest_bounded_wait(uint64_t timeout_ns) {
    clear_error();
    TLC_CUDA_TRY(cudaDeviceSynchronize());
    TLC_TRY(take_device_error());
    TLC_TRY(bounded_wait_selftest(timeout_ns, nullptr));
    TLC_CUDA_TRY(cudaDeviceSynchronize());
    return take_device_error();
}

int tlc_matmul_shape(const tlc_tensor* a, const tlc_tensor* b, int32_t* out_ndim,
                     int64_t* out_sizes) {
    clear_error();
    View va, vb;
    TLC_TRY(to_view(a, va, "a"));
    TLC_TRY(to_view(b, vb, "b"));
    Plan p;
    TLC_TRY(plan_matmul(va, vb, p));
    if (out_ndim) *out_ndim = (int32_t)p.result.size();
    if (out_sizes)
        for (size_t i = 0; i < p.result.size(); ++i) out_sizes[i] = p.result[i];
    return TLC_OK;
}

int tlc_matmul(const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, int mode, void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve_mode(mode, m));
    View va, vb;
    TLC_TRY(to_view(a, va, "a"));
    TLC_TRY(to_view(b, vb, "b"));
    Plan p;
    TLC_TRY(plan_matmul(va, vb, p));
    TLC_TRY(check_out(out, p.result, "out"));
    return matmul_planned(p, out->data, m, (cudaStream_t)stream);
}

int tlc_matmul_backward(const tlc_tensor* grad, const tlc_tensor* a, const tlc_tensor* b,
                        tlc_tensor* da, tlc_tensor* db, int accumulate, int mode, void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve_mode(mode, m));
    return backward_impl(grad, a, b, da, db, accumulate, m, (cudaStream_t)stream);
}

int tlc_gemm(const tlc_gemm_desc* d, int mode, void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve_mode(mode, m));
    if (!d) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gemm: desc is NULL");
    if (d->M < 0 || d->N < 0 || d->K < 0 || d->batch_ndim < 0 || d->batch_ndim > 3)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gemm: bad sizes");
    Gemm g{};
    g.M = d->M;
    g.N = d->N;
    g.K = d->K;
    g.A = d->A;
    g.B = d->B;
    g.C = d->C;
    g.c_rs = d->c_rs;
    if (!unit_stride_2d(d->M, d->K, d->a_rs, d->a_cs, g.a_rs, g.a_cs) ||
        !unit_stride_2d(d->K, d->N, d->b_rs, d->b_cs, g.b_rs, g.b_cs))
        return set_error(TLC_ERR_INVALID_ARGUMENT,
                         "tlc_gemm: A and B need a unit stride in one matrix dim");
    g.nb = d->batch_ndim;
    for (int i = 0; i < g.nb; ++i) {
        g.bsz[i] = d->batch_sizes[i];
        g.abs_[i] = d->a_bstride[i];
        g.bbs[i] = d->b_bstride[i];
        g.cbs[i] = d->c_bstride[i];
        if (g.bsz[i] < 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gemm: bad batch size");
    }
    if (g.batch() == 0 || g.M == 0 || g.N == 0) return TLC_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (g.K == 0) {
        // C is strided per batch; clear row by row through a zero-K exact GEMM.
        return gemm_exact(g, s);
    }
    return run_gemm(g, {}, m, s);
}

int tlc_matmul_host(const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, int mode,
                    void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve_mode(mode, m));
    View va, vb;
    TLC_TRY(to_view(a, va, "a"));
    TLC_TRY(to_view(b, vb, "b"));
    Plan p;
    TLC_TRY(plan_matmul(va, vb, p));
    TLC_TRY(check_out(out, p.result, "out"));
    cudaStream_t s = stream ? (cudaStream_t)stream : host_stream();
    {
        const int st = matmul_host_pipelined(p, va, vb, out->data, m, s);
        if (st == TLC_OK) {
            TLC_CUDA_TRY(cudaStreamSynchronize(s));
            return take_device_error();
        }
        if (st != TLC_ERR_UNSUPPORTED) return st;
        clear_error();
    }
    {
        DevCopy da(s), db(s), dc(s);
        TLC_TRY(da.up(a, s));
        TLC_TRY(db.up(b, s));
        TLC_TRY(dc.alloc_like(out));
        View dva, dvb;
        TLC_TRY(to_view(&da.t, dva, "a"));
        TLC_TRY(to_view(&db.t, dvb, "b"));
        Plan q;
        TLC_TRY(plan_matmul(dva, dvb, q));
        TLC_TRY(matmul_planned(q, dc.t.data, m, s));
        const int64_t n = prod(p.result);
        if (n) TLC_CUDA_TRY(cudaMemcpyAsync(out->data, dc.t.data, sizeof(float) * n, cudaMemcpyDeviceToHost, s));
    }
    TLC_CUDA_TRY(cudaStreamSynchronize(s));
    return take_device_error();
}

int tlc_matmul_backward_host(const tlc_tensor* grad, const tlc_tensor* a, const tlc_tensor* b,
                             tlc_tensor* da, tlc_tensor* db, int accumulate, int mode,
                             void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve_mode(mode, m));
    cudaStream_t s = stream ? (cudaStream_t)stream : host_stream();
    {
        DevCopy dg(s), dA(s), dB(s), gA(s), gB(s);
        TLC_TRY(dg.up(grad, s));
        TLC_TRY(dA.up(a, s));
        TLC_TRY(dB.up(b, s));
        const bool want_a = da && da->data, want_b = db && db->data;
        tlc_tensor ta{}, tb{};
        if (want_a) {
            TLC_TRY(accumulate ? gA.up(da, s) : gA.alloc_like(da));
            ta = gA.t;
        }
        if (want_b) {
            TLC_TRY(accumulate ? gB.up(db, s) : gB.alloc_like(db));
            tb = gB.t;
        }
        TLC_TRY(backward_impl(&dg.t, &dA.t, &dB.t, want_a ? &ta : nullptr, want_b ? &tb : nullptr,
                              accumulate, m, s));
        if (want_a) {
            View v;
            TLC_TRY(to_view(da, v, "da"));
            if (v.numel()) TLC_CUDA_TRY(cudaMemcpyAsync(da->data, ta.data, sizeof(float) * v.numel(), cudaMemcpyDeviceToHost, s));
        }
        if (want_b) {
            View v;
            TLC_TRY(to_view(db, v, "db"));
            if (v.numel()) TLC_CUDA_TRY(cudaMemcpyAsync(db->data, tb.data, sizeof(float) * v.numel(), cudaMemcpyDeviceToHost, s));
        }
    }
    TLC_CUDA_TRY(cudaStreamSynchronize(s));
    return take_device_error();
}

int tlc_sum_dim(const float* in, float* out, int64_t outer, int64_t D, int64_t inner,
                void* stream) {
    clear_error();
    if (outer < 0 || D < 0 || inner < 0)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_sum_dim: negative size");
    return launch_sum_dim(in, out, outer, D, inner, (cudaStream_t)stream);
}

int tlc_sum_dim_from(const float* in, const float* init, float* out, int64_t outer, int64_t D,
                     int64_t inner, void* stream) {
    clear_error();
    if (outer < 0 || D < 0 || inner < 0)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_sum_dim_from: negative size");
    return launch_sum_dim(in, out, outer, D, inner, (cudaStream_t)stream, init);
}

int tlc_add(const float* a, const float* b, float* out, int64_t n, void* stream) {
    clear_error();
    if (n < 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_add: negative size");
    return launch_add(a, b, out, n, (cudaStream_t)stream);
}

int tlc_contiguous(const tlc_tensor* src, float* dst, void* stream) {
    clear_error();
    View v;
    TLC_TRY(to_view(src, v, "src"));
    return launch_strided_copy(v.data, v.nd, v.sz, v.st, dst, (cudaStream_t)stream);
}

// ---- fused GEMM and the glue around it ----------------------------------------------

namespace tlc {
namespace {

std::vector<int64_t> shape_of(const View& v) { return std::vector<int64_t>(v.sz, v.sz + v.nd); }

// `v` itself when contiguous, else a contiguous copy in `sc`.
int dense_input(const View& v, Scratch& sc, const float** out, cudaStream_t s) {
    if (v.contiguous() || v.numel() == 0) {
        *out = v.data;
        return TLC_OK;
    }
    TLC_TRY(sc.alloc(sizeof(float) * (size_t)v.numel()));
    TLC_TRY(launch_strided_copy(v.data, v.nd, v.sz, v.st, sc.f(), s));
    *out = sc.f();
    return TLC_OK;
}

// Broadcast strides of `v` against an output of rank nd (0 on broadcast dims).
void bcast_strides(const View& v, int nd, int64_t* st) {
    for (int i = 0; i < nd; ++i) {
        const int iv = i - (nd - v.nd);
        st[i] = (iv >= 0 && v.sz[iv] != 1) ? v.st[iv] : 0;
    }
}

}  // namespace
}  // namespace tlc

using namespace tlc;

int tlc_matmul_fused(const tlc_tensor* a, const tlc_tensor* b, float scale, const tlc_tensor* bias,
                     tlc_tensor* out, int mode, void* stream) {
    clear_error();
    int m;
    TLC_TRY(resolve_mode(mode, m));
    cudaStream_t s = (cudaStream_t)stream;
    View va, vb;
    TLC_TRY(to_view(a, va, "a"));
    TLC_TRY(to_view(b, vb, "b"));
    Plan p;
    TLC_TRY(plan_matmul(va, vb, p));
    TLC_TRY(check_out(out, p.result, "out"));
    Epilogue ep;
    ep.scale = scale;
    ep.apply_scale = scale != 1.0f ? 1 : 0;
    Scratch sc(s);
    if (bias) {
        View vbias;
        TLC_TRY(to_view(bias, vbias, "bias"));
        if (vbias.nd != 1 || vbias.sz[0] != p.N)
            return set_error(TLC_ERR_INVALID_ARGUMENT,
                             "matmul_fused: bias must be a 1-D tensor of length N = " +
                                 std::to_string(p.N));
        TLC_TRY(dense_input(vbias, sc, &ep.bias, s));
    }
    return matmul_planned(p, out->data, m, s, ep);
}

int tlc_add_tensors(const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, void* stream) {
    clear_error();
    View va, vb;
    TLC_TRY(to_view(a, va, "a"));
    TLC_TRY(to_view(b, vb, "b"));
    std::vector<int64_t> shape;
    TLC_TRY(broadcast_shape(shape_of(va), shape_of(vb), shape));
    TLC_TRY(check_out(out, shape, "out"));
    const int nd = (int)shape.size();
    int64_t sa[TLC_MAX_DIMS] = {}, sb[TLC_MAX_DIMS] = {};
    bcast_strides(va, nd, sa);
    bcast_strides(vb, nd, sb);
    return launch_elementwise(va.data, vb.data, 0.0f, out->data, prod(shape), nd, shape.data(), sa,
                              sb, 0, (cudaStream_t)stream);
}

int tlc_scale(const tlc_tensor* x, float scale, tlc_tensor* out, void* stream) {
    clear_error();
    View vx;
    TLC_TRY(to_view(x, vx, "x"));
    const std::vector<int64_t> shape = shape_of(vx);
    TLC_TRY(check_out(out, shape, "out"));
    const int nd = (int)shape.size();
    int64_t sa[TLC_MAX_DIMS] = {}, sb[TLC_MAX_DIMS] = {};
    bcast_strides(vx, nd, sa);
    return launch_elementwise(vx.data, nullptr, scale, out->data, prod(shape), nd, shape.data(), sa,
                              sb, 1, (cudaStream_t)stream);
}

int tlc_softmax(const tlc_tensor* x, tlc_tensor* out, void* stream) {
    clear_error();
    cudaStream_t s = (cudaStream_t)stream;
    View vx;
    TLC_TRY(to_view(x, vx, "x"));
    if (vx.nd == 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "Softmax requires at least 1D tensor");
    const std::vector<int64_t> shape = shape_of(vx);
    TLC_TRY(check_out(out, shape, "out"));
    const int64_t D = shape.back(), n = prod(shape);
    if (D == 0 || n == 0) return TLC_OK;
    Scratch sc(s);
    const float* xd;
    TLC_TRY(dense_input(vx, sc, &xd, s));
    return launch_softmax(xd, out->data, n / D, D, s);
}

int tlc_softmax_backward(const tlc_tensor* grad, const tlc_tensor* y, tlc_tensor* dx, void* stream) {
    clear_error();
    cudaStream_t s = (cudaStream_t)stream;
    View vg, vy;
    TLC_TRY(to_view(grad, vg, "grad"));
    TLC_TRY(to_view(y, vy, "y"));
    if (vy.nd == 0) return set_error(TLC_ERR_INVALID_ARGUMENT, "softmax_backward: y must be at least 1-D");
    const std::vector<int64_t> shape = shape_of(vy);
    if (shape_of(vg) != shape)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "softmax_backward: grad and y differ in shape");
    TLC_TRY(check_out(dx, shape, "dx"));
    const int64_t D = shape.back(), n = prod(shape);
    if (D == 0 || n == 0) return TLC_OK;
    Scratch sg(s), sy(s);
    const float *gd, *yd;
    TLC_TRY(dense_input(vg, sg, &gd, s));
    TLC_TRY(dense_input(vy, sy, &yd, s));
    return launch_softmax_backward(gd, yd, dx->data, n / D, D, s);
}

int tlc_sum_to(const tlc_tensor* x, tlc_tensor* out, void* stream) {
    clear_error();
    cudaStream_t s = (cudaStream_t)stream;
    View vx;
    TLC_TRY(to_view(x, vx, "x"));
    if (!out) return set_error(TLC_ERR_INVALID_ARGUMENT, "out is NULL");
    const std::vector<int64_t> shape = shape_of(vx);
    const std::vector<int64_t> target(out->sizes, out->sizes + std::max(0, std::min(out->ndim, TLC_MAX_DIMS)));
    if (target.size() > shape.size())
        return set_error(TLC_ERR_INVALID_ARGUMENT, "sum_to: target has more dims than the input");
    const size_t off = shape.size() - target.size();
    for (size_t i = 0; i < target.size(); ++i)
        if (target[i] != shape[off + i] && target[i] != 1)
            return set_error(TLC_ERR_INVALID_ARGUMENT, "sum_to: target shape is not a reduction of the input");
    TLC_TRY(check_out(out, target, "out"));
    Scratch sc(s);
    const float* xd;
    TLC_TRY(dense_input(vx, sc, &xd, s));
    return sum_to(xd, shape, target, out->data, s);
}

int tlc_shard_range(int64_t count, int world, int rank, int64_t* begin, int64_t* end) {
    clear_error();
    if (count < 0 || world < 1 || rank < 0 || rank >= world || !begin || !end)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_shard_range: bad arguments");
    const int64_t base = count / world, extra = count % world;
    *begin = rank * base + std::min<int64_t>(rank, extra);
    *end = *begin + base + (rank < extra ? 1 : 0);
    return TLC_OK;
}

int tlc_shard_cols(int64_t N, int world, int rank, int64_t align, int64_t* begin, int64_t* end) {
    clear_error();
    if (N < 0 || world < 1 || rank < 0 || rank >= world || align < 1 || !begin || !end)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_shard_cols: bad arguments");
    const int64_t units = (N + align - 1) / align;
    int64_t ub, ue;
    tlc_shard_range(units, world, rank, &ub, &ue);
    *begin = std::min(N, ub * align);
    *end = std::min(N, ue * align);
    return TLC_OK;
}

int tlc_gather_colblocks(const float* gathered, float* out, int64_t M, int64_t N, int world,
                         const int64_t* col_begin, void* stream) {
    clear_error();
    if (M < 0 || N < 0 || !col_begin)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_gather_colblocks: bad arguments");
    return launch_gather_colblocks(gathered, out, M, N, world, col_begin, (cudaStream_t)stream);
}

}  // extern "C"
