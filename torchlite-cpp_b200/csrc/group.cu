// Device groups: one tl::matmul over several GPUs of the box, from one
// process and the caller's single host thread (include/tlc.h, "device groups").
//
// The reference parallelises a matmul over host threads only: its batch loop
// (src/ops.cpp:655-674) runs gemm_mt, which cuts each product into row bands,
// one std::thread each (src/ops.cpp:569-587).  A group cuts it over GPUs:
//   - a batched or broadcast product over its flattened batch: GPU i takes the
//     contiguous entries [begin_i, end_i) (tlc_shard_range); an operand that
//     broadcasts over the batch goes whole to every GPU;
//   - a single product from host buffers over row blocks of A and C (each
//     GPU's share of A and of C is one contiguous host range, so its copies
//     are plain DMA transfers over its own host link);
//   - a single product on device memory over output column blocks: every GPU
//     gets A whole (one NCCL broadcast from the first GPU) and its own column
//     block of B, and writes its block of C back into the caller's C.
// MatmulBackward of a batch split keeps dA (and a batched dB) on each GPU's
// shard; the dB of a broadcast B, a sum over every entry, is formed by an
// ordered chain: GPU i continues the running sum of GPU i-1 over its own
// entries (tlc_sum_dim_from), so the additions are those of the reference's
// single sequential sum_to and exact mode stays bit-identical.
//
// Host-buffer calls run one worker thread per group member, each calling the
// single-device tlc_matmul_host / tlc_matmul_backward_host on its share (those
// pipeline their own copies against the GEMMs).  Device-memory calls are
// asynchronous: peer copies, the NCCL broadcast and the GEMMs are queued on
// one stream per member, ordered after the caller's stream with events, and
// the caller's stream waits for every member before the call returns.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2), so a program that never
// uses a group does not need it; without it the broadcast falls back to peer
// copies.  A device may appear more than once in a group (its shares then run
// side by side on that device); NCCL is used only when all devices differ.
#include <dlfcn.h>
#include <nccl.h>

#include <condition_variable>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace tlc {
namespace {

// ---- NCCL, resolved at run time --------------------------------------------------------

struct Nccl {
    decltype(&ncclCommInitAll) init_all = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclBroadcast) broadcast = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

const Nccl& nccl() {
    static Nccl n = [] {
        Nccl r;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return r;
        r.init_all = reinterpret_cast<decltype(r.init_all)>(dlsym(h, "ncclCommInitAll"));
        r.destroy = reinterpret_cast<decltype(r.destroy)>(dlsym(h, "ncclCommDestroy"));
        r.broadcast = reinterpret_cast<decltype(r.broadcast)>(dlsym(h, "ncclBroadcast"));
        r.group_start = reinterpret_cast<decltype(r.group_start)>(dlsym(h, "ncclGroupStart"));
        r.group_end = reinterpret_cast<decltype(r.group_end)>(dlsym(h, "ncclGroupEnd"));
        r.error_string = reinterpret_cast<decltype(r.error_string)>(dlsym(h, "ncclGetErrorString"));
        r.ok = r.init_all && r.destroy && r.broadcast && r.group_start && r.group_end && r.error_string;
        return r;
    }();
    return n;
}

// ---- worker threads ----------------------------------------------------------------------

// n threads that run one job together: run(fn) calls fn(i) on worker i for
// every i and returns when all are done.
class Workers {
  public:
    explicit Workers(int n) : n_(n) {
        for (int i = 0; i < n; ++i) th_.emplace_back([this, i] { loop(i); });
    }
    ~Workers() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : th_) t.join();
    }
    void run(const std::function<void(int)>& fn) {
        std::unique_lock<std::mutex> lk(mu_);
        job_ = &fn;
        left_ = n_;
        ++gen_;
        cv_.notify_all();
        done_.wait(lk, [&] { return left_ == 0; });
        job_ = nullptr;
    }

  private:
    void loop(int i) {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(int)>* job;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
                job = job_;
            }
            (*job)(i);
            std::lock_guard<std::mutex> lk(mu_);
            if (--left_ == 0) done_.notify_all();
        }
    }
    int n_;
    std::vector<std::thread> th_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::function<void(int)>* job_ = nullptr;
    uint64_t gen_ = 0;
    int left_ = 0;
    bool stop_ = false;
};

// ---- views -----------------------------------------------------------------------------

int64_t prod_dims(const tlc_tensor& t, int from, int to) {
    int64_t n = 1;
    for (int i = from; i < to; ++i) n *= t.sizes[i];
    return n;
}

bool dense(const tlc_tensor& t) {
    int64_t e = 1;
    for (int i = t.ndim - 1; i >= 0; --i) {
        if (t.sizes[i] != 1 && t.strides[i] != e) return false;
        e *= t.sizes[i];
    }
    return true;
}

tlc_tensor view3(float* data, int64_t b, int64_t r, int64_t c) {
    tlc_tensor t{};
    t.data = data;
    t.ndim = 3;
    t.sizes[0] = b;
    t.sizes[1] = r;
    t.sizes[2] = c;
    t.strides[0] = r * c;
    t.strides[1] = c;
    t.strides[2] = 1;
    return t;
}

tlc_tensor view2(float* data, int64_t r, int64_t c, int64_t rs, int64_t cs) {
    tlc_tensor t{};
    t.data = data;
    t.ndim = 2;
    t.sizes[0] = r;
    t.sizes[1] = c;
    t.strides[0] = rs;
    t.strides[1] = cs;
    return t;
}

// How a product splits over the batch: both operands dense, each either
// batched exactly like the output or one matrix shared by every entry.
struct BatchSplit {
    bool ok = false;
    int64_t nbatch = 0, M = 0, N = 0, K = 0;
    bool a_batched = false, b_batched = false;
};

BatchSplit batch_split(const tlc_tensor& a, const tlc_tensor& b, const int64_t* out_sizes,
                       int out_nd) {
    BatchSplit s;
    if (a.ndim < 2 || b.ndim < 2 || out_nd < 3 || !dense(a) || !dense(b)) return s;
    s.M = a.sizes[a.ndim - 2];
    s.K = a.sizes[a.ndim - 1];
    s.N = b.sizes[b.ndim - 1];
    s.nbatch = 1;
    for (int i = 0; i < out_nd - 2; ++i) s.nbatch *= out_sizes[i];
    auto like_out = [&](const tlc_tensor& t) {
        if (t.ndim != out_nd) return false;
        for (int i = 0; i < out_nd - 2; ++i)
            if (t.sizes[i] != out_sizes[i]) return false;
        return true;
    };
    auto plain = [&](const tlc_tensor& t) { return prod_dims(t, 0, t.ndim - 2) == 1; };
    if (!(like_out(a) || plain(a)) || !(like_out(b) || plain(b))) return s;
    s.a_batched = !plain(a);
    s.b_batched = !plain(b);
    s.ok = s.nbatch >= 2 && s.M > 0 && s.N > 0;
    return s;
}

// One member's error, reported on the caller's thread.
struct Outcome {
    int status = TLC_OK;
    std::string msg;
};

int first_failure(const std::vector<Outcome>& r, const std::vector<int>& dev) {
    for (size_t i = 0; i < r.size(); ++i)
        if (r[i].status != TLC_OK)
            return set_error(r[i].status, "device " + std::to_string(dev[i]) + ": " + r[i].msg);
    return TLC_OK;
}

Outcome outcome(int st) {
    Outcome o;
    o.status = st;
    if (st != TLC_OK) o.msg = tlc_last_error();
    return o;
}

}  // namespace
}  // namespace tlc

using namespace tlc;

struct tlc_group {
    std::vector<int> dev;
    std::vector<cudaStream_t> stream;  // one per member, on its device
    std::vector<ncclComm_t> comm;      // one per member when NCCL serves the group
    std::unique_ptr<Workers> workers;
    std::mutex call_mu;  // one call at a time per group
    int n() const { return (int)dev.size(); }
};

namespace tlc {
namespace {

// Runs fn(i) with member i's device current, on every member at once.
int on_members(tlc_group* g, int count, const std::function<int(int)>& fn) {
    std::vector<Outcome> out(g->n());
    g->workers->run([&](int i) {
        if (i >= count) return;
        const cudaError_t e = cudaSetDevice(g->dev[i]);
        out[i] = e != cudaSuccess ? Outcome{TLC_ERR_CUDA, cudaGetErrorString(e)} : outcome(fn(i));
    });
    return first_failure(out, g->dev);
}

// Synchronises every member stream from the caller's thread (device order).
int sync_members(tlc_group* g, int count) {
    for (int i = 0; i < count; ++i) {
        TLC_CUDA_TRY(cudaSetDevice(g->dev[i]));
        TLC_TRY(tlc_stream_synchronize(g->stream[i]));
    }
    return TLC_OK;
}

// Restores the caller's current device on every return path.
struct DeviceGuard {
    int dev = 0;
    DeviceGuard() { cudaGetDevice(&dev); }
    ~DeviceGuard() { cudaSetDevice(dev); }
};

// ---- host-buffer forms ---------------------------------------------------------------------

int group_matmul_host(tlc_group* g, const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out,
                      int mode) {
    int32_t nd = 0;
    int64_t sz[TLC_MAX_DIMS];
    TLC_TRY(tlc_matmul_shape(a, b, &nd, sz));
    if (!out || out->ndim != nd)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "out: wrong rank");
    for (int i = 0; i < nd; ++i)
        if (out->sizes[i] != sz[i]) return set_error(TLC_ERR_INVALID_ARGUMENT, "out: wrong shape");
    const int P = g->n();
    const BatchSplit bs = batch_split(*a, *b, sz, nd);
    if (P > 1 && bs.ok && dense(*out)) {
        const int use = (int)std::min<int64_t>(P, bs.nbatch);
        return on_members(g, use, [&](int i) {
            int64_t u0, u1;
            tlc_shard_range(bs.nbatch, use, i, &u0, &u1);
            const int64_t cnt = u1 - u0;
            tlc_tensor ai = bs.a_batched ? view3(a->data + u0 * bs.M * bs.K, cnt, bs.M, bs.K)
                                         : view2(a->data, bs.M, bs.K, bs.K, 1);
            tlc_tensor bi = bs.b_batched ? view3(b->data + u0 * bs.K * bs.N, cnt, bs.K, bs.N)
                                         : view2(b->data, bs.K, bs.N, bs.N, 1);
            tlc_tensor oi = view3(out->data + u0 * bs.M * bs.N, cnt, bs.M, bs.N);
            return tlc_matmul_host(&ai, &bi, &oi, mode, g->stream[i]);
        });
    }
    // One product, A read along rows: row blocks of A and C (multiples of 256
    // rows, the tensor-core kernel's tile rows).
    const bool rows = a->ndim == 2 && nd == 2 && a->strides[1] == 1 && dense(*out);
    const int64_t M = rows ? a->sizes[0] : 0;
    const int64_t units = (M + 255) / 256;
    if (P > 1 && rows && units >= 2) {
        const int use = (int)std::min<int64_t>(P, units);
        const int64_t N = sz[1];
        return on_members(g, use, [&](int i) {
            int64_t u0, u1;
            tlc_shard_range(units, use, i, &u0, &u1);
            const int64_t r0 = u0 * 256, r1 = std::min(M, u1 * 256);
            tlc_tensor ai = view2(a->data + r0 * a->strides[0], r1 - r0, a->sizes[1], a->strides[0], 1);
            tlc_tensor oi = view2(out->data + r0 * N, r1 - r0, N, N, 1);
            return tlc_matmul_host(&ai, b, &oi, mode, g->stream[i]);
        });
    }
    return on_members(g, 1, [&](int i) { return tlc_matmul_host(a, b, out, mode, g->stream[i]); });
}

// dB of a broadcast B over a batch split, on the devices: member i uploads
// its entries of A and dC, forms A_b^T . dC_b for each of them, and continues
// the running sum of member i-1 over them (the reference's one sequential
// sum over the batch).  The last member adds the previous gradient if
// `accumulate` and writes `db`.  dA of each member's entries is written too
// when `da` is given.
int group_backward_chain(tlc_group* g, const BatchSplit& bs, const tlc_tensor* grad,
                         const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* da, tlc_tensor* db,
                         int accumulate, int mode) {
    const int use = (int)std::min<int64_t>(g->n(), bs.nbatch);
    const int64_t K = bs.K, N = bs.N, M = bs.M;
    const size_t kn = sizeof(float) * (size_t)(K * N);
    struct Member {
        float* A = nullptr;  // [cnt, M, K]
        float* G = nullptr;  // [cnt, M, N] upstream gradient, then reused for nothing
        float* P = nullptr;  // [cnt, K, N] per-entry products
        float* B = nullptr;  // [K, N] (dA needs it)
        float* dA = nullptr;
        float* run_in = nullptr;  // [K, N] the previous member's running sum
        float* run = nullptr;     // [K, N] this member's running sum
        cudaEvent_t done = nullptr;
        int64_t u0 = 0, cnt = 0;
    };
    std::vector<Member> m(use);
    auto release = [&] {
        for (int i = 0; i < use; ++i) {
            cudaSetDevice(g->dev[i]);
            for (float* p : {m[i].A, m[i].G, m[i].P, m[i].B, m[i].dA, m[i].run_in, m[i].run})
                if (p) cudaFree(p);
            if (m[i].done) cudaEventDestroy(m[i].done);
        }
    };
    // Phase 1, all members at once: uploads, dA of the member's entries,
    // per-entry products for dB.
    int st = on_members(g, use, [&](int i) {
        Member& x = m[i];
        int64_t u1;
        tlc_shard_range(bs.nbatch, use, i, &x.u0, &u1);
        x.cnt = u1 - x.u0;
        cudaStream_t s = g->stream[i];
        const size_t a_b = sizeof(float) * (size_t)(x.cnt * M * K);
        const size_t g_b = sizeof(float) * (size_t)(x.cnt * M * N);
        TLC_CUDA_TRY(cudaMalloc(&x.A, a_b));
        TLC_CUDA_TRY(cudaMalloc(&x.G, g_b));
        TLC_CUDA_TRY(cudaMalloc(&x.P, sizeof(float) * (size_t)(x.cnt * K * N)));
        TLC_CUDA_TRY(cudaMalloc(&x.run, kn));
        if (i > 0) TLC_CUDA_TRY(cudaMalloc(&x.run_in, kn));
        TLC_CUDA_TRY(cudaEventCreateWithFlags(&x.done, cudaEventDisableTiming));
        TLC_CUDA_TRY(cudaMemcpyAsync(x.A, a->data + x.u0 * M * K, a_b, cudaMemcpyHostToDevice, s));
        TLC_CUDA_TRY(cudaMemcpyAsync(x.G, grad->data + x.u0 * M * N, g_b, cudaMemcpyHostToDevice, s));
        if (da && da->data) {
            const size_t d_b = a_b;
            TLC_CUDA_TRY(cudaMalloc(&x.B, kn));
            TLC_CUDA_TRY(cudaMalloc(&x.dA, d_b));
            TLC_CUDA_TRY(cudaMemcpyAsync(x.B, b->data, kn, cudaMemcpyHostToDevice, s));
            if (accumulate)
                TLC_CUDA_TRY(cudaMemcpyAsync(x.dA, da->data + x.u0 * M * K, d_b,
                                             cudaMemcpyHostToDevice, s));
            tlc_tensor gv = view3(x.G, x.cnt, M, N), av = view3(x.A, x.cnt, M, K);
            tlc_tensor bv = view2(x.B, K, N, N, 1), dav = view3(x.dA, x.cnt, M, K);
            TLC_TRY(tlc_matmul_backward(&gv, &av, &bv, &dav, nullptr, accumulate, mode, s));
            TLC_CUDA_TRY(cudaMemcpyAsync(da->data + x.u0 * M * K, x.dA, d_b, cudaMemcpyDeviceToHost, s));
        }
        // P_b = A_b^T . dC_b, A read transposed in place
        tlc_tensor at{};
        at.data = x.A;
        at.ndim = 3;
        at.sizes[0] = x.cnt;
        at.sizes[1] = K;
        at.sizes[2] = M;
        at.strides[0] = M * K;
        at.strides[1] = 1;
        at.strides[2] = K;
        tlc_tensor gv = view3(x.G, x.cnt, M, N), pv = view3(x.P, x.cnt, K, N);
        return tlc_matmul(&at, &gv, &pv, mode, s);
    });
    // Phase 2, the chain in member order, queued from this thread.
    for (int i = 0; st == TLC_OK && i < use; ++i) {
        Member& x = m[i];
        cudaStream_t s = g->stream[i];
        if (cudaSetDevice(g->dev[i]) != cudaSuccess) {
            st = set_error(TLC_ERR_CUDA, "cudaSetDevice failed");
            break;
        }
        if (i > 0) {
            const Member& y = m[i - 1];
            if (cudaStreamWaitEvent(s, y.done, 0) != cudaSuccess ||
                cudaMemcpyPeerAsync(x.run_in, g->dev[i], y.run, g->dev[i - 1], kn, s) != cudaSuccess) {
                st = set_error(TLC_ERR_CUDA, "running-sum copy between devices failed");
                break;
            }
        }
        if ((st = tlc_sum_dim_from(x.P, i > 0 ? x.run_in : nullptr, x.run, 1, x.cnt, K * N, s)) != TLC_OK)
            break;
        if (i + 1 == use && accumulate) {
            // accumulate_grad: db + dB, one fp32 add per element
            if (cudaMemcpyAsync(x.run_in ? x.run_in : x.P, db->data, kn, cudaMemcpyHostToDevice, s) !=
                cudaSuccess) {
                st = set_error(TLC_ERR_CUDA, "upload of the previous gradient failed");
                break;
            }
            float* prev = x.run_in ? x.run_in : x.P;
            if ((st = tlc_add(prev, x.run, x.run, K * N, s)) != TLC_OK) break;
        }
        if (i + 1 == use &&
            cudaMemcpyAsync(db->data, x.run, kn, cudaMemcpyDeviceToHost, s) != cudaSuccess) {
            st = set_error(TLC_ERR_CUDA, "download of dB failed");
            break;
        }
        if (cudaEventRecord(x.done, s) != cudaSuccess) {
            st = set_error(TLC_ERR_CUDA, "cudaEventRecord failed");
            break;
        }
    }
    const int st_sync = sync_members(g, use);
    release();
    return st != TLC_OK ? st : st_sync;
}

int group_matmul_backward_host(tlc_group* g, const tlc_tensor* grad, const tlc_tensor* a,
                               const tlc_tensor* b, tlc_tensor* da, tlc_tensor* db, int accumulate,
                               int mode) {
    int32_t nd = 0;
    int64_t sz[TLC_MAX_DIMS];
    TLC_TRY(tlc_matmul_shape(a, b, &nd, sz));
    const bool want_a = da && da->data, want_b = db && db->data;
    const int P = g->n();
    const BatchSplit bs = batch_split(*a, *b, sz, nd);
    const bool grad_ok = grad && dense(*grad) && (!want_a || dense(*da)) && (!want_b || dense(*db));
    if (P > 1 && bs.ok && grad_ok && bs.a_batched) {
        if (bs.b_batched) {
            // every entry independent: each member's shard of dA and dB
            const int use = (int)std::min<int64_t>(P, bs.nbatch);
            return on_members(g, use, [&](int i) {
                int64_t u0, u1;
                tlc_shard_range(bs.nbatch, use, i, &u0, &u1);
                const int64_t c = u1 - u0, M = bs.M, N = bs.N, K = bs.K;
                tlc_tensor gi = view3(grad->data + u0 * M * N, c, M, N);
                tlc_tensor ai = view3(a->data + u0 * M * K, c, M, K);
                tlc_tensor bi = view3(b->data + u0 * K * N, c, K, N);
                tlc_tensor dai = view3(want_a ? da->data + u0 * M * K : nullptr, c, M, K);
                tlc_tensor dbi = view3(want_b ? db->data + u0 * K * N : nullptr, c, K, N);
                return tlc_matmul_backward_host(&gi, &ai, &bi, want_a ? &dai : nullptr,
                                                want_b ? &dbi : nullptr, accumulate, mode,
                                                g->stream[i]);
            });
        }
        if (want_b) return group_backward_chain(g, bs, grad, a, b, want_a ? da : nullptr, db, accumulate, mode);
        const int use = (int)std::min<int64_t>(P, bs.nbatch);
        return on_members(g, use, [&](int i) {
            int64_t u0, u1;
            tlc_shard_range(bs.nbatch, use, i, &u0, &u1);
            const int64_t c = u1 - u0, M = bs.M, N = bs.N, K = bs.K;
            tlc_tensor gi = view3(grad->data + u0 * M * N, c, M, N);
            tlc_tensor ai = view3(a->data + u0 * M * K, c, M, K);
            tlc_tensor bi = view2(b->data, K, N, N, 1);
            tlc_tensor dai = view3(da->data + u0 * M * K, c, M, K);
            return tlc_matmul_backward_host(&gi, &ai, &bi, &dai, nullptr, accumulate, mode, g->stream[i]);
        });
    }
    // A single product: dA = dC . B^T by row blocks over the members; dB =
    // A^T . dC sums over every row, so it runs on the first member alone
    // (split rows would change the order of its additions).
    const bool rows = nd == 2 && a->ndim == 2 && grad_ok && grad->ndim == 2;
    const int64_t M = rows ? a->sizes[0] : 0;
    const int64_t units = (M + 255) / 256;
    if (P > 1 && rows && units >= 2 && want_a && a->strides[1] == 1) {
        const int use = (int)std::min<int64_t>(P, units);
        const int64_t K = a->sizes[1], N = sz[1];
        return on_members(g, use, [&](int i) {
            int64_t u0, u1;
            tlc_shard_range(units, use, i, &u0, &u1);
            const int64_t r0 = u0 * 256, r1 = std::min(M, u1 * 256);
            tlc_tensor gi = view2(grad->data + r0 * N, r1 - r0, N, N, 1);
            tlc_tensor ai = view2(a->data + r0 * a->strides[0], r1 - r0, K, a->strides[0], 1);
            tlc_tensor dai = view2(da->data + r0 * K, r1 - r0, K, K, 1);
            TLC_TRY(tlc_matmul_backward_host(&gi, &ai, b, &dai, nullptr, accumulate, mode, g->stream[i]));
            if (i == 0 && want_b)
                return tlc_matmul_backward_host(grad, a, b, nullptr, db, accumulate, mode, g->stream[i]);
            return (int)TLC_OK;
        });
    }
    return on_members(g, 1, [&](int i) {
        return tlc_matmul_backward_host(grad, a, b, da, db, accumulate, mode, g->stream[i]);
    });
}

// ---- device-memory form ------------------------------------------------------------------------

// Queues a copy of a [rows, width] block of floats with row pitches
// `dpitch` / `spitch` (elements) between two devices.
int copy_block_between(float* dst, int ddev, int64_t dpitch, const float* src, int sdev,
                       int64_t spitch, int64_t rows, int64_t width, cudaStream_t s) {
    if (!rows || !width) return TLC_OK;
    cudaMemcpy3DPeerParms p = {};
    p.dstPtr = make_cudaPitchedPtr(dst, sizeof(float) * dpitch, sizeof(float) * width, rows);
    p.dstDevice = ddev;
    p.srcPtr = make_cudaPitchedPtr(const_cast<float*>(src), sizeof(float) * spitch,
                                   sizeof(float) * width, rows);
    p.srcDevice = sdev;
    p.extent = make_cudaExtent(sizeof(float) * width, rows, 1);
    TLC_CUDA_TRY(cudaMemcpy3DPeerAsync(&p, s));
    return TLC_OK;
}

// Queues a copy of `bytes` from `src` on device `sdev` to `dst` on device
// `ddev` (the same device: a plain device-to-device copy).
int copy_between(void* dst, int ddev, const void* src, int sdev, size_t bytes, cudaStream_t s) {
    if (!bytes) return TLC_OK;
    if (ddev == sdev)
        TLC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
    else
        TLC_CUDA_TRY(cudaMemcpyPeerAsync(dst, ddev, src, sdev, bytes, s));
    return TLC_OK;
}

int group_matmul(tlc_group* g, const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out, int mode,
                 cudaStream_t caller) {
    int32_t nd = 0;
    int64_t sz[TLC_MAX_DIMS];
    TLC_TRY(tlc_matmul_shape(a, b, &nd, sz));
    if (!out || out->ndim != nd) return set_error(TLC_ERR_INVALID_ARGUMENT, "out: wrong rank");
    for (int i = 0; i < nd; ++i)
        if (out->sizes[i] != sz[i]) return set_error(TLC_ERR_INVALID_ARGUMENT, "out: wrong shape");
    int cur = 0;
    TLC_CUDA_TRY(cudaGetDevice(&cur));
    if (cur != g->dev[0])
        return set_error(TLC_ERR_INVALID_ARGUMENT,
                         "tlc_group_matmul: operands must be on the group's first device (" +
                             std::to_string(g->dev[0]) + "), the current device");
    const int P = g->n();
    const int root = g->dev[0];
    const BatchSplit bs = batch_split(*a, *b, sz, nd);
    const bool cols = !bs.ok && nd == 2 && a->ndim == 2 && b->ndim == 2 && dense(*a) && dense(*b) &&
                      dense(*out) && sz[1] >= 2 * 256;
    if (P == 1 || !((bs.ok && dense(*out)) || cols)) return tlc_matmul(a, b, out, mode, caller);

    const int64_t M = sz[nd - 2], N = sz[nd - 1], K = a->sizes[a->ndim - 1];
    const int use = (int)std::min<int64_t>(P, bs.ok ? bs.nbatch : (N + 255) / 256);
    std::vector<int64_t> lo(use), hi(use);
    for (int i = 0; i < use; ++i) {
        if (bs.ok)
            tlc_shard_range(bs.nbatch, use, i, &lo[i], &hi[i]);
        else
            tlc_shard_cols(N, use, i, 256, &lo[i], &hi[i]);
    }
    struct Member {
        float *A = nullptr, *B = nullptr, *C = nullptr;
        cudaEvent_t done = nullptr;
    };
    std::vector<Member> m(use);
    cudaEvent_t ready = nullptr;
    int st = TLC_OK;
    auto fail = [&](const char* what) { return set_error(TLC_ERR_CUDA, std::string(what) + " failed"); };
    do {
        if (cudaEventCreateWithFlags(&ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventRecord(ready, caller) != cudaSuccess) {
            st = fail("cudaEventRecord");
            break;
        }
        // Buffers and inputs of members 1.. (member 0 works in place).
        for (int i = 1; st == TLC_OK && i < use; ++i) {
            Member& x = m[i];
            const int d = g->dev[i];
            cudaStream_t s = g->stream[i];
            if (cudaSetDevice(d) != cudaSuccess || cudaStreamWaitEvent(s, ready, 0) != cudaSuccess ||
                cudaEventCreateWithFlags(&x.done, cudaEventDisableTiming) != cudaSuccess) {
                st = fail("member set-up");
                break;
            }
            const int64_t cnt = hi[i] - lo[i];
            size_t a_b, b_b, c_b;
            if (bs.ok) {
                a_b = sizeof(float) * (size_t)((bs.a_batched ? cnt : 1) * M * K);
                b_b = sizeof(float) * (size_t)((bs.b_batched ? cnt : 1) * K * N);
                c_b = sizeof(float) * (size_t)(cnt * M * N);
            } else {
                a_b = sizeof(float) * (size_t)(M * K);
                b_b = sizeof(float) * (size_t)(K * cnt);
                c_b = sizeof(float) * (size_t)(M * cnt);
            }
            if (cudaMallocAsync((void**)&x.A, std::max<size_t>(a_b, 4), s) != cudaSuccess ||
                cudaMallocAsync((void**)&x.B, std::max<size_t>(b_b, 4), s) != cudaSuccess ||
                cudaMallocAsync((void**)&x.C, std::max<size_t>(c_b, 4), s) != cudaSuccess) {
                st = set_error(TLC_ERR_OUT_OF_MEMORY, "member buffers");
                break;
            }
            if (bs.ok) {
                const float* as = a->data + (bs.a_batched ? lo[i] * M * K : 0);
                const float* bsrc = b->data + (bs.b_batched ? lo[i] * K * N : 0);
                if ((st = copy_between(x.A, d, as, root, a_b, s)) != TLC_OK) break;
                if ((st = copy_between(x.B, d, bsrc, root, b_b, s)) != TLC_OK) break;
            } else {
                // B's column block [K, cnt] out of the row-major [K, N]
                if ((st = copy_block_between(x.B, d, cnt, b->data + lo[i], root, N, K, cnt, s)) !=
                    TLC_OK)
                    break;
            }
        }
        if (st != TLC_OK) break;
        // Column blocks: A to every member, one NCCL broadcast from the root.
        if (!bs.ok) {
            const Nccl& nc = nccl();
            // every rank of the communicator must take part in a collective:
            // NCCL only when every member has a block
            if (!g->comm.empty() && nc.ok && use == P) {
                nc.group_start();
                ncclResult_t r = ncclSuccess;
                for (int i = 0; i < P; ++i) {
                    void* recv = i == 0 ? a->data : (void*)m[i].A;
                    cudaStream_t s = i == 0 ? caller : g->stream[i];
                    const ncclResult_t ri =
                        nc.broadcast(a->data, recv, (size_t)(M * K), ncclFloat32, 0, g->comm[i], s);
                    if (ri != ncclSuccess && r == ncclSuccess) r = ri;
                }
                const ncclResult_t r2 = nc.group_end();
                if (r != ncclSuccess || r2 != ncclSuccess) {
                    st = set_error(TLC_ERR_CUDA, std::string("ncclBroadcast: ") +
                                                     nc.error_string(r != ncclSuccess ? r : r2));
                    break;
                }
            } else {
                for (int i = 1; st == TLC_OK && i < use; ++i) {
                    cudaSetDevice(g->dev[i]);
                    st = copy_between(m[i].A, g->dev[i], a->data, root,
                                      sizeof(float) * (size_t)(M * K), g->stream[i]);
                }
                if (st != TLC_OK) break;
            }
        }
        // The products, then the results back into the caller's C.
        for (int i = 0; st == TLC_OK && i < use; ++i) {
            const int d = g->dev[i];
            cudaStream_t s = i == 0 ? caller : g->stream[i];
            cudaSetDevice(d);
            const int64_t cnt = hi[i] - lo[i];
            tlc_gemm_desc gd{};
            gd.M = M;
            gd.N = bs.ok ? N : cnt;
            gd.K = K;
            gd.a_rs = K;
            gd.a_cs = 1;
            gd.b_cs = 1;
            if (bs.ok) {
                gd.A = i == 0 ? a->data : m[i].A;
                gd.B = i == 0 ? b->data : m[i].B;
                gd.C = i == 0 ? out->data : m[i].C;
                gd.b_rs = N;
                gd.c_rs = N;
                gd.batch_ndim = 1;
                gd.batch_sizes[0] = cnt;
                gd.a_bstride[0] = bs.a_batched ? M * K : 0;
                gd.b_bstride[0] = bs.b_batched ? K * N : 0;
                gd.c_bstride[0] = M * N;
                if (i == 0) {
                    // member 0's entries in place
                    gd.A = a->data + (bs.a_batched ? lo[0] * M * K : 0);
                    gd.B = b->data + (bs.b_batched ? lo[0] * K * N : 0);
                    gd.C = out->data + lo[0] * M * N;
                }
            } else {
                gd.A = i == 0 ? a->data : m[i].A;
                gd.B = i == 0 ? b->data + lo[0] : m[i].B;  // member 0 reads its block in place
                gd.b_rs = i == 0 ? N : cnt;
                gd.C = i == 0 ? out->data + lo[0] : m[i].C;
                gd.c_rs = i == 0 ? N : cnt;
            }
            if ((st = tlc_gemm(&gd, mode, s)) != TLC_OK) break;
            if (i == 0) continue;
            if (bs.ok) {
                st = copy_between(out->data + lo[i] * M * N, root, m[i].C, d,
                                  sizeof(float) * (size_t)(cnt * M * N), s);
            } else {
                st = copy_block_between(out->data + lo[i], root, N, m[i].C, d, cnt, M, cnt, s);
            }
            if (st != TLC_OK) break;
            cudaFreeAsync(m[i].A, s);
            cudaFreeAsync(m[i].B, s);
            cudaFreeAsync(m[i].C, s);
            m[i].A = m[i].B = m[i].C = nullptr;
            if (cudaEventRecord(m[i].done, s) != cudaSuccess) st = fail("cudaEventRecord");
        }
    } while (false);
    // The caller's stream waits for every member (also after a failure, so
    // nothing in flight outlives the call's buffers).
    cudaSetDevice(root);
    for (int i = 1; i < use; ++i) {
        if (!m[i].done) continue;
        if (st != TLC_OK) {
            cudaSetDevice(g->dev[i]);
            cudaEventRecord(m[i].done, g->stream[i]);
            for (float* p : {m[i].A, m[i].B, m[i].C})
                if (p) cudaFreeAsync(p, g->stream[i]);
            cudaSetDevice(root);
        }
        cudaStreamWaitEvent(caller, m[i].done, 0);
    }
    for (int i = 1; i < use; ++i)
        if (m[i].done) cudaEventDestroy(m[i].done);
    if (ready) cudaEventDestroy(ready);
    return st;
}

}  // namespace
}  // namespace tlc

extern "C" {

int tlc_group_create(const int* devices, int n, tlc_group** out) {
    clear_error();
    if (!out) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_group_create: out is NULL");
    *out = nullptr;
    if (!devices || n < 1 || n > 64)
        return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_group_create: 1 to 64 devices");
    int count = 0;
    TLC_CUDA_TRY(cudaGetDeviceCount(&count));
    for (int i = 0; i < n; ++i)
        if (devices[i] < 0 || devices[i] >= count)
            return set_error(TLC_ERR_INVALID_ARGUMENT,
                             "tlc_group_create: no device " + std::to_string(devices[i]));
    DeviceGuard keep;
    auto g = std::make_unique<tlc_group>();
    g->dev.assign(devices, devices + n);
    g->stream.assign(n, nullptr);
    for (int i = 0; i < n; ++i) {
        TLC_CUDA_TRY(cudaSetDevice(devices[i]));
        TLC_CUDA_TRY(cudaStreamCreateWithFlags(&g->stream[i], cudaStreamNonBlocking));
    }
    // Direct NVLink paths between the members (copies between devices then
    // need no staging through host memory).
    bool distinct = true;
    for (int i = 0; i < n; ++i)
        for (int j = i + 1; j < n; ++j)
            if (devices[i] == devices[j]) distinct = false;
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j) {
            if (devices[i] == devices[j]) continue;
            int can = 0;
            cudaDeviceCanAccessPeer(&can, devices[i], devices[j]);
            if (!can) continue;
            cudaSetDevice(devices[i]);
            cudaDeviceEnablePeerAccess(devices[j], 0);
            cudaGetLastError();  // "already enabled" is fine
        }
    const Nccl& nc = nccl();
    if (n > 1 && distinct && nc.ok) {
        std::vector<ncclComm_t> comm(n, nullptr);
        if (nc.init_all(comm.data(), n, devices) == ncclSuccess) g->comm = comm;
    }
    g->workers = std::make_unique<Workers>(n);
    *out = g.release();
    return TLC_OK;
}

int tlc_group_destroy(tlc_group* g) {
    clear_error();
    if (!g) return TLC_OK;
    DeviceGuard keep;
    for (int i = 0; i < g->n(); ++i) {
        cudaSetDevice(g->dev[i]);
        cudaStreamSynchronize(g->stream[i]);
    }
    if (!g->comm.empty())
        for (ncclComm_t c : g->comm) nccl().destroy(c);
    for (int i = 0; i < g->n(); ++i) {
        cudaSetDevice(g->dev[i]);
        cudaStreamDestroy(g->stream[i]);
    }
    delete g;
    return TLC_OK;
}

int tlc_group_size(const tlc_group* g, int* n, int* uses_nccl) {
    clear_error();
    if (!g || !n) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_group_size: NULL argument");
    *n = g->n();
    if (uses_nccl) *uses_nccl = g->comm.empty() ? 0 : 1;
    return TLC_OK;
}

int tlc_group_matmul_host(tlc_group* g, const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out,
                          int mode) {
    clear_error();
    if (!g) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_group_matmul_host: group is NULL");
    std::lock_guard<std::mutex> lk(g->call_mu);
    DeviceGuard keep;
    return group_matmul_host(g, a, b, out, mode);
}

int tlc_group_matmul_backward_host(tlc_group* g, const tlc_tensor* grad, const tlc_tensor* a,
                                   const tlc_tensor* b, tlc_tensor* da, tlc_tensor* db,
                                   int accumulate, int mode) {
    clear_error();
    if (!g) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_group_matmul_backward_host: group is NULL");
    std::lock_guard<std::mutex> lk(g->call_mu);
    DeviceGuard keep;
    return group_matmul_backward_host(g, grad, a, b, da, db, accumulate, mode);
}

int tlc_group_matmul(tlc_group* g, const tlc_tensor* a, const tlc_tensor* b, tlc_tensor* out,
                     int mode, void* stream) {
    clear_error();
    if (!g) return set_error(TLC_ERR_INVALID_ARGUMENT, "tlc_group_matmul: group is NULL");
    std::lock_guard<std::mutex> lk(g->call_mu);
    DeviceGuard keep;
    return group_matmul(g, a, b, out, mode, (cudaStream_t)stream);
}

}  // extern "C"
