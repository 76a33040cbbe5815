// Tests of the GPU tl:: layer, written like the reference's own tests
// (tests/test_ops.cpp:21-114, tests/test_autograd.cpp:150-261 of
// torchlite-cpp): same inputs, same asserted values, plus bit-exact checks
// against a scalar fma chain (the reference's gemm_blocked order) and the
// transposed-operand (Linear X.W^T) forward and backward.
//
//   tl_tests            all tests (needs a GPU)
//   tl_tests --cpu      only the shape / exception tests (no GPU needed)
#include <tl/autograd.h>
#include <tl/model_io.h>
#include <tl/ops.h>
#include <tl/tensor.h>
#include <tlc.h>

#include <cmath>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::cerr << "FAIL: " #cond " at " __FILE__ ":" << __LINE__ << "\n"; \
            std::exit(1);                                                        \
        }                                                                        \
    } while (0)

static bool is_close(float a, float b, float e = 1e-5f) { return std::fabs(a - b) < e; }
static bool same_bits(float a, float b) { return std::memcmp(&a, &b, sizeof(float)) == 0; }

template <typename F>
static void expect_invalid(F f, const char* msg) {
    try {
        f();
    } catch (const std::invalid_argument& e) {
        CHECK(std::string(e.what()) == msg);
        return;
    }
    CHECK(!"expected std::invalid_argument");
}

static void test_errors() {
    tl::Tensor a({3, 4}), b({5, 6});
    expect_invalid([&] { tl::matmul(a, b); }, "Incompatible dimensions for matmul");
    tl::Tensor c({2, 3, 4}), d({3, 4, 5});
    expect_invalid([&] { tl::matmul(c, d); }, "Incompatible dimensions for broadcasting");
    tl::Tensor v({5}), w({4});
    expect_invalid([&] { tl::matmul(v, w); }, "Incompatible dimensions for matmul");
    tl::Tensor s(std::vector<int64_t>{});  // 0-D
    expect_invalid([&] { tl::matmul(s, a); }, "matmul: requires at least 1D tensors");
    std::cout << "errors ok\n";
}

static void test_forward_kats() {
    // tests/test_ops.cpp:21-32
    tl::Tensor A({2, 3});
    tl::Tensor B({3, 2});
    for (int i = 0; i < A.numel(); ++i) A.data()[i] = i + 1.0f;
    for (int i = 0; i < B.numel(); ++i) B.data()[i] = i + 7.0f;
    tl::Tensor C = tl::matmul(A, B);
    CHECK(C.data()[0] == 58.0f);
    CHECK(C.data()[3] == 154.0f);

    // tests/test_ops.cpp:56-76: (2,3,2,2) @ (2,4) -> (2,3,2,4)
    tl::Tensor input({2, 3, 2, 2});
    for (int i = 0; i < input.numel(); ++i) input.data()[i] = 1.0f;
    tl::Tensor weights({2, 4});
    for (int i = 0; i < weights.numel(); ++i) weights.data()[i] = 0.5f;
    tl::Tensor out = tl::matmul(input, weights);
    CHECK(out.sizes().size() == 4 && out.sizes()[0] == 2 && out.sizes()[1] == 3 &&
          out.sizes()[2] == 2 && out.sizes()[3] == 4);
    for (int i = 0; i < out.numel(); ++i) CHECK(is_close(out.data()[i], 1.0f));

    // tests/test_ops.cpp:78-89: ones (256,512) @ (512,256) -> 512
    tl::Tensor ha({256, 512}), hb({512, 256});
    for (int64_t i = 0; i < ha.numel(); ++i) ha.data()[i] = 1.0f;
    for (int64_t i = 0; i < hb.numel(); ++i) hb.data()[i] = 1.0f;
    tl::Tensor ho = tl::matmul(ha, hb);
    for (int64_t i = 0; i < ho.numel(); ++i) CHECK(ho.data()[i] == 512.0f);

    // tests/test_ops.cpp:91-114: ragged integer-valued (259,300) @ (300,277);
    // every element equal to the ascending-k fma chain (exact mode: same bits)
    const int64_t LM = 259, LK = 300, LN = 277;
    tl::Tensor la({LM, LK}), lb({LK, LN});
    for (int64_t i = 0; i < la.numel(); ++i) la.data()[i] = (float)((i * 3 + 1) % 11 - 5);
    for (int64_t i = 0; i < lb.numel(); ++i) lb.data()[i] = (float)((i * 7 + 2) % 13 - 6);
    tl::Tensor lo = tl::matmul(la, lb);
    CHECK(lo.sizes()[0] == LM && lo.sizes()[1] == LN);
    const float* pa = la.data();
    const float* pb = lb.data();
    const float* po = lo.data();
    for (int64_t i = 0; i < LM; ++i)
        for (int64_t j = 0; j < LN; ++j) {
            float ref = 0.0f;
            for (int64_t k = 0; k < LK; ++k) ref = std::fmaf(pa[i * LK + k], pb[k * LN + j], ref);
            CHECK(same_bits(po[i * LN + j], ref));
        }
    std::cout << "forward kats ok\n";
}

static void test_transposed_bit_exact() {
    uint32_t s = 12345;
    auto rnd = [&] {
        s = s * 1664525u + 1013904223u;
        return ((s >> 8) & 0xFFFF) / 32768.0f - 1.0f;
    };
    const int64_t M = 67, K = 131, N = 45;
    tl::Tensor X({M, K}), W({N, K});  // Linear: Y = X . W^T, W stored [out, in]
    for (int64_t i = 0; i < X.numel(); ++i) X.data()[i] = rnd();
    for (int64_t i = 0; i < W.numel(); ++i) W.data()[i] = rnd();
    tl::Tensor Y = tl::matmul(X, tl::transpose(W, 0, 1));
    const float* x = X.data();
    const float* w = W.data();
    const float* y = Y.data();
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) {
            float ref = 0.0f;
            for (int64_t k = 0; k < K; ++k) ref = std::fmaf(x[i * K + k], w[j * K + k], ref);
            CHECK(same_bits(y[i * N + j], ref));
        }
    std::cout << "transposed operand bit-exact ok\n";
}

static void test_backward_levels() {
    auto close = [](float a, float b) { return std::fabs(a - b) < 1e-4f; };
    {  // Level 1 (tests/test_autograd.cpp:150-195)
        tl::Tensor A({2, 3}), B({3, 2});
        for (int i = 0; i < 6; ++i) {
            A.data()[i] = i + 1.0f;
            B.data()[i] = i + 1.0f;
        }
        A.set_requires_grad(true);
        B.set_requires_grad(true);
        tl::Tensor C = tl::matmul(A, B);
        C.backward();
        CHECK(!A.grad().empty() && !B.grad().empty());
        const float da[6] = {3, 7, 11, 3, 7, 11}, db[6] = {5, 5, 7, 7, 9, 9};
        for (int i = 0; i < 6; ++i) {
            CHECK(close(A.grad().data()[i], da[i]));
            CHECK(close(B.grad().data()[i], db[i]));
        }
    }
    {  // Level 2 (batched)
        tl::Tensor A({2, 2, 3}), B({2, 3, 2});
        for (int i = 0; i < 12; ++i) {
            A.data()[i] = 1.0f;
            B.data()[i] = 1.0f;
        }
        A.set_requires_grad(true);
        B.set_requires_grad(true);
        tl::Tensor C = tl::matmul(A, B);
        C.backward();
        for (int i = 0; i < 12; ++i) CHECK(close(A.grad().data()[i], 2.0f));
        for (int i = 0; i < 12; ++i) CHECK(close(B.grad().data()[i], 2.0f));
    }
    {  // Level 3 (broadcast batch)
        tl::Tensor A({2, 3, 4}), B({4, 2});
        for (int i = 0; i < 24; ++i) A.data()[i] = 1.0f;
        for (int i = 0; i < 8; ++i) B.data()[i] = 1.0f;
        A.set_requires_grad(true);
        B.set_requires_grad(true);
        tl::Tensor C = tl::matmul(A, B);
        C.backward();
        for (int i = 0; i < 24; ++i) CHECK(close(A.grad().data()[i], 2.0f));
        for (int i = 0; i < 8; ++i) CHECK(close(B.grad().data()[i], 6.0f));
    }
    {  // Level 4a ((K,) @ (K, N))
        tl::Tensor a({4}), B({4, 3});
        for (int i = 0; i < 4; ++i) a.data()[i] = 1.0f;
        for (int i = 0; i < 12; ++i) B.data()[i] = 1.0f;
        a.set_requires_grad(true);
        B.set_requires_grad(true);
        tl::Tensor c = tl::matmul(a, B);
        CHECK(c.sizes().size() == 1 && c.sizes()[0] == 3);
        c.backward();
        for (int i = 0; i < 4; ++i) CHECK(close(a.grad().data()[i], 3.0f));
        for (int i = 0; i < 12; ++i) CHECK(close(B.grad().data()[i], 1.0f));
    }
    {  // Level 4b ((M, K) @ (K,))
        tl::Tensor A({3, 4}), b({4});
        for (int i = 0; i < 12; ++i) A.data()[i] = 1.0f;
        for (int i = 0; i < 4; ++i) b.data()[i] = 1.0f;
        A.set_requires_grad(true);
        b.set_requires_grad(true);
        tl::Tensor c = tl::matmul(A, b);
        c.backward();
        for (int i = 0; i < 12; ++i) CHECK(close(A.grad().data()[i], 1.0f));
        for (int i = 0; i < 4; ++i) CHECK(close(b.grad().data()[i], 3.0f));
    }
    std::cout << "backward levels ok\n";
}

static void test_linear_backward_transposed() {
    // Y = X . W^T with W [out, in]; dW flows back through TransposeBackward.
    const int64_t M = 33, K = 20, N = 17;
    tl::Tensor X({M, K}), W({N, K});
    for (int64_t i = 0; i < X.numel(); ++i) X.data()[i] = (float)((i * 5 + 3) % 9 - 4);
    for (int64_t i = 0; i < W.numel(); ++i) W.data()[i] = (float)((i * 3 + 1) % 7 - 3);
    X.set_requires_grad(true);
    W.set_requires_grad(true);
    tl::Tensor Y = tl::matmul(X, tl::transpose(W, 0, 1));
    tl::Tensor dY({M, N});
    for (int64_t i = 0; i < dY.numel(); ++i) dY.data()[i] = (float)((i * 7 + 2) % 5 - 2);
    Y.grad() = dY;
    Y.backward();
    const float* x = X.data();
    const float* w = W.data();
    const float* dy = dY.data();
    const float* dx = X.grad().data();
    const float* dw = W.grad().data();
    CHECK(W.grad().sizes()[0] == N && W.grad().sizes()[1] == K);
    for (int64_t i = 0; i < M; ++i)
        for (int64_t k = 0; k < K; ++k) {  // dX = dY . W
            float ref = 0.0f;
            for (int64_t n = 0; n < N; ++n) ref = std::fmaf(dy[i * N + n], w[n * K + k], ref);
            CHECK(same_bits(dx[i * K + k], ref));
        }
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {  // dW = (X^T . dY)^T
            float ref = 0.0f;
            for (int64_t i = 0; i < M; ++i) ref = std::fmaf(x[i * K + k], dy[i * N + n], ref);
            CHECK(same_bits(dw[n * K + k], ref));
        }
    std::cout << "linear backward (transposed weight) ok\n";
}

static void test_tensor_core_modes() {
    const int64_t M = 300, K = 500, N = 280;
    tl::Tensor A({M, K}), B({K, N});
    uint32_t s = 7;
    auto rnd = [&] {
        s = s * 1664525u + 1013904223u;
        return ((s >> 8) & 0xFFFF) / 32768.0f - 1.0f;
    };
    for (int64_t i = 0; i < A.numel(); ++i) A.data()[i] = rnd();
    for (int64_t i = 0; i < B.numel(); ++i) B.data()[i] = rnd();
    tl::Tensor ref = tl::matmul(A, B, TLC_MODE_EXACT);
    const float* r = ref.data();
    for (int mode : {(int)TLC_MODE_TF32, (int)TLC_MODE_3XTF32}) {
        tl::Tensor C = tl::matmul(A, B, mode);
        const float* c = C.data();
        double num = 0, den = 0;
        for (int64_t i = 0; i < C.numel(); ++i) {
            num += (double)(c[i] - r[i]) * (c[i] - r[i]);
            den += (double)r[i] * r[i];
        }
        CHECK(std::sqrt(num / den) <= (mode == TLC_MODE_TF32 ? 1e-2 : 1e-5));
    }
    std::cout << "tf32 / 3xtf32 tolerance ok\n";
}

// tests/test_model_io.cpp of the reference: save, load into fresh tensors of
// the same shapes (values identical), a shape mismatch throws runtime_error;
// here the data moves straight between the file and device storage.
static void test_model_io() {
    tl::Tensor W({4, 8}), b({8}), s(std::vector<int64_t>{});
    for (int64_t i = 0; i < W.numel(); ++i) W.data()[i] = 0.25f * i - 3.0f;
    for (int64_t i = 0; i < b.numel(); ++i) b.data()[i] = -0.5f * i;
    s.data()[0] = 7.0f;
    tl::Tensor Wd = tl::matmul(W, tl::ones({8, 8}));  // a device-only tensor (product)
    const std::string path = "tl_test_model_io.tl";
    tl::save_model(path, {&W, &b, &s, &Wd});
    tl::Tensor W2({4, 8}), b2({8}), s2(std::vector<int64_t>{}), Wd2({4, 8});
    tl::load_model(path, {&W2, &b2, &s2, &Wd2});
    for (int64_t i = 0; i < W.numel(); ++i) CHECK(same_bits(W.data()[i], W2.data()[i]));
    for (int64_t i = 0; i < b.numel(); ++i) CHECK(same_bits(b.data()[i], b2.data()[i]));
    CHECK(s2.data()[0] == 7.0f);
    for (int64_t i = 0; i < Wd.numel(); ++i) CHECK(same_bits(Wd.data()[i], Wd2.data()[i]));
    tl::Tensor wrong({4, 16});
    bool threw = false;
    try {
        tl::load_model(path, {&wrong, &b2, &s2, &Wd2});
    } catch (const std::runtime_error& e) {
        threw = std::string(e.what()) == "load_model: shape mismatch";
    }
    CHECK(threw);
    std::remove(path.c_str());
    std::cout << "model_io ok\n";
}

// tests/test_ops.cpp:651-704 of the reference: flash attention against the
// materialised path (scaled matmul, softmax, matmul), forward and the
// gradients of backward() seeded with ones, S = 80 crossing the 64-row tile.
static void test_flash_attention() {
    const int64_t S = 80, d = 16;
    uint32_t st = 12345u;
    auto fill = [&](tl::Tensor& t) {
        for (int64_t i = 0; i < t.numel(); ++i) {
            st = st * 1664525u + 1013904223u;
            t.data()[i] = ((st >> 8) & 0xFFFF) / 16384.0f - 2.0f;
        }
    };
    tl::Tensor Q({S, d}), K({S, d}), V({S, d});
    fill(Q);
    fill(K);
    fill(V);
    const float sm_scale = 1.0f / std::sqrt((float)d);
    {
        tl::Tensor scores = tl::scale(tl::matmul(Q, tl::transpose(K, 0, 1)), sm_scale);
        tl::Tensor ref = tl::matmul(tl::softmax(scores), V);
        tl::Tensor flash = tl::flash_attention(Q, K, V, sm_scale);
        CHECK(flash.sizes()[0] == S && flash.sizes()[1] == d);
        for (int64_t i = 0; i < S * d; ++i) CHECK(is_close(flash.data()[i], ref.data()[i], 1e-4f));
    }
    Q.set_requires_grad(true);
    K.set_requires_grad(true);
    V.set_requires_grad(true);
    tl::Tensor ref = tl::matmul(tl::softmax(tl::scale(tl::matmul(Q, tl::transpose(K, 0, 1)), sm_scale)), V);
    ref.backward();
    std::vector<float> dq(Q.grad().data(), Q.grad().data() + S * d),
        dk(K.grad().data(), K.grad().data() + S * d), dv(V.grad().data(), V.grad().data() + S * d);
    Q.grad() = tl::Tensor();
    K.grad() = tl::Tensor();
    V.grad() = tl::Tensor();
    tl::Tensor flash = tl::flash_attention(Q, K, V, sm_scale);
    flash.backward();
    for (int64_t i = 0; i < S * d; ++i) {
        CHECK(is_close(Q.grad().data()[i], dq[i], 1e-4f));
        CHECK(is_close(K.grad().data()[i], dk[i], 1e-4f));
        CHECK(is_close(V.grad().data()[i], dv[i], 1e-4f));
    }
    std::cout << "flash_attention ok\n";
}

// With TL_NUM_GPUS > 1 (and that many GPUs): a batched product with a broadcast
// weight and its MatmulBackward through the device group, from host operands
// (the host-buffer split) and from device-resident ones (split from device 0),
// bit-identical to the single-GPU entry points in exact mode.
static void test_multi_gpu_group() {
    if (!tl::multi_gpu_group()) {
        std::cout << "multi-GPU group skipped (TL_NUM_GPUS unset or one GPU)\n";
        return;
    }
    const int64_t Bn = 6, M = 512, K = 96, N = 384;  // 1.2 M outputs: above the group threshold
    uint32_t s = 99;
    auto fill = [&](tl::Tensor& t) {
        for (int64_t i = 0; i < t.numel(); ++i) {
            s = s * 1664525u + 1013904223u;
            t.data()[i] = ((s >> 8) & 0xFFFF) / 32768.0f - 1.0f;
        }
    };
    tl::Tensor A({Bn, M, K}), W({K, N}), G({Bn, M, N});
    fill(A);
    fill(W);
    fill(G);
    // single-GPU results through the C ABI
    auto hv = [](const tl::Tensor& t) {
        tlc_tensor v{};
        v.ndim = (int32_t)t.sizes().size();
        for (int i = 0; i < v.ndim; ++i) {
            v.sizes[i] = t.sizes()[i];
            v.strides[i] = t.strides()[i];
        }
        v.data = const_cast<float*>(t.data());
        return v;
    };
    std::vector<float> refC(Bn * M * N), refdA(Bn * M * K), refdW(K * N);
    {
        tlc_tensor a = hv(A), w = hv(W), g = hv(G), c = hv(G), da = hv(A), dw = hv(W);
        c.data = refC.data();
        da.data = refdA.data();
        dw.data = refdW.data();
        CHECK(tlc_matmul_host(&a, &w, &c, TLC_MODE_EXACT, nullptr) == TLC_OK);
        CHECK(tlc_matmul_backward_host(&g, &a, &w, &da, &dw, 0, TLC_MODE_EXACT, nullptr) == TLC_OK);
    }
    for (int pass = 0; pass < 2; ++pass) {
        tl::Tensor a = A.clone(), w = W.clone(), g = G.clone();
        if (pass == 0) {  // host-only copies: the host-buffer split
            a = tl::Tensor({Bn, M, K});
            w = tl::Tensor({K, N});
            g = tl::Tensor({Bn, M, N});
            std::memcpy(a.data(), A.data(), sizeof(float) * A.numel());
            std::memcpy(w.data(), W.data(), sizeof(float) * W.numel());
            std::memcpy(g.data(), G.data(), sizeof(float) * G.numel());
            CHECK(a.host_only() && w.host_only());
        } else {
            CHECK(!a.host_only() && !w.host_only());
        }
        a.set_requires_grad(true);
        w.set_requires_grad(true);
        tl::Tensor c = tl::matmul(a, w, TLC_MODE_EXACT);
        for (int64_t i = 0; i < c.numel(); ++i) CHECK(same_bits(c.data()[i], refC[i]));
        if (pass == 0) {
            c.grad() = g;
            c.backward();
            for (int64_t i = 0; i < a.numel(); ++i) CHECK(same_bits(a.grad().data()[i], refdA[i]));
            for (int64_t i = 0; i < w.numel(); ++i) CHECK(same_bits(w.grad().data()[i], refdW[i]));
        }
    }
    std::cout << "multi-GPU group ok\n";
}

int main(int argc, char** argv) {
    const bool cpu_only = argc > 1 && std::string(argv[1]) == "--cpu";
    test_errors();
    if (cpu_only) return 0;
    test_forward_kats();
    test_transposed_bit_exact();
    test_backward_levels();
    test_linear_backward_transposed();
    test_tensor_core_modes();
    test_model_io();
    test_flash_attention();
    test_multi_gpu_group();
    std::cout << "all tl:: tests passed\n";
    return 0;
}
