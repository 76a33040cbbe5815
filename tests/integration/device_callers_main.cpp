// The scenarios of ref_callers_main.cpp (Linear forward + backward on 2-D and
// batched inputs, MultiHeadAttention forward + backward, a broadcast batched
// matmul, X . W^T), written against the device-resident C++ tl:: layer
// (torchlite-cpp_b200/host) instead of the reference library (and a grouped,
// strided Conv2d through tl::conv2d): the same seeded
// inputs in the same order, the same ops in the reference's order
// (src/nn.cpp:77-83 Linear::forward, :401-445 MultiHeadAttention::forward),
// with Linear's bias add and the attention scale fused into their GEMMs.
// Every output and gradient goes to argv[1] as raw float32, in the order of
// ref_callers_main.cpp; tests/test_reference_callers.py compares the two.
#include <tl/autograd.h>
#include <tl/ops.h>
#include <tl/tensor.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <vector>

static uint32_t g_state = 20240601u;
static float next_value() {
    g_state = g_state * 1664525u + 1013904223u;
    return ((g_state >> 8) & 0xFFFF) / 32768.0f - 1.0f;
}

static tl::Tensor filled(const std::vector<int64_t>& sizes, float scale = 1.0f) {
    tl::Tensor t(sizes);
    float* p = t.data();
    for (int64_t i = 0; i < t.numel(); ++i) p[i] = next_value() * scale;
    return t;
}

static std::vector<float> g_out;
static void dump(const tl::Tensor& t) {
    tl::Tensor c = t.contiguous();
    const float* p = c.data();
    g_out.insert(g_out.end(), p, p + c.numel());
}

// nn::Linear: weight [in, out], out = x . W + b
struct Linear {
    tl::Tensor W, b;
    Linear(int64_t in, int64_t out) {
        W = filled({in, out}, 0.05f);
        b = filled({out}, 0.1f);
        W.set_requires_grad(true);
        b.set_requires_grad(true);
    }
    tl::Tensor forward(const tl::Tensor& x) const { return tl::matmul_add(x, W, b); }
};

struct MultiHeadAttention {
    int64_t d_model, heads, head_dim;
    Linear q, k, v, o;
    MultiHeadAttention(int64_t dm, int64_t h)
        : d_model(dm), heads(h), head_dim(dm / h), q(dm, dm), k(dm, dm), v(dm, dm), o(dm, dm) {}
    tl::Tensor forward(const tl::Tensor& input) const {
        const int64_t batch = input.sizes()[0], seq = input.sizes()[1];
        tl::Tensor Q = q.forward(input), K = k.forward(input), V = v.forward(input);
        Q = tl::transpose(tl::reshape(Q, {batch, seq, heads, head_dim}), 1, 2);
        K = tl::transpose(tl::reshape(K, {batch, seq, heads, head_dim}), 1, 2);
        V = tl::transpose(tl::reshape(V, {batch, seq, heads, head_dim}), 1, 2);
        tl::Tensor scores = tl::matmul_scale(Q, tl::transpose(K, -2, -1),
                                             1.0f / std::sqrt(static_cast<float>(head_dim)));
        tl::Tensor attn = tl::softmax(scores);
        tl::Tensor out = tl::matmul(attn, V);
        out = tl::reshape(tl::transpose(out, 1, 2), {batch, seq, d_model});
        return o.forward(out);
    }
};

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s out.bin\n", argv[0]);
        return 2;
    }
    {
        Linear lin(300, 257);
        tl::Tensor x = filled({129, 300});
        x.set_requires_grad(true);
        tl::Tensor y = lin.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(lin.W.grad());
        dump(lin.b.grad());
    }
    {
        Linear lin(70, 50);
        tl::Tensor x = filled({4, 33, 70});
        x.set_requires_grad(true);
        tl::Tensor y = lin.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(lin.W.grad());
    }
    {
        MultiHeadAttention mha(96, 4);
        tl::Tensor x = filled({2, 40, 96});
        x.set_requires_grad(true);
        tl::Tensor y = mha.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(mha.q.W.grad());
        dump(mha.v.W.grad());
    }
    {
        tl::Tensor a = filled({3, 20, 30});
        tl::Tensor b = filled({30, 25});
        a.set_requires_grad(true);
        b.set_requires_grad(true);
        tl::Tensor c = tl::matmul(a, b);
        c.grad() = filled(c.sizes());
        c.backward();
        dump(c);
        dump(a.grad());
        dump(b.grad());
    }
    {
        tl::Tensor x = filled({65, 48});
        tl::Tensor w = filled({31, 48});
        x.set_requires_grad(true);
        w.set_requires_grad(true);
        tl::Tensor y = tl::matmul(x, tl::transpose(w, 0, 1));
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(w.grad());
    }
    {
        tl::Tensor w = filled({6, 2, 3, 3}, 0.2f);
        tl::Tensor b = filled({6}, 0.1f);
        w.set_requires_grad(true);
        b.set_requires_grad(true);
        tl::Tensor x = filled({2, 4, 9, 11});
        x.set_requires_grad(true);
        tl::Tensor y = tl::conv2d(x, w, b, 2, 1, 2);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(w.grad());
        dump(b.grad());
    }
    std::FILE* f = std::fopen(argv[1], "wb");
    if (!f) return 3;
    std::fwrite(g_out.data(), sizeof(float), g_out.size(), f);
    std::fclose(f);
    std::printf("floats %zu\n", g_out.size());
    return 0;
}
