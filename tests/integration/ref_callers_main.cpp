// The reference library's own callers of tl::matmul, unchanged, driven on
// seeded inputs: nn::Linear forward + backward (2-D and batched input),
// MultiHeadAttention forward + backward, a broadcast batched matmul and a
// transposed-weight product with their MatmulBackward.  Every output and
// gradient is written to argv[1] as raw float32.
//
// With a second argument "encoder" it runs instead one full-size
// transformer-encoder MultiHeadAttention (batch 16, seq 512, d_model 768,
// 12 heads of 64: src/nn.cpp:401-445) forward + backward, x ~ N(0,1) and
// weights ~ N(0, 0.02) (Box-Muller over the same LCG), and writes the output,
// the input gradient and the query / value projection weight gradients.
//
// Linked (oracle/Makefile, target `callers`) twice from the reference's
// objects: ref_callers_{v3,v4} with tl::matmul redirected to libtl_cuda
// (torchlite-cpp_b200/integration/reference_matmul_gpu.cpp), and
// ref_callers_cpu_{v3,v4} with the reference's own CPU matmul.
// tests/test_reference_callers.py runs both and compares the two files, bit
// for bit in exact mode.
#include <tl/autograd.h>
#include <tl/nn.h>
#include <tl/ops.h>
#include <tl/tensor.h>

#include <tlc.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
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

// N(0, std^2) by the Box-Muller transform of two LCG draws mapped to (0, 1].
static tl::Tensor normal(const std::vector<int64_t>& sizes, float std_dev) {
    tl::Tensor t(sizes);
    float* p = t.data();
    for (int64_t i = 0; i < t.numel(); i += 2) {
        g_state = g_state * 1664525u + 1013904223u;
        const double u1 = ((g_state >> 8) + 1.0) / 16777216.0;
        g_state = g_state * 1664525u + 1013904223u;
        const double u2 = (g_state >> 8) / 16777216.0;
        const double r = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586 * u2;
        p[i] = static_cast<float>(r * std::cos(th) * std_dev);
        if (i + 1 < t.numel()) p[i + 1] = static_cast<float>(r * std::sin(th) * std_dev);
    }
    return t;
}

static std::vector<float> g_out;
static void dump(const tl::Tensor& t) {
    tl::Tensor c = t.contiguous();
    const float* p = c.data();
    g_out.insert(g_out.end(), p, p + c.numel());
}

// Linear::weight()/bias() return const references; their grad() lives in the
// shared grad storage, so reading it through a non-const alias is safe.
static tl::Tensor& grad_of(const tl::Tensor& t) { return const_cast<tl::Tensor&>(t).grad(); }

static void set_params(tl::nn::Linear& lin, int64_t in, int64_t out) {
    tl::Tensor w = filled({in, out}, 0.05f);
    tl::Tensor b = filled({out}, 0.1f);
    w.set_requires_grad(true);
    b.set_requires_grad(true);
    lin.set_weight(w);
    lin.set_bias(b);
}

// Transformer-encoder attention at full size.
static void encoder_scenario() {
    tl::nn::MultiHeadAttention mha(768, 12);
    tl::nn::Linear* projs[4] = {&mha.q_proj(), &mha.k_proj(), &mha.v_proj(), &mha.out_proj()};
    for (tl::nn::Linear* l : projs) {
        tl::Tensor w = normal({768, 768}, 0.02f);
        tl::Tensor b = normal({768}, 0.02f);
        w.set_requires_grad(true);
        b.set_requires_grad(true);
        l->set_weight(w);
        l->set_bias(b);
    }
    tl::Tensor x = normal({16, 512, 768}, 1.0f);
    x.set_requires_grad(true);
    tl::Tensor y = mha.forward(x);
    y.grad() = normal(y.sizes(), 1.0f);
    y.backward();
    dump(y);
    dump(x.grad());
    dump(grad_of(mha.q_proj().weight()));
    dump(grad_of(mha.v_proj().weight()));
}

static void small_scenarios() {
    {  // Linear on a 2-D input (y = x W + b, W stored [in, out])
        tl::nn::Linear lin(300, 257);
        set_params(lin, 300, 257);
        tl::Tensor x = filled({129, 300});
        x.set_requires_grad(true);
        tl::Tensor y = lin.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(grad_of(lin.weight()));
        dump(grad_of(lin.bias()));
    }
    {  // Linear on a batched input [4, 33, 70]: the weight broadcasts over the batch
        tl::nn::Linear lin(70, 50);
        set_params(lin, 70, 50);
        tl::Tensor x = filled({4, 33, 70});
        x.set_requires_grad(true);
        tl::Tensor y = lin.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(grad_of(lin.weight()));
    }
    {  // MultiHeadAttention: projections, Q.K^T on transposed views, softmax, A.V
        tl::nn::MultiHeadAttention mha(96, 4);
        set_params(mha.q_proj(), 96, 96);
        set_params(mha.k_proj(), 96, 96);
        set_params(mha.v_proj(), 96, 96);
        set_params(mha.out_proj(), 96, 96);
        tl::Tensor x = filled({2, 40, 96});
        x.set_requires_grad(true);
        tl::Tensor y = mha.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(grad_of(mha.q_proj().weight()));
        dump(grad_of(mha.v_proj().weight()));
    }
    {  // broadcast batched matmul and its MatmulBackward
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
    {  // X . W^T with W [out, in] read through a transposed view
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
    {  // nn::Conv2d (im2col + matmul, src/ops.cpp:1443-1548) forward and backward
        tl::nn::Conv2d conv(4, 6, 3, 2, 1, 2);
        tl::Tensor w = filled({6, 2, 3, 3}, 0.2f);
        tl::Tensor b = filled({6}, 0.1f);
        w.set_requires_grad(true);
        b.set_requires_grad(true);
        conv.set_weight(w);
        conv.set_bias(b);
        tl::Tensor x = filled({2, 4, 9, 11});
        x.set_requires_grad(true);
        tl::Tensor y = conv.forward(x);
        y.grad() = filled(y.sizes());
        y.backward();
        dump(y);
        dump(x.grad());
        dump(grad_of(conv.weight()));
        dump(grad_of(conv.bias()));
    }
}

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s out.bin [encoder]\n", argv[0]);
        return 2;
    }
    if (argc >= 3 && std::strcmp(argv[2], "encoder") == 0)
        encoder_scenario();
    else
        small_scenarios();
    std::FILE* f = std::fopen(argv[1], "wb");
    if (!f) return 3;
    std::fwrite(g_out.data(), sizeof(float), g_out.size(), f);
    std::fclose(f);
    // kernels libtl_cuda launched (0 when every matmul ran on the CPU)
    std::printf("floats %zu launches %llu\n", g_out.size(),
                static_cast<unsigned long long>(tlc_launch_count()));
    return 0;
}
