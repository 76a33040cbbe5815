// The reference library's own callers of tl::matmul, unchanged, driven on
// seeded inputs: nn::Linear forward + backward (2-D and batched input),
// MultiHeadAttention forward + backward, a broadcast batched matmul and a
// transposed-weight product with their MatmulBackward.  Every output and
// gradient is written to argv[1] as raw float32.
//
// Linked (oracle/Makefile, target `callers`) from the reference's objects with
// tl::matmul redirected to libtl_cuda (torchlite-cpp_b200/integration/
// reference_matmul_gpu.cpp).  tests/test_reference_callers.py runs it twice,
// with the redirection and with TLC_REFERENCE_MATMUL=1 (the reference's CPU
// matmul), and compares the two files bit for bit in exact mode.
#include <tl/autograd.h>
#include <tl/nn.h>
#include <tl/ops.h>
#include <tl/tensor.h>

#include <tlc.h>

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

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s out.bin\n", argv[0]);
        return 2;
    }
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
    std::FILE* f = std::fopen(argv[1], "wb");
    if (!f) return 3;
    std::fwrite(g_out.data(), sizeof(float), g_out.size(), f);
    std::fclose(f);
    // kernels libtl_cuda launched (0 when every matmul ran on the CPU)
    std::printf("floats %zu launches %llu\n", g_out.size(),
                static_cast<unsigned long long>(tlc_launch_count()));
    return 0;
}
