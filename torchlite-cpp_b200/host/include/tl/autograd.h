// Autograd for the matmul path (include/tl/autograd.h of torchlite-cpp):
// the same GradFunction / track<> protocol, with MatmulBackward running
// libtl_cuda's backward (dA = dC.B^T, dB = A^T.dC reduced with sum_to) on the
// GPU, transposed operands read in place.
#pragma once

#include <tl/tensor.h>

#include <cstdint>
#include <initializer_list>
#include <memory>
#include <vector>

namespace tl {

inline bool& grad_enabled() {
    static bool e = true;
    return e;
}

struct NoGradGuard {
    bool prev;
    NoGradGuard() : prev(grad_enabled()) { grad_enabled() = false; }
    ~NoGradGuard() { grad_enabled() = prev; }
};

class GradFunction {
  public:
    virtual ~GradFunction() = default;
    virtual void backward(const Tensor& grad_output) = 0;
    std::vector<Tensor> inputs;
};

// src/autograd.cpp:341-384
class MatmulBackward : public GradFunction {
  public:
    Tensor a_cache, b_cache;  // the inputs as given (views; no contiguous copies)
    bool squeeze_a = false, squeeze_b = false;
    int mode = -1;
    void backward(const Tensor& grad_output) override;
};

// src/autograd.cpp:131-133
class TransposeBackward : public GradFunction {
  public:
    int64_t dim0 = 0, dim1 = 0;
    void backward(const Tensor& grad_output) override;
};

class ReshapeBackward : public GradFunction {
  public:
    std::vector<int64_t> input_shape;
    void backward(const Tensor& grad_output) override;
};

// src/autograd.cpp:68-71: each input receives sum_to(grad, its shape)
class AddBackward : public GradFunction {
  public:
    void backward(const Tensor& grad_output) override;
};

// src/autograd.cpp:82-84
class ScaleBackward : public GradFunction {
  public:
    float scalar = 1.0f;
    void backward(const Tensor& grad_output) override;
};

// src/autograd.cpp:228-256 (row dot rounded as the reference's x86-64-v4 build)
class SoftmaxBackward : public GradFunction {
  public:
    Tensor output_cache;
    void backward(const Tensor& grad_output) override;
};

// src/autograd.cpp:386-517 (inputs: input, weight, bias)
class Conv2dBackward : public GradFunction {
  public:
    Tensor input_cache, weight_cache;
    int64_t stride = 1, padding = 0, groups = 1;
    int mode = -1;
    void backward(const Tensor& grad_output) override;
};

// src/autograd.cpp:575-669 (inputs: Q, K, V); the caches as the reference keeps
// them (contiguous Q, K, V, the output O and L = m + log(l) per row)
class FlashAttentionBackward : public GradFunction {
  public:
    Tensor Q_cache, K_cache, V_cache, O_cache, L_cache;
    float sm_scale = 1.0f;
    int mode = -1;
    void backward(const Tensor& grad_output) override;
};

// matmul_add / matmul_scale: the reference's AddBackward or ScaleBackward
// followed by MatmulBackward, in one node
class FusedMatmulBackward : public GradFunction {
  public:
    Tensor a_cache, b_cache;
    bool has_bias = false;  // inputs[2] is the bias
    float scalar = 1.0f;
    bool apply_scale = false;
    int mode = -1;
    void backward(const Tensor& grad_output) override;
};

// grad += d (grad = zeros + d when empty), src/autograd.cpp:16-22
void accumulate_grad(Tensor& t, const Tensor& grad);

template <typename BackwardFn>
std::shared_ptr<BackwardFn> track(Tensor& out, std::initializer_list<const Tensor*> inputs) {
    if (!grad_enabled()) return nullptr;
    out.requires_grad = true;
    out.ensure_grad();
    auto fn = std::make_shared<BackwardFn>();
    for (auto* t : inputs) {
        const_cast<Tensor*>(t)->ensure_grad();
        fn->inputs.push_back(*const_cast<Tensor*>(t));  // shallow copy, shared grad_
    }
    out.grad_fn = fn;
    return fn;
}

}  // namespace tl
