// tl:: ops of the matmul path over libtl_cuda (include/tlc.h).  Shapes, views
// and error messages follow src/ops.cpp of torchlite-cpp; the arithmetic runs
// on the GPU.
#include <tl/autograd.h>
#include <tl/ops.h>

#include <tlc.h>

#include <algorithm>
#include <cstdlib>
#include <memory>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

namespace tl {

namespace {

void check(int status, const char* what) {
    if (status == TLC_OK) return;
    if (status == TLC_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tlc_last_error());
    if (status == TLC_ERR_OUT_OF_MEMORY) throw std::bad_alloc();
    throw std::runtime_error(std::string(what) + ": " + tlc_last_error());
}

// The C-ABI view of a tensor; `device` picks the device copy as data pointer.
tlc_tensor view_of(const Tensor& t, bool device) {
    tlc_tensor v{};
    if (t.sizes().size() > TLC_MAX_DIMS) throw std::invalid_argument("matmul: more than 8 dims");
    v.ndim = static_cast<int32_t>(t.sizes().size());
    for (int i = 0; i < v.ndim; ++i) {
        v.sizes[i] = t.sizes()[i];
        v.strides[i] = t.strides()[i];
    }
    v.data = device && t.numel() > 0 ? const_cast<float*>(t.device_data()) : nullptr;
    return v;
}

// The C-ABI view of a tensor's host copy (refreshed if stale).
tlc_tensor host_view_of(const Tensor& t) {
    tlc_tensor v = view_of(t, false);
    v.data = t.numel() > 0 ? const_cast<float*>(t.data()) : nullptr;
    return v;
}

// The same storage and view without the autograd links: what a node keeps of
// its own output, so that the node and the output do not own each other.
Tensor detached(const Tensor& t) {
    Tensor d = t;
    d.grad_fn.reset();
    d.requires_grad = false;
    return d;
}

}  // namespace

Tensor matmul(const Tensor& a_in, const Tensor& b_in) {
    return matmul(a_in, b_in, TLC_MODE_DEFAULT);
}

tlc_group* multi_gpu_group() {
    static tlc_group* group = []() -> tlc_group* {
        const char* e = std::getenv("TL_NUM_GPUS");
        const int want = e ? std::atoi(e) : 1;
        if (want <= 1) return nullptr;
        int count = 0;
        check(tlc_device_count(&count), "tlc_device_count");
        std::vector<int> devs(std::min(want, count));
        for (size_t i = 0; i < devs.size(); ++i) devs[i] = static_cast<int>(i);
        if (devs.size() < 2) return nullptr;
        tlc_group* g = nullptr;  // lives as long as the process
        check(tlc_group_create(devs.data(), static_cast<int>(devs.size()), &g), "tlc_group_create");
        return g;
    }();
    return group;
}

namespace {
// Products smaller than this stay on one GPU: below it the copies and
// launches on more devices cost more than their share of the work.
constexpr int64_t kGroupMinOutputs = int64_t(1) << 20;
}  // namespace

// src/ops.cpp:605-699
Tensor matmul(const Tensor& a_in, const Tensor& b_in, int mode) {
    // shape rules and their exceptions first; they need no GPU
    tlc_tensor va = view_of(a_in, false), vb = view_of(b_in, false);
    int32_t nd = 0;
    int64_t sz[TLC_MAX_DIMS];
    check(tlc_matmul_shape(&va, &vb, &nd, sz), "tlc_matmul_shape");
    const std::vector<int64_t> shape(sz, sz + nd);
    int64_t outputs = 1;
    for (int64_t v : shape) outputs *= v;
    tlc_group* group = outputs >= kGroupMinOutputs ? multi_gpu_group() : nullptr;
    Tensor out;
    if (group && a_in.host_only() && b_in.host_only()) {
        // host operands: every GPU copies in its share; the result stays on the host
        out = Tensor(shape);
        va = host_view_of(a_in);
        vb = host_view_of(b_in);
        tlc_tensor vo = view_of(out, false);
        vo.data = out.data();
        check(tlc_group_matmul_host(group, &va, &vb, &vo, mode), "tlc_group_matmul_host");
    } else {
        out = Tensor::device_empty(shape);
        if (out.numel() > 0) {
            va = view_of(a_in, true);
            vb = view_of(b_in, true);
            tlc_tensor vo = view_of(out, false);
            vo.data = out.device_data();
            if (group)
                check(tlc_group_matmul(group, &va, &vb, &vo, mode, nullptr), "tlc_group_matmul");
            else
                check(tlc_matmul(&va, &vb, &vo, mode, nullptr), "tlc_matmul");
        }
    }
    if (a_in.requires_grad || b_in.requires_grad) {
        if (auto fn = track<MatmulBackward>(out, {&a_in, &b_in})) {
            fn->a_cache = a_in;  // views are read in place: no contiguous copies
            fn->b_cache = b_in;
            fn->squeeze_a = a_in.sizes().size() == 1;
            fn->squeeze_b = b_in.sizes().size() == 1;
            fn->mode = mode;
        }
    }
    return out;
}

// src/ops.cpp:702-730
Tensor transpose(const Tensor& a, int64_t dim0, int64_t dim1) {
    const int64_t ndim = static_cast<int64_t>(a.sizes().size());
    if (dim0 < 0) dim0 += ndim;
    if (dim1 < 0) dim1 += ndim;
    if (dim0 < 0 || dim0 >= ndim || dim1 < 0 || dim1 >= ndim)
        throw std::invalid_argument("tranpose: dimension out of range");
    auto sizes = a.sizes();
    auto strides = a.strides();
    std::swap(sizes[dim0], sizes[dim1]);
    std::swap(strides[dim0], strides[dim1]);
    Tensor out = a.view(sizes, strides, a.storage_offset());
    if (a.requires_grad) {
        if (auto fn = track<TransposeBackward>(out, {&a})) {
            fn->dim0 = dim0;
            fn->dim1 = dim1;
        }
    }
    return out;
}

// src/ops.cpp:732-767
Tensor reshape(const Tensor& a, const std::vector<int64_t>& new_sizes) {
    int64_t n = 1;
    for (int64_t s : new_sizes) {
        if (s < 0) throw std::invalid_argument("reshape: negative dims not allowed");
        n *= s;
    }
    if (n != a.numel())
        throw std::invalid_argument("reshape: new shape must have same number of elements");
    Tensor c = a.is_contiguous() ? a : a.contiguous();
    std::vector<int64_t> st(new_sizes.size());
    int64_t s = 1;
    for (int i = static_cast<int>(new_sizes.size()) - 1; i >= 0; --i) {
        st[i] = s;
        s *= new_sizes[i];
    }
    Tensor out = c.view(new_sizes, st, c.storage_offset());
    if (a.requires_grad) {
        if (auto fn = track<ReshapeBackward>(out, {&a})) fn->input_shape = a.sizes();
    }
    return out;
}

Tensor unsqueeze(const Tensor& input, int64_t dim) {
    const int64_t nd = static_cast<int64_t>(input.sizes().size());
    if (dim < 0) dim += nd + 1;
    if (dim < 0 || dim > nd) throw std::invalid_argument("unsqueeze: dim out of range");
    auto s = input.sizes();
    s.insert(s.begin() + dim, 1);
    return reshape(input, s);
}

Tensor squeeze(const Tensor& input, int64_t dim) {
    const int64_t nd = static_cast<int64_t>(input.sizes().size());
    if (dim < 0) dim += nd;
    if (dim < 0 || dim >= nd) throw std::invalid_argument("squeeze: dim out of range");
    if (input.sizes()[dim] != 1) throw std::invalid_argument("squeeze: dim is not size 1");
    if (nd == 1) throw std::invalid_argument("squeeze: cannot squeeze 1D to 0D");
    auto s = input.sizes();
    s.erase(s.begin() + dim);
    return reshape(input, s);
}

// The result shape of a broadcast (src/ops.cpp:55-72; a size-0 dim against a
// size-1 dim gives 0).
std::vector<int64_t> broadcast_sizes(const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
    const size_t nd = std::max(a.size(), b.size());
    std::vector<int64_t> out(nd);
    for (size_t i = 0; i < nd; ++i) {
        const int64_t sa = i < nd - a.size() ? 1 : a[i - (nd - a.size())];
        const int64_t sb = i < nd - b.size() ? 1 : b[i - (nd - b.size())];
        if (sa != sb && sa != 1 && sb != 1)
            throw std::invalid_argument("Incompatible dimensions for broadcasting");
        out[i] = sa == 1 ? sb : sa;
    }
    return out;
}

// src/ops.cpp:74-103
Tensor add(const Tensor& a_in, const Tensor& b_in) {
    Tensor out = Tensor::device_empty(broadcast_sizes(a_in.sizes(), b_in.sizes()));
    if (out.numel() > 0) {
        tlc_tensor va = view_of(a_in, true), vb = view_of(b_in, true), vo = view_of(out, false);
        vo.data = out.device_data();
        check(tlc_add_tensors(&va, &vb, &vo, nullptr), "tlc_add_tensors");
    }
    if (a_in.requires_grad || b_in.requires_grad) track<AddBackward>(out, {&a_in, &b_in});
    return out;
}

// src/ops.cpp:963-983
Tensor scale(const Tensor& input, float scalar) {
    Tensor out = Tensor::device_empty(input.sizes());
    if (out.numel() > 0) {
        tlc_tensor vx = view_of(input, true), vo = view_of(out, false);
        vo.data = out.device_data();
        check(tlc_scale(&vx, scalar, &vo, nullptr), "tlc_scale");
    }
    if (input.requires_grad) {
        if (auto fn = track<ScaleBackward>(out, {&input})) fn->scalar = scalar;
    }
    return out;
}

// src/ops.cpp:985-1037
Tensor softmax(const Tensor& input) {
    if (input.sizes().empty()) throw std::invalid_argument("Softmax requires at least 1D tensor");
    Tensor out = Tensor::device_empty(input.sizes());
    if (out.numel() > 0) {
        tlc_tensor vx = view_of(input, true), vo = view_of(out, false);
        vo.data = out.device_data();
        check(tlc_softmax(&vx, &vo, nullptr), "tlc_softmax");
    }
    if (input.requires_grad) {
        if (auto fn = track<SoftmaxBackward>(out, {&input})) fn->output_cache = detached(out);
    }
    return out;
}

// src/autograd.cpp:24-36
Tensor sum_to(const Tensor& grad, const std::vector<int64_t>& target_shape) {
    Tensor out = Tensor::device_empty(target_shape);
    tlc_tensor vx = view_of(grad, true), vo = view_of(out, false);
    vo.data = out.numel() > 0 ? out.device_data() : nullptr;
    check(tlc_sum_to(&vx, &vo, nullptr), "tlc_sum_to");
    return out;
}

namespace {

Tensor matmul_fused(const Tensor& a_in, const Tensor& b_in, const Tensor* bias, float scalar,
                    bool apply_scale, int mode) {
    tlc_tensor va = view_of(a_in, false), vb = view_of(b_in, false);
    int32_t nd = 0;
    int64_t sz[TLC_MAX_DIMS];
    check(tlc_matmul_shape(&va, &vb, &nd, sz), "tlc_matmul_shape");
    Tensor out = Tensor::device_empty(std::vector<int64_t>(sz, sz + nd));
    if (out.numel() > 0) {
        va = view_of(a_in, true);
        vb = view_of(b_in, true);
        tlc_tensor vo = view_of(out, false);
        vo.data = out.device_data();
        tlc_tensor vbias{};
        if (bias) vbias = view_of(*bias, true);
        check(tlc_matmul_fused(&va, &vb, apply_scale ? scalar : 1.0f, bias ? &vbias : nullptr, &vo,
                               mode, nullptr),
              "tlc_matmul_fused");
    }
    const bool grads = a_in.requires_grad || b_in.requires_grad || (bias && bias->requires_grad);
    if (grads) {
        std::shared_ptr<FusedMatmulBackward> fn =
            bias ? track<FusedMatmulBackward>(out, {&a_in, &b_in, bias})
                 : track<FusedMatmulBackward>(out, {&a_in, &b_in});
        if (fn) {
            fn->a_cache = a_in;
            fn->b_cache = b_in;
            fn->has_bias = bias != nullptr;
            fn->scalar = scalar;
            fn->apply_scale = apply_scale;
            fn->mode = mode;
        }
    }
    return out;
}

}  // namespace

Tensor matmul_add(const Tensor& a, const Tensor& b, const Tensor& bias) {
    if (bias.sizes().size() != 1)
        throw std::invalid_argument("matmul_add: bias must be 1-D");
    return matmul_fused(a, b, &bias, 1.0f, false, TLC_MODE_DEFAULT);
}

Tensor matmul_scale(const Tensor& a, const Tensor& b, float scalar) {
    return matmul_fused(a, b, nullptr, scalar, true, TLC_MODE_DEFAULT);
}

// src/ops.cpp:1443-1548
Tensor conv2d(const Tensor& input, const Tensor& weight, const Tensor& bias, int64_t stride,
              int64_t padding, int64_t groups) {
    tlc_tensor vi = view_of(input, false), vw = view_of(weight, false);
    int64_t sz[4];
    check(tlc_conv2d_shape(&vi, &vw, stride, padding, groups, sz), "tlc_conv2d_shape");
    Tensor out = Tensor::device_empty(std::vector<int64_t>(sz, sz + 4));
    if (out.numel() > 0) {
        vi = view_of(input, true);
        vw = view_of(weight, true);
        tlc_tensor vb{}, vo = view_of(out, false);
        vo.data = out.device_data();
        if (!bias.empty()) vb = view_of(bias, true);
        check(tlc_conv2d(&vi, &vw, bias.empty() ? nullptr : &vb, stride, padding, groups, &vo,
                         TLC_MODE_DEFAULT, nullptr),
              "tlc_conv2d");
    }
    if (input.requires_grad || weight.requires_grad) {
        if (auto fn = track<Conv2dBackward>(out, {&input, &weight, &bias})) {
            fn->input_cache = input;
            fn->weight_cache = weight;
            fn->stride = stride;
            fn->padding = padding;
            fn->groups = groups;
            fn->mode = TLC_MODE_DEFAULT;
        }
    }
    return out;
}

// src/ops.cpp:1040-1137
Tensor flash_attention(const Tensor& Q, const Tensor& K, const Tensor& V, float sm_scale) {
    if (Q.sizes().size() < 2) throw std::invalid_argument("flash_attention: tensors must be at least 2-D [S, d]");
    Tensor Qc = Q.contiguous(), Kc = K.contiguous(), Vc = V.contiguous();
    Tensor O = Tensor::device_empty(Qc.sizes());
    Tensor L = Tensor::device_empty(std::vector<int64_t>(Qc.sizes().begin(), Qc.sizes().end() - 1));
    tlc_tensor vq = view_of(Qc, true), vk = view_of(Kc, true), vv = view_of(Vc, true);
    tlc_tensor vo = view_of(O, false), vl = view_of(L, false);
    if (O.numel() > 0) vo.data = O.device_data();
    if (L.numel() > 0) vl.data = L.device_data();
    check(tlc_flash_attention(&vq, &vk, &vv, sm_scale, &vo, &vl, TLC_MODE_DEFAULT, nullptr),
          "tlc_flash_attention");
    if (Q.requires_grad || K.requires_grad || V.requires_grad) {
        if (auto fn = track<FlashAttentionBackward>(O, {&Q, &K, &V})) {
            fn->Q_cache = Qc;
            fn->K_cache = Kc;
            fn->V_cache = Vc;
            fn->O_cache = detached(O);
            fn->L_cache = L;
            fn->sm_scale = sm_scale;
            fn->mode = TLC_MODE_DEFAULT;
        }
    }
    return O;
}

Tensor sum(const Tensor& input, int64_t dim, bool keepdim) {
    Tensor a = input.contiguous();
    const auto& sizes = a.sizes();
    const int64_t nd = static_cast<int64_t>(sizes.size());
    if (dim < 0) dim += nd;
    if (dim < 0 || dim >= nd) throw std::invalid_argument("sum: dimension out of range");
    std::vector<int64_t> out_sizes;
    int64_t outer = 1, inner = 1;
    for (int64_t i = 0; i < nd; ++i) {
        if (i == dim) {
            if (keepdim) out_sizes.push_back(1);
        } else {
            out_sizes.push_back(sizes[i]);
        }
        if (i < dim) outer *= sizes[i];
        if (i > dim) inner *= sizes[i];
    }
    Tensor out = Tensor::device_empty(out_sizes);
    if (out.numel() > 0)
        check(tlc_sum_dim(a.device_data(), out.device_data(), outer, sizes[dim], inner, nullptr),
              "tlc_sum_dim");
    return out;
}

Tensor zeros(const std::vector<int64_t>& sizes) { return Tensor(sizes); }

Tensor full(const std::vector<int64_t>& sizes, float value) {
    Tensor t(sizes);
    float* p = t.data();
    for (int64_t i = 0; i < t.numel(); ++i) p[i] = value;
    return t;
}

Tensor ones(const std::vector<int64_t>& sizes) { return full(sizes, 1.0f); }

}  // namespace tl
