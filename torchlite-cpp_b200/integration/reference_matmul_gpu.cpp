// Link-time drop-in for the reference library's tl::matmul: no source change
// in torchlite-cpp.  Compile this file against the reference's headers and
// link the reference objects with
//     -Wl,--wrap=_ZN2tl6matmulERKNS_6TensorES2_  -ltl_cuda
// Every call to tl::matmul from another object file of the library (nn::Linear,
// MultiHeadAttention, SelfAttention2d, DinoAttention, MatmulBackward::backward,
// Conv2dBackward, ...) then lands here and runs on the GPU through
// tlc_matmul_host; calls made inside ops.cpp itself keep the CPU kernels.
//
// Semantics are those of src/ops.cpp:605-699: the shape rules and exception
// texts come from tlc_matmul_shape, transposed / strided views are read in
// place (no contiguous() copy), and the MatmulBackward node is recorded exactly
// as the reference records it (caches of the contiguous inputs, squeeze flags),
// so the backward pass (whose two products call tl::matmul again) also runs on
// the GPU.  TL_GEMM_MODE selects exact (default, bit-identical) / tf32 / 3xtf32.
// There is no route back to the CPU: every call runs on the device or fails.
#include <tl/autograd.h>
#include <tl/ops.h>
#include <tl/tensor.h>

#include <tlc.h>

#include <stdexcept>
#include <string>
#include <vector>

namespace {

tlc_tensor host_view(const tl::Tensor& t) {
    tlc_tensor v{};
    if (t.sizes().size() > TLC_MAX_DIMS) throw std::invalid_argument("matmul: more than 8 dims");
    v.ndim = static_cast<int32_t>(t.sizes().size());
    for (int i = 0; i < v.ndim; ++i) {
        v.sizes[i] = t.sizes()[i];
        v.strides[i] = t.strides()[i];
    }
    v.data = t.numel() > 0 ? const_cast<float*>(t.data()) : nullptr;
    return v;
}

}  // namespace

extern "C" tl::Tensor __wrap__ZN2tl6matmulERKNS_6TensorES2_(const tl::Tensor& a_in,
                                                             const tl::Tensor& b_in) {
    tlc_tensor va = host_view(a_in), vb = host_view(b_in);
    int32_t nd = 0;
    int64_t sz[TLC_MAX_DIMS];
    if (tlc_matmul_shape(&va, &vb, &nd, sz) != TLC_OK)
        throw std::invalid_argument(tlc_last_error());
    tl::Tensor result(std::vector<int64_t>(sz, sz + nd));
    if (result.numel() > 0) {
        tlc_tensor vo = host_view(result);
        vo.data = result.data();
        const int st = tlc_matmul_host(&va, &vb, &vo, TLC_MODE_DEFAULT, nullptr);
        if (st == TLC_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tlc_last_error());
        if (st != TLC_OK) throw std::runtime_error(std::string("tlc_matmul_host: ") + tlc_last_error());
    }
    // the autograd record of src/ops.cpp:689-696
    if (a_in.requires_grad || b_in.requires_grad) {
        if (auto fn = tl::track<tl::MatmulBackward>(result, {&a_in, &b_in})) {
            fn->a_cache = a_in.contiguous();
            fn->b_cache = b_in.contiguous();
            fn->squeeze_a = a_in.sizes().size() == 1;
            fn->squeeze_b = b_in.sizes().size() == 1;
        }
    }
    return result;
}
