// Backward functions of the matmul path (src/autograd.cpp of torchlite-cpp).
#include <tl/autograd.h>
#include <tl/ops.h>

#include <tlc.h>

#include <stdexcept>
#include <string>

namespace tl {

namespace {

void check(int status, const char* what) {
    if (status == TLC_OK) return;
    if (status == TLC_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tlc_last_error());
    throw std::runtime_error(std::string(what) + ": " + tlc_last_error());
}

tlc_tensor dview(const Tensor& t) {
    tlc_tensor v{};
    v.ndim = static_cast<int32_t>(t.sizes().size());
    for (int i = 0; i < v.ndim; ++i) {
        v.sizes[i] = t.sizes()[i];
        v.strides[i] = t.strides()[i];
    }
    v.data = t.numel() > 0 ? const_cast<float*>(t.device_data()) : nullptr;
    return v;
}

tlc_tensor hview(const Tensor& t) {
    tlc_tensor v{};
    v.ndim = static_cast<int32_t>(t.sizes().size());
    for (int i = 0; i < v.ndim; ++i) {
        v.sizes[i] = t.sizes()[i];
        v.strides[i] = t.strides()[i];
    }
    v.data = t.numel() > 0 ? const_cast<float*>(t.data()) : nullptr;
    return v;
}

}  // namespace

// src/autograd.cpp:16-22: the first gradient is zeros + d, later ones add.
void accumulate_grad(Tensor& t, const Tensor& grad) {
    if (!t.requires_grad) return;
    if (t.grad().empty()) {
        Tensor z = Tensor::device_empty(t.sizes());  // zeros, made on the device
        if (z.numel() > 0)
            check(tlc_memset_zero(z.device_data(), sizeof(float) * z.numel(), nullptr),
                  "tlc_memset_zero");
        t.grad() = add(z, grad);
    } else {
        t.grad() = add(t.grad(), grad);
    }
}

// src/autograd.cpp:341-384: dA = sum_to(dC.B^T, A.shape), dB = sum_to(A^T.dC,
// B.shape), 1-D operands unsqueezed and squeezed back; both products and the
// sum_to reductions run in libtl_cuda (tlc_matmul_backward), which reads the
// transposed operands in place.  A gradient nobody requires is not computed.
void MatmulBackward::backward(const Tensor& grad_output) {
    const bool want_a = inputs[0].requires_grad, want_b = inputs[1].requires_grad;
    if (!want_a && !want_b) return;
    tlc_group* group = grad_output.numel() >= (int64_t(1) << 20) ? multi_gpu_group() : nullptr;
    if (group && grad_output.host_only() && a_cache.host_only() && b_cache.host_only()) {
        // the multi-GPU host-buffer form (TL_NUM_GPUS > 1), gradients on the host
        Tensor da(want_a ? a_cache.sizes() : std::vector<int64_t>{0});
        Tensor db(want_b ? b_cache.sizes() : std::vector<int64_t>{0});
        tlc_tensor g = hview(grad_output), a = hview(a_cache), b = hview(b_cache);
        tlc_tensor vda = hview(da), vdb = hview(db);
        if (want_a) vda.data = da.data();
        if (want_b) vdb.data = db.data();
        check(tlc_group_matmul_backward_host(group, &g, &a, &b, want_a ? &vda : nullptr,
                                             want_b ? &vdb : nullptr, 0, mode),
              "tlc_group_matmul_backward_host");
        if (want_a) accumulate_grad(inputs[0], da);
        if (want_b) accumulate_grad(inputs[1], db);
        return;
    }
    tlc_tensor g = dview(grad_output), a = dview(a_cache), b = dview(b_cache);
    Tensor da, db;
    tlc_tensor vda{}, vdb{};
    if (want_a) {
        da = Tensor::device_empty(a_cache.sizes());
        vda = dview(da);
        if (!vda.data) vda.data = reinterpret_cast<float*>(16);  // empty: nothing is written
    }
    if (want_b) {
        db = Tensor::device_empty(b_cache.sizes());
        vdb = dview(db);
        if (!vdb.data) vdb.data = reinterpret_cast<float*>(16);
    }
    check(tlc_matmul_backward(&g, &a, &b, want_a ? &vda : nullptr, want_b ? &vdb : nullptr, 0,
                              mode, nullptr),
          "tlc_matmul_backward");
    if (want_a) accumulate_grad(inputs[0], da);
    if (want_b) accumulate_grad(inputs[1], db);
}

// src/autograd.cpp:131-133
void TransposeBackward::backward(const Tensor& grad_output) {
    accumulate_grad(inputs[0], transpose(grad_output, dim0, dim1));
}

void ReshapeBackward::backward(const Tensor& grad_output) {
    accumulate_grad(inputs[0], reshape(grad_output, input_shape));
}

// src/autograd.cpp:68-71
void AddBackward::backward(const Tensor& grad_output) {
    if (inputs[0].requires_grad) accumulate_grad(inputs[0], sum_to(grad_output, inputs[0].sizes()));
    if (inputs[1].requires_grad) accumulate_grad(inputs[1], sum_to(grad_output, inputs[1].sizes()));
}

// src/autograd.cpp:82-84
void ScaleBackward::backward(const Tensor& grad_output) {
    accumulate_grad(inputs[0], scale(grad_output, scalar));
}

// src/autograd.cpp:228-256
void SoftmaxBackward::backward(const Tensor& grad_output) {
    if (!inputs[0].requires_grad) return;
    Tensor dx = Tensor::device_empty(output_cache.sizes());
    if (dx.numel() > 0) {
        tlc_tensor g = dview(grad_output), y = dview(output_cache), vd = dview(dx);
        check(tlc_softmax_backward(&g, &y, &vd, nullptr), "tlc_softmax_backward");
    }
    accumulate_grad(inputs[0], dx);
}

// src/autograd.cpp:575-669: dQ, dK, dV from libtl_cuda (recomputed
// probabilities, batched GEMMs), then accumulate_grad into Q, K, V.
void FlashAttentionBackward::backward(const Tensor& grad_output) {
    Tensor dq = Tensor::device_empty(Q_cache.sizes()), dk = Tensor::device_empty(Q_cache.sizes()),
           dv = Tensor::device_empty(Q_cache.sizes());
    if (dq.numel() > 0) {
        Tensor g = grad_output.contiguous();
        tlc_tensor vg = dview(g), vq = dview(Q_cache), vk = dview(K_cache), vv = dview(V_cache),
                   vo = dview(O_cache), vl = dview(L_cache), vdq = dview(dq), vdk = dview(dk),
                   vdv = dview(dv);
        check(tlc_flash_attention_backward(&vg, &vq, &vk, &vv, &vo, &vl, sm_scale, &vdq, &vdk, &vdv,
                                           mode, nullptr),
              "tlc_flash_attention_backward");
    }
    if (inputs[0].requires_grad) accumulate_grad(inputs[0], dq);
    if (inputs[1].requires_grad) accumulate_grad(inputs[1], dk);
    if (inputs[2].requires_grad) accumulate_grad(inputs[2], dv);
}

// src/autograd.cpp:386-517: all three gradients from libtl_cuda in the
// reference's summation orders, then accumulate_grad.
void Conv2dBackward::backward(const Tensor& grad_output) {
    const bool want_i = inputs[0].requires_grad, want_w = inputs[1].requires_grad;
    const bool want_b = inputs.size() > 2 && inputs[2].requires_grad && !inputs[2].empty();
    if (!want_i && !want_w && !want_b) return;
    Tensor di, dw, db;
    tlc_tensor vdi{}, vdw{}, vdb{};
    if (want_i) {
        di = Tensor::device_empty(input_cache.sizes());
        vdi = dview(di);
    }
    if (want_w) {
        dw = Tensor::device_empty(weight_cache.sizes());
        vdw = dview(dw);
    }
    if (want_b) {
        db = Tensor::device_empty({weight_cache.sizes()[0]});
        vdb = dview(db);
    }
    tlc_tensor g = dview(grad_output), x = dview(input_cache), w = dview(weight_cache);
    check(tlc_conv2d_backward(&g, &x, &w, stride, padding, groups, want_i ? &vdi : nullptr,
                              want_w ? &vdw : nullptr, want_b ? &vdb : nullptr, mode, nullptr),
          "tlc_conv2d_backward");
    if (want_i) accumulate_grad(inputs[0], di);
    if (want_w) accumulate_grad(inputs[1], dw);
    if (want_b) accumulate_grad(inputs[2], db);
}

// ScaleBackward (scale(grad, s)) or AddBackward (grad to the product unchanged,
// sum_to(grad, [N]) to the bias), then MatmulBackward, as the reference's
// separate nodes would run them.
void FusedMatmulBackward::backward(const Tensor& grad_output) {
    Tensor g = apply_scale ? scale(grad_output, scalar) : grad_output;
    if (has_bias && inputs[2].requires_grad)
        accumulate_grad(inputs[2], sum_to(grad_output, inputs[2].sizes()));
    MatmulBackward mm;
    mm.inputs = {inputs[0], inputs[1]};
    mm.a_cache = a_cache;
    mm.b_cache = b_cache;
    mm.squeeze_a = a_cache.sizes().size() == 1;
    mm.squeeze_b = b_cache.sizes().size() == 1;
    mm.mode = mode;
    mm.backward(g);
}

}  // namespace tl
