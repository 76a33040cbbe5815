// save_model / load_model (src/model_io.cpp of torchlite-cpp) over libtl_cuda's
// TLMD entry points: the data goes straight to and from device storage.
#include <tl/model_io.h>

#include <tlc.h>

#include <new>
#include <stdexcept>
#include <string>
#include <vector>

namespace tl {

namespace {

void check(int status) {
    if (status == TLC_OK) return;
    if (status == TLC_ERR_OUT_OF_MEMORY) throw std::bad_alloc();
    if (status == TLC_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tlc_last_error());
    throw std::runtime_error(tlc_last_error());  // TLC_ERR_IO: the reference's messages
}

std::vector<tlc_tensor> views(const std::vector<Tensor*>& params, bool writable) {
    std::vector<tlc_tensor> v(params.size());
    for (size_t i = 0; i < params.size(); ++i) {
        Tensor& t = *params[i];
        if (t.sizes().size() > TLC_MAX_DIMS) throw std::invalid_argument("model_io: more than 8 dims");
        v[i].ndim = static_cast<int32_t>(t.sizes().size());
        for (int d = 0; d < v[i].ndim; ++d) {
            v[i].sizes[d] = t.sizes()[d];
            v[i].strides[d] = t.strides()[d];
        }
        if (t.numel() > 0)
            v[i].data = writable ? t.device_data() : const_cast<float*>(static_cast<const Tensor&>(t).device_data());
    }
    return v;
}

}  // namespace

void save_model(const std::string& path, const std::vector<Tensor*>& params) {
    std::vector<tlc_tensor> v = views(params, false);
    check(tlc_save_tlmd(path.c_str(), static_cast<int32_t>(v.size()), v.data(), nullptr));
}

void load_model(const std::string& path, const std::vector<Tensor*>& params) {
    for (Tensor* p : params)
        if (!p->is_contiguous())
            throw std::invalid_argument("load_model: parameters must be contiguous");
    std::vector<tlc_tensor> v = views(params, true);  // device copy current, host copy stale
    check(tlc_load_tlmd(path.c_str(), static_cast<int32_t>(v.size()), v.data(), nullptr));
}

}  // namespace tl
