// tl::Tensor with mirrored host / device storage (see tensor.h).  Shape,
// stride and autograd logic follow src/tensor.cpp of torchlite-cpp.
#include <tl/autograd.h>
#include <tl/tensor.h>

#include <tlc.h>

#include <algorithm>
#include <cstring>
#include <functional>
#include <new>
#include <set>
#include <stdexcept>
#include <string>

namespace tl {

namespace {

void check(int status, const char* what) {
    if (status == TLC_OK) return;
    if (status == TLC_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tlc_last_error());
    if (status == TLC_ERR_OUT_OF_MEMORY) throw std::bad_alloc();
    throw std::runtime_error(std::string(what) + ": " + tlc_last_error());
}

int64_t compute_numel(const std::vector<int64_t>& sizes) {
    int64_t n = 1;
    for (int64_t d : sizes) n *= d;
    return n;
}

std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& sizes) {
    std::vector<int64_t> st(sizes.size());
    int64_t s = 1;
    for (int i = static_cast<int>(sizes.size()) - 1; i >= 0; --i) {
        st[i] = s;
        s *= sizes[i];
    }
    return st;
}

}  // namespace

// ---- Storage ---------------------------------------------------------------------------

Storage::Storage(int64_t n, bool zero_host) : n_(n) {
    if (zero_host) {
        host_.assign(static_cast<size_t>(n), 0.0f);
        host_valid_ = true;
    } else {
        host_valid_ = false;
    }
}

Storage::~Storage() {
    if (dev_) tlc_free(dev_);
}

float* Storage::device_raw() {
    if (!dev_ && n_ > 0) {
        void* p = nullptr;
        check(tlc_malloc(&p, sizeof(float) * static_cast<size_t>(n_)), "tlc_malloc");
        dev_ = static_cast<float*>(p);
    }
    return dev_;
}

float* Storage::device() {
    float* d = device_raw();
    if (!dev_valid_ && n_ > 0) {
        if (host_valid_)
            check(tlc_memcpy(d, host_.data(), sizeof(float) * n_, 0, nullptr), "h2d");
        dev_valid_ = true;
    }
    return d;
}

float* Storage::host() {
    if (host_.size() != static_cast<size_t>(n_)) host_.assign(static_cast<size_t>(n_), 0.0f);
    if (!host_valid_ && n_ > 0) {
        if (dev_valid_) {
            check(tlc_memcpy(host_.data(), dev_, sizeof(float) * n_, 1, nullptr), "d2h");
            check(tlc_stream_synchronize(nullptr), "sync");
        }
        host_valid_ = true;
    }
    return host_.data();
}

// ---- Tensor ----------------------------------------------------------------------------

Tensor::Tensor() : data_(nullptr), numel_(0), offset_(0) {}

Tensor::Tensor(const std::vector<int64_t>& sizes)
    : sizes_(sizes), strides_(contiguous_strides(sizes)), offset_(0) {
    numel_ = compute_numel(sizes_);
    data_ = std::make_shared<Storage>(numel_);
}

Tensor Tensor::device_empty(const std::vector<int64_t>& sizes) {
    Tensor t;
    t.sizes_ = sizes;
    t.strides_ = contiguous_strides(sizes);
    t.numel_ = compute_numel(sizes);
    t.data_ = std::make_shared<Storage>(t.numel_, /*zero_host=*/false);
    t.data_->device_raw();
    t.data_->wrote_device();
    return t;
}

Tensor Tensor::view(const std::vector<int64_t>& sizes, const std::vector<int64_t>& strides,
                    int64_t offset) const {
    Tensor t;
    t.data_ = data_;
    t.sizes_ = sizes;
    t.strides_ = strides;
    t.offset_ = offset;
    t.numel_ = compute_numel(sizes);
    return t;
}

float* Tensor::data() {
    if (!data_) return nullptr;
    float* p = data_->host() + offset_;
    data_->wrote_host();  // the caller may write
    return p;
}

const float* Tensor::data() const {
    if (!data_) return nullptr;
    return data_->host() + offset_;
}

float* Tensor::device_data() {
    if (!data_) return nullptr;
    float* p = data_->device() + offset_;
    data_->wrote_device();  // the caller may write
    return p;
}

const float* Tensor::device_data() const {
    if (!data_) return nullptr;
    return data_->device() + offset_;
}

float& Tensor::at(int64_t i) {
    if (i < 0 || i >= numel_) throw std::out_of_range("Tensor::at index out of range");
    return data()[i];
}

const float& Tensor::at(int64_t i) const {
    if (i < 0 || i >= numel_) throw std::out_of_range("Tensor::at index out of range");
    return data()[i];
}

bool Tensor::host_only() const {
    return !data_ || (data_->host_valid() && !data_->device_valid());
}

const std::vector<int64_t>& Tensor::sizes() const { return sizes_; }
const std::vector<int64_t>& Tensor::strides() const { return strides_; }
int64_t Tensor::numel() const { return numel_; }
int64_t Tensor::storage_offset() const { return offset_; }
bool Tensor::empty() const { return numel_ == 0; }

bool Tensor::is_contiguous() const {
    if (sizes_.empty()) return true;
    int64_t expected = 1;
    for (int i = static_cast<int>(sizes_.size()) - 1; i >= 0; --i) {
        if (strides_[i] != expected) return false;
        expected *= sizes_[i];
    }
    return true;
}

// Tensor::contiguous (src/tensor.cpp:174-193), done on the device.
Tensor Tensor::contiguous() const {
    if (is_contiguous()) return *this;
    Tensor out = Tensor::device_empty(sizes_);
    if (numel_ > 0) {
        tlc_tensor v{};
        v.data = const_cast<float*>(device_data());
        v.ndim = static_cast<int32_t>(sizes_.size());
        for (size_t i = 0; i < sizes_.size(); ++i) {
            v.sizes[i] = sizes_[i];
            v.strides[i] = strides_[i];
        }
        check(tlc_contiguous(&v, out.data_->device_raw(), nullptr), "tlc_contiguous");
    }
    return out;
}

Tensor Tensor::clone() const {
    Tensor c = contiguous();
    if (c.data_ != data_) return c;
    Tensor out = Tensor::device_empty(sizes_);
    if (numel_ > 0)
        check(tlc_memcpy(out.data_->device_raw(), c.device_data(), sizeof(float) * numel_, 2,
                         nullptr),
              "d2d");
    return out;
}

void Tensor::ensure_grad() {
    if (!grad_) grad_ = std::make_shared<Tensor>();
}

void Tensor::set_requires_grad(bool val) {
    requires_grad = val;
    if (val) ensure_grad();
}

Tensor& Tensor::grad() {
    ensure_grad();
    return *grad_;
}

// Tensor::backward (src/tensor.cpp:209-242): seed ones if the grad is empty,
// topological sort, reverse walk under NoGradGuard.
void Tensor::backward() {
    if (!grad_) grad_ = std::make_shared<Tensor>();
    if (grad_->empty()) {
        *grad_ = Tensor(sizes_);
        float* p = grad_->data();
        for (int64_t i = 0; i < numel_; ++i) p[i] = 1.0f;
    }
    std::vector<Tensor*> order;
    std::set<void*> visited;
    std::function<void(Tensor*)> topo = [&](Tensor* t) {
        void* key = t->grad_ ? static_cast<void*>(t->grad_.get()) : static_cast<void*>(t);
        if (visited.count(key)) return;
        visited.insert(key);
        if (t->grad_fn)
            for (auto& input : t->grad_fn->inputs) topo(&input);
        order.push_back(t);
    };
    topo(this);
    NoGradGuard no_grad;
    for (auto it = order.rbegin(); it != order.rend(); ++it)
        if ((*it)->grad_fn) (*it)->grad_fn->backward(*(*it)->grad_);
}

std::ostream& operator<<(std::ostream& os, const Tensor& t) {
    os << "Tensor(sizes=[";
    for (size_t i = 0; i < t.sizes().size(); ++i) os << (i ? ", " : "") << t.sizes()[i];
    os << "])";
    return os;
}

}  // namespace tl
