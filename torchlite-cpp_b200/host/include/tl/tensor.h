// tl::Tensor with CUDA device-buffer backing, for the matmul path on B200.
//
// Same interface as the reference's Tensor (include/tl/tensor.h:13-67 of
// torchlite-cpp): a strided fp32 view (sizes, strides, offset) over shared
// storage, with the same autograd members.  The storage is mirrored: a host
// copy (what data() returns) and a device copy (what device_data() returns,
// allocated through libtl_cuda), each with a validity bit.  Writing through
// non-const data() invalidates the device copy; GPU results invalidate the
// host copy; the stale side is refreshed on its next use.  So code written
// against the reference (fill data(), call tl::matmul, read data()) runs
// unchanged, while chains of GPU ops never leave the device.
#pragma once

#include <cstdint>
#include <memory>
#include <ostream>
#include <vector>

namespace tl {

class GradFunction;

// Host + device copies of one buffer of floats.
struct Storage {
    explicit Storage(int64_t n, bool zero_host = true);
    ~Storage();
    Storage(const Storage&) = delete;
    Storage& operator=(const Storage&) = delete;

    float* host();                // valid host copy (copies device -> host if stale)
    float* device();              // valid device copy (allocates / copies host -> device)
    void wrote_host() { dev_valid_ = false; host_valid_ = true; }
    void wrote_device() { host_valid_ = false; dev_valid_ = true; }
    float* device_raw();          // device buffer, contents not refreshed (for outputs)
    int64_t size() const { return n_; }
    bool host_valid() const { return host_valid_; }
    bool device_valid() const { return dev_valid_; }

  private:
    int64_t n_;
    std::vector<float> host_;
    float* dev_ = nullptr;
    bool host_valid_ = true, dev_valid_ = false;
};

class Tensor {
  public:
    Tensor();
    explicit Tensor(const std::vector<int64_t>& sizes);  // zero-filled, like the reference

    // A contiguous tensor whose only copy is on the device (contents undefined):
    // the output of a GPU op.
    static Tensor device_empty(const std::vector<int64_t>& sizes);

    // host access (refreshes the host copy; non-const marks the device copy stale)
    float* data();
    const float* data() const;
    float& at(int64_t index);
    const float& at(int64_t index) const;
    // device access (refreshes the device copy; non-const marks the host copy stale)
    float* device_data();
    const float* device_data() const;

    Tensor contiguous() const;
    Tensor clone() const;

    // Only the host copy is current (a tensor filled through data() and not
    // yet used on the device): the multi-GPU host-buffer path reads it there.
    bool host_only() const;

    const std::vector<int64_t>& sizes() const;
    const std::vector<int64_t>& strides() const;
    int64_t numel() const;
    bool is_contiguous() const;
    int64_t storage_offset() const;
    bool empty() const;

    void set_requires_grad(bool val);
    void ensure_grad();
    Tensor& grad();
    void backward();
    bool requires_grad = false;
    std::shared_ptr<GradFunction> grad_fn;

    // view over the same storage (used by transpose / reshape)
    Tensor view(const std::vector<int64_t>& sizes, const std::vector<int64_t>& strides,
                int64_t offset) const;

  private:
    std::shared_ptr<Storage> data_;
    std::vector<int64_t> sizes_;
    std::vector<int64_t> strides_;
    int64_t numel_ = 0;
    int64_t offset_ = 0;
    std::shared_ptr<Tensor> grad_;
};

std::ostream& operator<<(std::ostream& os, const Tensor& t);

}  // namespace tl
