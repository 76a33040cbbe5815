// The matmul path of tl:: (include/tl/ops.h:24-35 of torchlite-cpp), on the GPU.
#pragma once

#include <tl/tensor.h>

#include <cstdint>
#include <vector>

namespace tl {

// matrix multiplication: out = a @ b, NumPy batch broadcasting, 1-D squeeze
// (src/ops.cpp:605-699).  Runs in libtl_cuda's GEMM in the process default
// mode (environment variable TL_GEMM_MODE: exact | tf32 | 3xtf32; exact,
// bit-identical to the reference, if unset).  Throws std::invalid_argument
// with the reference's messages.
Tensor matmul(const Tensor& a_in, const Tensor& b_in);
// the same with an explicit mode (TLC_MODE_EXACT / _TF32 / _3XTF32)
Tensor matmul(const Tensor& a_in, const Tensor& b_in, int mode);

// matrix transpose: a view with two dims swapped (src/ops.cpp:702-730)
Tensor transpose(const Tensor& a, int64_t dim0, int64_t dim1);
// tensor reshape: a view when contiguous, else a copy (src/ops.cpp:732-767)
Tensor reshape(const Tensor& a, const std::vector<int64_t>& new_sizes);
Tensor unsqueeze(const Tensor& input, int64_t dim);
Tensor squeeze(const Tensor& input, int64_t dim);

// element-wise addition of same-shape tensors (src/ops.cpp:75-103, no broadcast)
Tensor add(const Tensor& a, const Tensor& b);
// sum along a dimension (src/ops.cpp:1181-1233); no autograd node
Tensor sum(const Tensor& input, int64_t dim, bool keepdim = false);

// factories (src/factory.cpp)
Tensor zeros(const std::vector<int64_t>& sizes);
Tensor ones(const std::vector<int64_t>& sizes);
Tensor full(const std::vector<int64_t>& sizes, float value);

}  // namespace tl
