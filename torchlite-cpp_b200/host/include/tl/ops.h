// The matmul path of tl:: (include/tl/ops.h:24-35 of torchlite-cpp), on the GPU.
#pragma once

#include <tl/tensor.h>

#include <cstdint>
#include <vector>

struct tlc_group;  // a libtl_cuda device group (include/tlc.h)

namespace tl {

// matrix multiplication: out = a @ b, NumPy batch broadcasting, 1-D squeeze
// (src/ops.cpp:605-699).  Runs in libtl_cuda's GEMM in the process default
// mode (environment variable TL_GEMM_MODE: exact | tf32 | 3xtf32; exact,
// bit-identical to the reference, if unset).  Throws std::invalid_argument
// with the reference's messages.
// With TL_NUM_GPUS = n > 1 in the environment, products of at least
// 2^20 output elements (and their MatmulBackward) run over GPUs 0..n-1 of the
// box through one device group (tlc_group_*): operands whose only current
// copy is on the host are copied in by every GPU for its share and the result
// is left on the host; device-resident operands are split from device 0 and
// the result gathered there.  The results are the single-GPU ones bit for
// bit (no product's additions are split across GPUs).
Tensor matmul(const Tensor& a_in, const Tensor& b_in);
// The device group TL_NUM_GPUS selects (NULL when it is unset or 1).
::tlc_group* multi_gpu_group();
// the same with an explicit mode (TLC_MODE_EXACT / _TF32 / _3XTF32)
Tensor matmul(const Tensor& a_in, const Tensor& b_in, int mode);

// matrix transpose: a view with two dims swapped (src/ops.cpp:702-730)
Tensor transpose(const Tensor& a, int64_t dim0, int64_t dim1);
// tensor reshape: a view when contiguous, else a copy (src/ops.cpp:732-767)
Tensor reshape(const Tensor& a, const std::vector<int64_t>& new_sizes);
Tensor unsqueeze(const Tensor& input, int64_t dim);
Tensor squeeze(const Tensor& input, int64_t dim);

// element-wise addition with NumPy broadcasting (src/ops.cpp:74-103)
Tensor add(const Tensor& a, const Tensor& b);
// scale a tensor by a factor (src/ops.cpp:963-983)
Tensor scale(const Tensor& input, float scalar);
// softmax over the last dim (src/ops.cpp:985-1037); CUDA's expf, so a few
// ulp from the reference; its backward is bit-identical
Tensor softmax(const Tensor& input);
// reduce a gradient to a broadcast input's shape (sum_to, src/autograd.cpp:24-36)
Tensor sum_to(const Tensor& grad, const std::vector<int64_t>& target_shape);

// Fused forms of the reference's call sequences, same results and gradients:
//   matmul_add(x, w, b)   == add(matmul(x, w), b)        (Linear::forward, src/nn.cpp:77-83)
//   matmul_scale(q, k, s) == scale(matmul(q, k), s)      (MultiHeadAttention, src/nn.cpp:423-424)
// The bias add / scale run in the GEMM's epilogue; b is 1-D of length N.
Tensor matmul_add(const Tensor& a, const Tensor& b, const Tensor& bias);
Tensor matmul_scale(const Tensor& a, const Tensor& b, float scalar);

// 2-D convolution of NCHW tensors (src/ops.cpp:1443-1548): im2col + one
// batched GEMM on the GPU; bias empty or [C_out].  Throws the reference's
// std::invalid_argument messages.
Tensor conv2d(const Tensor& input, const Tensor& weight, const Tensor& bias, int64_t stride = 1,
              int64_t padding = 0, int64_t groups = 1);
// flash attention (src/ops.cpp:1040-1137): out = softmax(Q . K^T * sm_scale) . V
// for [S, d] tensors (or [..., S, d], one head per leading index), d <= 128:
// one fused device kernel with the reference's 64 x 64 tiles and online
// softmax; FlashAttentionBackward in the process default GEMM mode.  Agrees
// with the reference to its own 1e-4 bar (CUDA's expf / logf).
Tensor flash_attention(const Tensor& Q, const Tensor& K, const Tensor& V, float sm_scale);
// sum along a dimension (src/ops.cpp:1181-1233); no autograd node
Tensor sum(const Tensor& input, int64_t dim, bool keepdim = false);

// factories (src/factory.cpp)
Tensor zeros(const std::vector<int64_t>& sizes);
Tensor ones(const std::vector<int64_t>& sizes);
Tensor full(const std::vector<int64_t>& sizes, float value);

}  // namespace tl
