// TLMD model files (include/tl/model_io.h of torchlite-cpp) for the device
// tl:: layer: the same file format and checks, with tensor data streamed
// straight between the file and device memory (tlc_load_tlmd / tlc_save_tlmd).
#pragma once

#include <tl/tensor.h>

#include <string>
#include <vector>

namespace tl {

// src/model_io.cpp:22-44; throws std::runtime_error with the reference's texts
void save_model(const std::string& path, const std::vector<Tensor*>& params);
// src/model_io.cpp:46-94: loads into the parameters' device storage
void load_model(const std::string& path, const std::vector<Tensor*>& params);

}  // namespace tl
