// Compat shim -- TEST INFRASTRUCTURE ONLY.
//
// oracle/Makefile (target `compat`) puts oracle/compat first on the include
// path of exactly two unmodified reference sources, src/model/qwen2_model.cpp
// and src/model/llama_model.cpp.  Their `#include
// "smallm/backend/cpu_backend.h"` then finds this file, and their
// `backend_(std::make_unique<CPUBackend>())` (qwen2_model.cpp:31,
// llama_model.cpp:21) constructs the B200 CUDABackend: the engine's own
// forward pass running on the per-op Backend boundary, no reference line
// edited.  Every other reference source is compiled with its real
// cpu_backend.h.
#pragma once

#include "smallm/backend/cuda_backend.h"

namespace smallm {
using CPUBackend = CUDABackend;
}  // namespace smallm
