// internal.h — launchers shared between the translation units of libw4a8_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace w4a8 {

// row_limit (optional, device): rows at or past row_limit[0] are skipped.
int launch_act_quant(const void* x, uint8_t* xq, float* scales, int64_t M, int64_t K,
                     cudaStream_t stream, const int32_t* row_limit = nullptr);

}  // namespace w4a8
