// Shared declarations for the b200moe kernels and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ptx.cuh"

namespace b200moe {

enum Dtype : int { kDtypeBF16 = 0, kDtypeF32 = 1 };

inline int dtype_bytes(int dt) { return dt == kDtypeBF16 ? 2 : 4; }

// Multiprocessor count of the current device (cached per device).
int num_sms();

}  // namespace b200moe
