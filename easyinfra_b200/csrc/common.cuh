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

// Upper bound on a persistent grouped-GEMM grid: the SM count, or fewer CTAs when
// B200MOE_GEMM_MAX_CTAS is set (a test knob: a small grid makes every CTA walk many
// tiles, the regime of prefill-sized launches, on inputs the checker handles quickly).
int gemm_grid_limit();

// Programmatic dependent launch on/off (B200MOE_PDL=0 turns it off).
bool pdl_enabled();

// Launch `kern` on `stream`, with programmatic stream serialization when enabled.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace b200moe
