// The MoE block's stage-1 prologue in one pass: residual add + RMSNorm.
//
// Mirrors MoeAll2AllBlock.all2all_chunk_routing_compute's first two steps
// (easyinfra/generation/blocks/moe/moe_all2all.py:331-335):
//   residual = residual + hidden                      (_add_to_residual, compute_utils.py)
//   normed   = weight * (residual_f32 * rsqrt(mean(residual_f32^2) + eps)).to(dtype)
//                                                     (_rmsnorm, rmsnorm/base_rmsnorm.py:6-12)
// with the reference's rounding points: the sum is rounded to the activation dtype,
// the normalisation runs in fp32 and is rounded before the weight multiply, whose
// product is rounded again.  One CTA per token; the row is read once from HBM and
// kept in registers for the second pass.
#include "norm_row.cuh"

namespace b200moe {

// One CTA per token; the row is read once from HBM and kept in registers for the
// second pass (add_rmsnorm_row, norm_row.cuh).
template <typename E>
__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(const __grid_constant__ AddNormParams p) {
  __shared__ float red[NORM_THREADS / 32];
  pdl_trigger();
  // the norm weight toward L2 before the wait (one CTA: L2 is shared by all)
  if (blockIdx.x == 0) prefetch_l2_lines(p.weight, static_cast<int64_t>(p.H) * sizeof(E));
  pdl_wait();
  const int64_t t = blockIdx.x;
  E* rout = static_cast<E*>(p.residual_out) + t * p.ld;
  E* nout = p.normed ? static_cast<E*>(p.normed) + t * p.ld_normed : nullptr;
  add_rmsnorm_row<E>(p, t, rout, nout, nullptr, red);
}

int launch_add_rmsnorm(const AddNormParams& p, cudaStream_t stream) {
  if (p.T == 0) return 0;
  const int vec = 16 / (p.dtype == kDtypeBF16 ? 2 : 4);
  if (p.H / vec > NORM_THREADS * NORM_MAXV) return -1;
  if (p.dtype == kDtypeBF16)
    launch_kernel(add_rmsnorm_kernel<__nv_bfloat16>, dim3(p.T), dim3(NORM_THREADS), 0, stream, p);
  else
    launch_kernel(add_rmsnorm_kernel<float>, dim3(p.T), dim3(NORM_THREADS), 0, stream, p);
  return 0;
}

}  // namespace b200moe
