// One token row of the block prologue (residual add + RMSNorm) for a 256-thread CTA.
// Shared by the prologue kernel (norm.cu) and the fused small-batch router
// (router.cu) so both produce the same bits: the same thread -> element mapping, the
// same per-thread accumulation order and the same fixed-order block reduction.
//
// Mirrors MoeAll2AllBlock.all2all_chunk_routing_compute's first two steps
// (easyinfra/generation/blocks/moe/moe_all2all.py:331-335):
//   residual = residual + hidden                      (_add_to_residual, compute_utils.py)
//   normed   = weight * (residual_f32 * rsqrt(mean(residual_f32^2) + eps)).to(dtype)
//                                                     (_rmsnorm, rmsnorm/base_rmsnorm.py:6-12)
// with the reference's rounding points: the sum is rounded to the activation dtype,
// the normalisation runs in fp32 and is rounded before the weight multiply, whose
// product is rounded again.
#pragma once

#include "kernels.cuh"

namespace b200moe {

template <typename E>
__device__ __forceinline__ float to_f(E v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

template <typename E>
__device__ __forceinline__ E from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }

// Each thread holds up to NORM_MAXV 16-byte vectors of the row in registers between
// the two passes; the sum of squares is reduced across the CTA.
constexpr int NORM_THREADS = 256;
constexpr int NORM_MAXV = 8;   // rows up to 256 * 8 * 16 B = 32 KB (H <= 16384 bf16)

// Row t: residual_out[t] = round(residual[t] + hidden[t]) when rout != null; the normed
// row goes to every non-null destination among nout_a / nout_b (row pointers).
// red: 8 floats of shared memory.  Must be called by all 256 threads.
template <typename E>
__device__ __forceinline__ void add_rmsnorm_row(const AddNormParams& p, int64_t t, E* rout, E* nout_a,
                                                E* nout_b, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const E* res = static_cast<const E*>(p.residual) + t * p.ld;
  const E* hid = p.hidden ? static_cast<const E*>(p.hidden) + t * p.ld : nullptr;
  constexpr int V = 16 / sizeof(E);  // elements per 16-byte vector
  const int nvec = p.H / V;
  uint4 keep[NORM_MAXV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NORM_MAXV; ++i) {
    const int vi = threadIdx.x + i * NORM_THREADS;
    if (vi < nvec) {
      const uint4 a = *reinterpret_cast<const uint4*>(res + vi * V);
      uint4 o = a;
      E* oe = reinterpret_cast<E*>(&o);
      if (hid) {
        const uint4 b = *reinterpret_cast<const uint4*>(hid + vi * V);
        const E* ae = reinterpret_cast<const E*>(&a);
        const E* be = reinterpret_cast<const E*>(&b);
#pragma unroll
        for (int j = 0; j < V; ++j) oe[j] = from_f<E>(to_f<E>(ae[j]) + to_f<E>(be[j]));
      }
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float f = to_f<E>(oe[j]);
        ss = fmaf(f, f, ss);
      }
      if (rout) *reinterpret_cast<uint4*>(rout + vi * V) = o;
      keep[i] = o;
    }
  }
  if (nout_a == nullptr && nout_b == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int q = 0; q < NORM_THREADS / 32; ++q) tot += red[q];
  __syncthreads();  // red is reused by the next row
  const float inv = rsqrtf(tot / static_cast<float>(p.H) + p.eps);
  const E* w = static_cast<const E*>(p.weight);
#pragma unroll
  for (int i = 0; i < NORM_MAXV; ++i) {
    const int vi = threadIdx.x + i * NORM_THREADS;
    if (vi < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * V);
      const E* ae = reinterpret_cast<const E*>(&keep[i]);
      const E* we = reinterpret_cast<const E*>(&wv);
      uint4 o;
      E* oe = reinterpret_cast<E*>(&o);
#pragma unroll
      for (int j = 0; j < V; ++j) oe[j] = from_f<E>(to_f<E>(we[j]) * to_f<E>(from_f<E>(to_f<E>(ae[j]) * inv)));
      if (nout_a) *reinterpret_cast<uint4*>(nout_a + vi * V) = o;
      if (nout_b) *reinterpret_cast<uint4*>(nout_b + vi * V) = o;
    }
  }
}

}  // namespace b200moe
