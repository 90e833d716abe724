// fp32 grouped expert GEMMs (SwiGLU gate/up and down) for fp32 models.
//
// Same contract as the bf16 tcgen05 kernels (grouped_gemm.cu) — rows of expert e are
// [off[e], off[e+1]) of A, weights stacked [P, w_rows, K], SwiGLU fused, optional
// output row map — on CUDA cores in fp32 (the reference's fp32 eager path,
// NativeMoE.forward_ep, easyinfra/generation/modules/moe/native_moe.py:56-103, runs
// fp32 matmuls; tensor cores would round the inputs).  Used for the fp32
// configuration; the bf16 kernels carry the large models.
//
// 64 x 64 output tiles, 256 threads, 4 x 4 outputs per thread (4 x 4 gate + 4 x 4 up
// for SwiGLU), K staged through shared memory 16 at a time.  Grid y walks the m-tiles
// of all experts; each CTA finds its expert by scanning the row offsets.
#include "kernels.cuh"

namespace b200moe {

constexpr int F32_TM = 64, F32_TN = 64, F32_TK = 16;

template <bool SWIGLU>
__global__ void __launch_bounds__(256) grouped_gemm_f32_kernel(GemmF32Params p) {
  __shared__ float As[F32_TK][F32_TM + 4];
  __shared__ float Bs[F32_TK][F32_TN + 4];
  __shared__ float Us[SWIGLU ? F32_TK : 1][F32_TN + 4];
  __shared__ int s_e, s_m0;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    // m-tile blockIdx.y -> (expert, first row)
    int tile = blockIdx.y, e = -1, m0 = 0;
    for (int q = 0; q < p.P; ++q) {
      const int rows = p.offsets[q + 1] - p.offsets[q];
      const int mt = (rows + F32_TM - 1) / F32_TM;
      if (tile < mt) { e = q; m0 = tile * F32_TM; break; }
      tile -= mt;
    }
    s_e = e;
    s_m0 = m0;
  }
  __syncthreads();
  const int e = s_e;
  if (e < 0) return;
  const int row_base = p.offsets[e];
  const int rows = p.offsets[e + 1] - row_base;
  const int m0 = s_m0;
  const int n0 = blockIdx.x * F32_TN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const float* Wg = p.w + (static_cast<int64_t>(e) * p.w_rows) * p.K;
  float acc[4][4] = {}, accu[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += F32_TK) {
    for (int i = threadIdx.x; i < F32_TM * F32_TK; i += 256) {
      const int r = i / F32_TK, k = i % F32_TK;
      const int gr = m0 + r, gk = k0 + k;
      As[k][r] = (gr < rows && gk < p.K) ? p.a[(static_cast<int64_t>(row_base) + gr) * p.lda + gk] : 0.f;
      const int gn = n0 + r;
      Bs[k][r] = (gn < p.N && gk < p.K) ? Wg[static_cast<int64_t>(gn) * p.K + gk] : 0.f;
      if (SWIGLU) Us[k][r] = (gn < p.N && gk < p.K) ? Wg[static_cast<int64_t>(p.up_row + gn) * p.K + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < F32_TK; ++k) {
      float a[4], b[4], u[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[k][ty * 4 + i];
        b[i] = Bs[k][tx * 4 + i];
        if (SWIGLU) u[i] = Us[k][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          if (SWIGLU) accu[i][j] = fmaf(a[i], u[j], accu[i][j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = m0 + ty * 4 + i;
    if (r >= rows) continue;
    int64_t orow = row_base + r;
    if (p.out_row_map) orow = p.out_row_map[orow];
    float* o = p.out + orow * p.ldo;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tx * 4 + j;
      if (c >= p.N) continue;
      const float g = acc[i][j];
      o[c] = SWIGLU ? g / (1.f + expf(-g)) * accu[i][j] : g;
    }
  }
}

int launch_grouped_gemm_f32(const GemmF32Params& p, bool swiglu, cudaStream_t stream) {
  if (p.rows_cap == 0) return 0;
  dim3 grid((p.N + F32_TN - 1) / F32_TN, static_cast<unsigned>((p.rows_cap + F32_TM - 1) / F32_TM + p.P));
  if (swiglu)
    launch_kernel(grouped_gemm_f32_kernel<true>, grid, dim3(256), 0, stream, p);
  else
    launch_kernel(grouped_gemm_f32_kernel<false>, grid, dim3(256), 0, stream, p);
  return 0;
}

}  // namespace b200moe
