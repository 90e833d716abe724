// Kernel family (1): the MoE router.
//
// Mirrors the reference's routing for one chunk of tokens:
//   logits = F.linear(x, W_gate, b_gate)            (Qwen3MoeSparseMoeBlock._routing,
//   p      = softmax(logits, dtype=float32)          easyinfra/models/qwen3_moe/
//   w, e   = topk(p, K)                               modeling_qwen3_moe.py:255-266)
//   if norm_topk_prob: w = w / w.sum(-1)
//   w      = w.to(x.dtype)
// followed by the EPLB replica pick
//   phys = log2phy[e][(t*K + k) % replica_count[e]]  (blocks/moe/base.py:40-64)
// and the per-slot token histogram (blocks/moe/base.py:343-364).
//
// Kernels (a logits kernel, then the selection; one fused launch up to 8 tokens):
//   router_logits_bf16  T > 256: one warp per 16 tokens, mma.sync m16n8k16 bf16 ->
//                       fp32 on a cp.async ring; logits rounded to bf16 exactly like
//                       F.linear's bf16 output.
//   router_logits_gemv  T <= 256: one CTA per (8 tokens, router column), fixed-order
//                       reduction; router_logits_gemv_cols, the same reduction for a
//                       group of columns per CTA with the token rows in registers, once
//                       there are enough token groups to fill the SMs.
//   router_logits_f32   SIMT fp32 dot products (fp32 activations).
//   router_select       one warp per token: fp32 softmax, top-k with ties broken to
//                       the lowest expert index (warp reductions), renorm, scaling,
//                       dtype rounding, replica pick, per-block slot histogram; the
//                       last CTA to finish turns the histograms into slot counts,
//                       slot offsets and per-(slot, block) write offsets for the
//                       permute kernel.
//   router_small_fused  T <= 8: optional residual add + RMSNorm, the GEMV logits and
//                       the selection in one launch, with the bits of the kernels above;
//                       optionally also the permute (send rows straight from the rows
//                       the CTA holds in shared memory).
#include <cstdlib>

#include <atomic>

#include "kernels.cuh"
#include "norm_row.cuh"

namespace b200moe {

// ------------------------------------------------------------------ logits (bf16)
// CTA = 4 warps, 64 tokens.  Chunks of 64 hidden elements of x and of the CTA's W_gate
// rows stream through a RL_STAGES-deep cp.async ring in shared memory (padded row
// stride), so the HBM reads of later chunks overlap the MMAs of the current one; each
// warp owns 16 tokens and every 8-expert column tile (mma.sync m16n8k16, fp32 acc).
constexpr int RL_TOK = 64;
constexpr int RL_HC = 64;        // hidden elements per chunk
constexpr int RL_LD = RL_HC + 8; // padded smem row (bf16 elements)
constexpr int RL_MAXNT = 17;     // up to 136 logit columns per pass

// RL_STAGES chunks in flight: 8 for narrow column groups (few router columns: the
// kernel is a pure stream over x and needs the most bytes in flight), 4 otherwise.
// NT: compile-time bound on the CTA's 8-column tiles, so a router with few experts
// issues only the MMAs it needs.
template <int RL_STAGES, int NT>
__global__ void __launch_bounds__(128) router_logits_bf16(const __grid_constant__ RouterLogitsParams p,
                                                          int cols_per_cta) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  pdl_trigger();
  pdl_wait();

  const int col0 = blockIdx.y * cols_per_cta;
  const int ncols = min(cols_per_cta, p.E1 - col0);
  const int nt = (ncols + 7) / 8;
  const int ncols_pad = nt * 8;
  const int stage_elems = (RL_TOK + cols_per_cta) * RL_LD;
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * RL_TOK;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x);
  const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(p.w);
  const int nchunks = (p.H + RL_HC - 1) / RL_HC;

  auto load_chunk = [&](int c) {
    __nv_bfloat16* xs = ring + (c % RL_STAGES) * stage_elems;
    __nv_bfloat16* ws = xs + RL_TOK * RL_LD;
    const int h0 = c * RL_HC;
    for (int i = threadIdx.x; i < RL_TOK * 8; i += 128) {
      const int r = i >> 3, cc = (i & 7) * 8;
      const int t = tok0 + r;
      const bool ok = t < p.T && h0 + cc < p.H;
      cp_async_16(xs + r * RL_LD + cc, ok ? x + static_cast<int64_t>(t) * p.ldx + h0 + cc : x, ok);
    }
    for (int i = threadIdx.x; i < ncols_pad * 8; i += 128) {
      const int r = i >> 3, cc = (i & 7) * 8;
      const bool ok = r < ncols && h0 + cc < p.H;
      cp_async_16(ws + r * RL_LD + cc, ok ? w + static_cast<int64_t>(col0 + r) * p.H + h0 + cc : w, ok);
    }
  };

  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

#pragma unroll
  for (int c = 0; c < RL_STAGES - 1; ++c) {
    if (c < nchunks) load_chunk(c);
    cp_async_commit();
  }
  const int ar = warp * 16 + (lane >> 2);
  const int ac = (lane & 3) * 2;
  for (int c = 0; c < nchunks; ++c) {
    cp_async_wait<RL_STAGES - 2>();  // chunk c has landed (this thread's copies)
    __syncthreads();                 // ... and everyone's; chunk c-1's stage is free
    const __nv_bfloat16* xs = ring + (c % RL_STAGES) * stage_elems;
    const __nv_bfloat16* ws = xs + RL_TOK * RL_LD;
#pragma unroll
    for (int k0 = 0; k0 < RL_HC; k0 += 16) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(xs + ar * RL_LD + k0 + ac);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(xs + (ar + 8) * RL_LD + k0 + ac);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(xs + ar * RL_LD + k0 + ac + 8);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(xs + (ar + 8) * RL_LD + k0 + ac + 8);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        if (j < nt) {
          const int bn = j * 8 + (lane >> 2);
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(ws + bn * RL_LD + k0 + ac);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(ws + bn * RL_LD + k0 + ac + 8);
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
              "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
              : "+f"(acc[j][0]), "+f"(acc[j][1]), "+f"(acc[j][2]), "+f"(acc[j][3])
              : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
        }
      }
    }
    const int nc = c + RL_STAGES - 1;
    if (nc < nchunks) load_chunk(nc);
    cp_async_commit();
  }
  cp_async_wait<0>();
  // C fragment: c0,c1 -> (row lane/4, cols 2*(lane%4)+{0,1}); c2,c3 -> row + 8.
  const int r0 = tok0 + warp * 16 + (lane >> 2);
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    if (j < nt) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = r0 + (q >> 1) * 8;
        const int col = j * 8 + (lane & 3) * 2 + (q & 1);
        if (row < p.T && col < ncols) {
          float v = acc[j][q];
          if (p.bias) v += p.bias[col0 + col];
          p.logits[static_cast<int64_t>(row) * p.E1 + col0 + col] = p.round_bf16 ? bf16_round(v) : v;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ logits (small T)
// Decode-sized batches: one CTA per (router column, group of RG tokens); its 256
// threads stride over the hidden dimension with 16-byte loads (the weight row is
// read once per group), keep RG partial dot products in registers, and reduce them
// through shared memory in a fixed order (deterministic, no atomics).
constexpr int RG = 8;

template <typename E>
__global__ void __launch_bounds__(256) router_logits_gemv(RouterLogitsParams p) {
  __shared__ float red[8][RG];
  pdl_trigger();
  if (blockIdx.x == 0)  // this column's router row toward L2 before the wait (once per column)
    prefetch_l2_lines(static_cast<const E*>(p.w) + static_cast<int64_t>(blockIdx.y) * p.H,
                      static_cast<int64_t>(p.H) * sizeof(E));
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.y, t0 = blockIdx.x * RG;
  const int nt = min(RG, p.T - t0);
  constexpr int V = 16 / sizeof(E);
  const E* w = static_cast<const E*>(p.w) + static_cast<int64_t>(e) * p.H;
  const E* x = static_cast<const E*>(p.x) + static_cast<int64_t>(t0) * p.ldx;
  float acc[RG];
#pragma unroll
  for (int i = 0; i < RG; ++i) acc[i] = 0.f;
  for (int c = threadIdx.x * V; c < p.H; c += 256 * V) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + c));
    uint4 xv[RG];
#pragma unroll
    for (int i = 0; i < RG; ++i)
      xv[i] = (i < nt) ? __ldg(reinterpret_cast<const uint4*>(x + i * p.ldx + c)) : make_uint4(0, 0, 0, 0);
    const E* we = reinterpret_cast<const E*>(&wv);
#pragma unroll
    for (int i = 0; i < RG; ++i) {
      const E* xe = reinterpret_cast<const E*>(&xv[i]);
#pragma unroll
      for (int j = 0; j < V; ++j) acc[i] = fmaf(static_cast<float>(xe[j]), static_cast<float>(we[j]), acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < RG; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < RG; ++i) red[warp][i] = acc[i];
  }
  __syncthreads();
  if (threadIdx.x < nt) {
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) v += red[q][threadIdx.x];
    if (p.bias) v += p.bias[e];
    if (sizeof(E) == 2 && p.round_bf16) v = bf16_round(v);
    p.logits[static_cast<int64_t>(t0 + threadIdx.x) * p.E1 + e] = v;
  }
}

// Decode batches of 9-256 tokens: one CTA per (RG tokens, CG router columns).  The
// CTA's token rows are held in registers (NX 16-byte vectors per token and thread,
// H == NX * 256 * V) and reused for its CG columns, so x is read from L2 once per
// column group instead of once per column.  Every column is reduced exactly like
// router_logits_gemv (same per-thread order, same shuffle tree, same fixed cross-warp
// order): the logits are bit-identical to that kernel's for every CG.
template <typename E, int NX, int CG>
__global__ void __launch_bounds__(256) router_logits_gemv_cols(RouterLogitsParams p) {
  __shared__ float red[CG][8][RG];
  pdl_trigger();
  const int col0 = blockIdx.y * CG;
  const int ncols = min(CG, p.E1 - col0);
  if (blockIdx.x == 0)  // this CTA's router rows toward L2 before the wait (once per column group)
    prefetch_l2_lines(static_cast<const E*>(p.w) + static_cast<int64_t>(col0) * p.H,
                      static_cast<int64_t>(ncols) * p.H * sizeof(E));
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * RG;
  const int nt = min(RG, p.T - t0);
  constexpr int V = 16 / sizeof(E);
  const E* x = static_cast<const E*>(p.x) + static_cast<int64_t>(t0) * p.ldx;
  // the token rows in fp32, converted once for all of the CTA's columns (exact)
  float xf[NX][RG][V];
#pragma unroll
  for (int j = 0; j < NX; ++j) {
    const int c = (threadIdx.x + j * 256) * V;
#pragma unroll
    for (int i = 0; i < RG; ++i) {
      const uint4 u = (i < nt) ? __ldg(reinterpret_cast<const uint4*>(x + i * p.ldx + c)) : make_uint4(0, 0, 0, 0);
      const E* ue = reinterpret_cast<const E*>(&u);
#pragma unroll
      for (int q = 0; q < V; ++q) xf[j][i][q] = static_cast<float>(ue[q]);
    }
  }
  const E* wbase = static_cast<const E*>(p.w) + static_cast<int64_t>(col0) * p.H;
  uint4 wv[NX];
#pragma unroll
  for (int j = 0; j < NX; ++j) wv[j] = __ldg(reinterpret_cast<const uint4*>(wbase + (threadIdx.x + j * 256) * V));
#pragma unroll 1
  for (int cc = 0; cc < ncols; ++cc) {
    uint4 wn[NX];  // next column's weights, loaded before this column's arithmetic
    if (cc + 1 < ncols) {
#pragma unroll
      for (int j = 0; j < NX; ++j)
        wn[j] = __ldg(reinterpret_cast<const uint4*>(wbase + static_cast<int64_t>(cc + 1) * p.H +
                                                     (threadIdx.x + j * 256) * V));
    }
    float acc[RG];
#pragma unroll
    for (int i = 0; i < RG; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < NX; ++j) {
      const E* we = reinterpret_cast<const E*>(&wv[j]);
      float wf[V];
#pragma unroll
      for (int q = 0; q < V; ++q) wf[q] = static_cast<float>(we[q]);
#pragma unroll
      for (int i = 0; i < RG; ++i) {
#pragma unroll
        for (int q = 0; q < V; ++q) acc[i] = fmaf(xf[j][i][q], wf[q], acc[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < RG; ++i) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < RG; ++i) red[cc][warp][i] = acc[i];
    }
    if (cc + 1 < ncols) {
#pragma unroll
      for (int j = 0; j < NX; ++j) wv[j] = wn[j];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < ncols * RG; idx += blockDim.x) {
    const int cc = idx / RG, i = idx - cc * RG;
    if (i >= nt) continue;
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) v += red[cc][q][i];
    const int e = col0 + cc;
    if (p.bias) v += p.bias[e];
    if (sizeof(E) == 2 && p.round_bf16) v = bf16_round(v);
    p.logits[static_cast<int64_t>(t0 + i) * p.E1 + e] = v;
  }
}

// ------------------------------------------------------------------ logits (fp32)
// One warp per token; lanes stride over the hidden dimension; 8 experts per pass.
__global__ void __launch_bounds__(256) router_logits_f32(RouterLogitsParams p) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= p.T) return;
  const float* x = static_cast<const float*>(p.x) + warp * p.ldx;
  const float* w = static_cast<const float*>(p.w);
  for (int e0 = 0; e0 < p.E1; e0 += 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int h = lane; h < p.H; h += 32) {
      const float xv = x[h];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (e0 + j < p.E1) acc[j] = fmaf(xv, w[static_cast<int64_t>(e0 + j) * p.H + h], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane < 8 && e0 + lane < p.E1) {
      float v = acc[0];
#pragma unroll
      for (int j = 1; j < 8; ++j)
        if (lane == j) v = acc[j];
      if (p.bias) v += p.bias[e0 + lane];
      p.logits[static_cast<int64_t>(warp) * p.E1 + e0 + lane] = v;
    }
  }
}

// ------------------------------------------------------------------ selection
constexpr int RS_MAXJ = 8;  // up to 256 routed experts

__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Unsigned key with the order of the float (-0 taken as +0): key(a) > key(b) <=> a > b.
__device__ __forceinline__ uint32_t order_key(float v) {
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Warp-wide maximum of a float (redux.sync, sm_100a); exact, so order-independent.
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// One warp per token of [t_begin, t_end): selection, weights, replica pick and the
// CTA's slot histogram (hist, shared, zeroed by the caller; the scoring-1 scratch
// follows it).  Shared by router_select and the fused small-batch router.  NJ =
// ceil(E / 32) experts per lane (compile time, so loops cover only live experts); the
// next token's logits are loaded before the current token is processed.
template <int NJ>
__device__ __forceinline__ void select_tokens(const RouterSelectParams& p, int t_begin, int t_end,
                                              int32_t* hist) {
  float* cbuf = reinterpret_cast<float*>(hist + p.num_slots) + (threadIdx.x >> 5) * 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int step = blockDim.x >> 5;
  float nxt[NJ];
  auto load_logits = [&](int t) {
    const float* lg = p.logits + static_cast<int64_t>(t) * p.E1;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int e = lane + 32 * j;
      nxt[j] = (e < p.E) ? lg[e] : -INFINITY;
    }
  };
  if (t_begin + warp < t_end) load_logits(t_begin + warp);
  for (int t = t_begin + warp; t < t_end; t += step) {
    const float* lg = p.logits + static_cast<int64_t>(t) * p.E1;
    float v[NJ];     // selection key per owned expert
    float sc[NJ];    // value reported as the routing weight (before renorm)
#pragma unroll
    for (int j = 0; j < NJ; ++j) v[j] = nxt[j];
    if (t + step < t_end) load_logits(t + step);
    if (p.scoring == 0) {
      // softmax over the experts (fp32), select on the probabilities
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < NJ; ++j) m = fmaxf(m, v[j]);
      m = warp_max_f32(m);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        v[j] = (e < p.E) ? expf(v[j] - m) : 0.f;
        s += v[j];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        v[j] = (lane + 32 * j < p.E) ? v[j] / s : -1.f;
        sc[j] = v[j];
      }
    } else {
      // sigmoid scores; choice = score + correction bias; keep the topk_group groups
      // with the largest sum of their two best choices; others' choices become 0.0
      const int gs = p.E / p.n_group;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if (e < p.E) {
          sc[j] = 1.f / (1.f + expf(-v[j]));
          v[j] = sc[j] + p.correction_bias[e];
          cbuf[e] = v[j];
        } else {
          sc[j] = 0.f;
          v[j] = -INFINITY;
        }
      }
      __syncwarp();
      float gsum = -INFINITY;
      if (lane < p.n_group) {
        float b1 = -INFINITY, b2 = -INFINITY;
        for (int q = 0; q < gs; ++q) {
          const float c = cbuf[lane * gs + q];
          if (c > b1) { b2 = b1; b1 = c; } else if (c > b2) { b2 = c; }
        }
        gsum = b1 + b2;
      }
      uint32_t keep = 0;
      for (int r = 0; r < p.topk_group; ++r) {
        float bv = ((keep >> lane) & 1u) ? -INFINITY : gsum;
        int bi = (lane < p.n_group && !((keep >> lane) & 1u)) ? lane : 0x7fffffff;
        if (bi == 0x7fffffff) bv = -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (bi < 32) keep |= 1u << bi;
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if (e < p.E && !((keep >> (e / gs)) & 1u)) v[j] = 0.f;
      }
      __syncwarp();
    }

    // top-k: K rounds of a warp arg-max on (key desc, expert asc): each lane offers its
    // best untaken expert, one redux picks the largest key and a second the lowest
    // expert holding it; the winner's reported value (probability, or sigmoid score)
    // comes from its lane.  Lane k keeps round k's result.
    uint32_t taken = 0;
    float denom = 0.f, wk = 0.f;
    int ek = 0;
    for (int k = 0; k < p.K; ++k) {
      uint32_t bkey = 0;  // 0: no candidate (below the key of every float but NaN)
      int bj = -1;
      float bs = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if (e < p.E && !((taken >> j) & 1u)) {
          const uint32_t kj = order_key(v[j]);
          if (bj < 0 || kj > bkey) {  // strict: ties keep the lower expert
            bkey = kj;
            bj = j;
            bs = sc[j];
          }
        }
      }
      const uint32_t mkey = __reduce_max_sync(0xffffffffu, bkey);
      const uint32_t cand = (bj >= 0 && bkey == mkey) ? static_cast<uint32_t>(lane + 32 * bj) : 0xffffffffu;
      const int win = static_cast<int>(__reduce_min_sync(0xffffffffu, cand));
      const float ws = __shfl_sync(0xffffffffu, bs, win & 31);
      if ((win & 31) == lane) taken |= 1u << (win >> 5);
      if (k == lane) {
        wk = ws;
        ek = win;
      }
      denom += ws;
    }
    if (p.renorm) {
      if (p.scoring == 1) denom += 1e-20f;
    } else {
      denom = 1.f;
    }
    if (lane < p.K) {
      if (p.renorm) wk = wk / denom;
      wk *= p.scale;
      if (p.round_bf16) wk = bf16_round(wk);
      const int64_t flat = static_cast<int64_t>(t) * p.K + lane;
      int phys = ek;
      if (p.log2phy) {
        const int rc = p.rep_count[ek];
        const int r = (rc > 0) ? static_cast<int>(flat % rc) : 0;
        phys = p.log2phy[ek * p.max_rep + r];
      }
      if (phys < 0 || phys >= p.num_slots) {
        record_status(p.status, kStatusBadIndex);
        phys = 0;
      }
      p.topk_ids[flat] = ek;
      p.topk_w[flat] = wk;
      p.phys_ids[flat] = phys;
      atomicAdd(&hist[phys], 1);
    }
    if (p.has_shared_gate && lane == 0) {
      const float g = lg[p.E];
      p.shared_gate[t] = 1.f / (1.f + expf(-g));
    }
  }
}

// select_tokens for the expert count in p (NJ from E).
__device__ __forceinline__ void select_tokens_any(const RouterSelectParams& p, int t_begin, int t_end,
                                                  int32_t* hist) {
  if (p.E <= 32)
    select_tokens<1>(p, t_begin, t_end, hist);
  else if (p.E <= 64)
    select_tokens<2>(p, t_begin, t_end, hist);
  else if (p.E <= 128)
    select_tokens<4>(p, t_begin, t_end, hist);
  else
    select_tokens<RS_MAXJ>(p, t_begin, t_end, hist);
}

// Column pass of the last CTA over block_counts [num_slots][nb]: each slot's column
// becomes absolute write offsets (exclusive prefix from the slot offset in hist).  SB
// slots per warp iteration; a column is walked in chunks of 32 * PL blocks, each lane
// owning PL contiguous blocks of a chunk, with a carry between chunks.  Every load of a
// chunk is issued before any arithmetic, so a warp has SB * PL loads in flight.
template <int SB, int PL>
__device__ __forceinline__ void slot_columns(const RouterSelectParams& p, const int32_t* hist, int nb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int s0 = warp * SB; s0 < p.num_slots; s0 += nwarps * SB) {
    int carry[SB];
#pragma unroll
    for (int i = 0; i < SB; ++i) carry[i] = (s0 + i < p.num_slots) ? hist[s0 + i] : 0;
    for (int b0 = 0; b0 < nb; b0 += 32 * PL) {
      int v[SB][PL];
#pragma unroll
      for (int i = 0; i < SB; ++i) {
#pragma unroll
        for (int k = 0; k < PL; ++k) {
          const int b = b0 + lane * PL + k;
          v[i][k] = (b < nb && s0 + i < p.num_slots)
                        ? __ldcg(p.block_counts + static_cast<int64_t>(s0 + i) * nb + b)
                        : 0;
        }
      }
#pragma unroll
      for (int i = 0; i < SB; ++i) {
        int part = 0;
#pragma unroll
        for (int k = 0; k < PL; ++k) part += v[i][k];
        int incl = part;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int n = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += n;
        }
        if (s0 + i < p.num_slots) {
          int32_t* col = p.block_counts + static_cast<int64_t>(s0 + i) * nb;
          int run = carry[i] + incl - part;
#pragma unroll
          for (int k = 0; k < PL; ++k) {
            const int b = b0 + lane * PL + k;
            if (b < nb) {
              col[b] = run;
              run += v[i][k];
            }
          }
        }
        carry[i] += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
  }
}

__device__ __forceinline__ void slot_columns_any(const RouterSelectParams& p, const int32_t* hist, int nb) {
  if (nb <= 64)
    slot_columns<8, 2>(p, hist, nb);
  else
    slot_columns<2, 8>(p, hist, nb);  // chunks of 256 blocks
}

// Exclusive scan of the slot totals in hist (warp 0): writes slot_counts and
// slot_offsets; hist[] becomes the slot offsets.
__device__ __forceinline__ void scan_slot_totals(const RouterSelectParams& p, int32_t* hist) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp != 0) return;
  int run = 0;
  for (int base = 0; base < p.num_slots; base += 32) {
    const int s = base + lane;
    const int c = (s < p.num_slots) ? hist[s] : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (s < p.num_slots) {
      p.slot_counts[s] = c;
      p.slot_offsets[s] = run + incl - c;
      hist[s] = run + incl - c;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) p.slot_offsets[p.num_slots] = run;
}

// One token block (the fused small-batch router): its histogram in hist already holds
// the slot totals and its write offsets are the slot offsets — no round trip through
// block_counts.  Called by every thread after a __syncthreads.
__device__ __forceinline__ void select_finish_one_block(const RouterSelectParams& p, int32_t* hist) {
  scan_slot_totals(p, hist);
  __syncthreads();
  for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) p.block_counts[s] = hist[s];
  if (threadIdx.x == 0) *p.ticket = 0u;
}

// Up to this many token blocks the last CTA sums each slot's column itself (one load
// round trip); above it every CTA also adds its histogram into slot_totals.
constexpr int kSmallNb = 16;

// Run by every thread of the CTA that arrived last, once every CTA's histogram is in
// block_counts: slot totals, slot offsets, absolute per-(slot, block) offsets; resets
// the ticket (and slot_totals).  hist is shared scratch of num_slots ints.
__device__ __forceinline__ void select_finish(const RouterSelectParams& p, int32_t* hist) {
  // ---- last CTA: slot totals, slot offsets, absolute per-(slot, block) offsets.
  __threadfence();
  const int nb = p.nblocks;
  if (nb > kSmallNb) {
    // every CTA added its histogram into slot_totals: one round trip, then reset
    for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) {
      hist[s] = __ldcg(p.slot_totals + s);
      p.slot_totals[s] = 0;
    }
  } else {
    // few blocks (decode batches): one thread per slot, one round trip of loads
    for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) {
      const int32_t* col = p.block_counts + static_cast<int64_t>(s) * nb;
      int tot = 0;
#pragma unroll
      for (int b = 0; b < kSmallNb; ++b)
        if (b < nb) tot += __ldcg(col + b);
      hist[s] = tot;
    }
  }
  __syncthreads();
  scan_slot_totals(p, hist);
  __syncthreads();
  if (nb <= kSmallNb) {
    for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) {
      int32_t* col = p.block_counts + static_cast<int64_t>(s) * nb;
      int c[kSmallNb];
#pragma unroll
      for (int b = 0; b < kSmallNb; ++b) c[b] = (b < nb) ? __ldcg(col + b) : 0;
      int run = hist[s];
#pragma unroll
      for (int b = 0; b < kSmallNb; ++b)
        if (b < nb) {
          col[b] = run;
          run += c[b];
        }
    }
  } else {
    slot_columns_any(p, hist, nb);
  }
  if (threadIdx.x == 0) *p.ticket = 0u;
}

template <int NJ>
__global__ void __launch_bounds__(256, 4) router_select(const __grid_constant__ RouterSelectParams p) {
  extern __shared__ int32_t hist[];  // [num_slots], then (scoring 1) 8 warps x 256 floats
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) hist[s] = 0;
  __syncthreads();
  const int t_begin = blockIdx.x * p.tb;
  select_tokens<NJ>(p, t_begin, min(p.T, t_begin + p.tb), hist);
  __syncthreads();
  for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) {
    const int c = hist[s];
    p.block_counts[static_cast<int64_t>(s) * p.nblocks + blockIdx.x] = c;
    if (p.nblocks > kSmallNb && c != 0) atomicAdd(p.slot_totals + s, c);  // order-free integer sum
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.ticket, 1u) == static_cast<uint32_t>(p.nblocks - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  select_finish(p, hist);
}

// ------------------------------------------------------------------ fused small batch
// T <= RG tokens (decode): one CTA per router column computes that column's logits for
// every token — the GEMV of router_logits_gemv with the same thread mapping and
// reduction order, on token rows staged in shared memory — and the CTA that finishes
// last runs the selection for all tokens (select_tokens / select_finish, one token
// block).  With the block prologue fused in (has_norm), every CTA first builds the
// normed rows itself with add_rmsnorm_row (CTA 0 also writes residual_out and
// normed).  One launch replaces two (router) or three (prologue + router); the bits
// are those of the separate kernels.
constexpr size_t kFusedSmemMax = 160 * 1024;

template <typename E>
__global__ void __launch_bounds__(256) router_small_fused(const __grid_constant__ RouterLogitsParams lp,
                                                          const __grid_constant__ RouterSelectParams sp,
                                                          const __grid_constant__ AddNormParams np, int has_norm,
                                                          const __grid_constant__ SmallPermuteOut po) {
  extern __shared__ __align__(16) uint8_t dyn[];
  __shared__ float red[8][RG];
  __shared__ float nred[NORM_THREADS / 32];
  __shared__ int s_last;
  pdl_trigger();
  // the router row and the norm weight are model weights: fetch them toward L2 while
  // the previous kernel finishes
  prefetch_l2_lines(static_cast<const E*>(lp.w) + static_cast<int64_t>(blockIdx.x) * lp.H,
                    static_cast<int64_t>(lp.H) * sizeof(E));
  if (has_norm && blockIdx.x == 0) prefetch_l2_lines(np.weight, static_cast<int64_t>(np.H) * sizeof(E));
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x;
  const int T = lp.T, H = lp.H;
  constexpr int V = 16 / sizeof(E);
  E* xs = reinterpret_cast<E*>(dyn);  // [T][H]
  int32_t* hist = reinterpret_cast<int32_t*>(dyn + ((static_cast<size_t>(T) * H * sizeof(E) + 15) & ~size_t(15)));

  if (has_norm) {
    for (int t = 0; t < T; ++t) {
      E* rout = (e == 0) ? static_cast<E*>(np.residual_out) + static_cast<int64_t>(t) * np.ld : nullptr;
      E* ng = (e == 0 && np.normed) ? static_cast<E*>(np.normed) + static_cast<int64_t>(t) * np.ld_normed : nullptr;
      add_rmsnorm_row<E>(np, t, rout, xs + static_cast<int64_t>(t) * H, ng, nred);
    }
  } else {
    const E* x = static_cast<const E*>(lp.x);
    const int vpr = H / V;
    for (int i = threadIdx.x; i < T * vpr; i += blockDim.x) {
      const int t = i / vpr, c = (i - t * vpr) * V;
      *reinterpret_cast<uint4*>(xs + static_cast<int64_t>(t) * H + c) =
          __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * lp.ldx + c));
    }
  }
  __syncthreads();

  const E* w = static_cast<const E*>(lp.w) + static_cast<int64_t>(e) * H;
  float acc[RG];
#pragma unroll
  for (int i = 0; i < RG; ++i) acc[i] = 0.f;
  for (int c = threadIdx.x * V; c < H; c += 256 * V) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + c));
    const E* we = reinterpret_cast<const E*>(&wv);
#pragma unroll
    for (int i = 0; i < RG; ++i) {
      if (i < T) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + static_cast<int64_t>(i) * H + c);
        const E* xe = reinterpret_cast<const E*>(&xv);
#pragma unroll
        for (int j = 0; j < V; ++j) acc[i] = fmaf(static_cast<float>(xe[j]), static_cast<float>(we[j]), acc[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < RG; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < RG; ++i) red[warp][i] = acc[i];
  }
  __syncthreads();
  if (threadIdx.x < T) {
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) v += red[q][threadIdx.x];
    if (lp.bias) v += lp.bias[e];
    if (sizeof(E) == 2 && lp.round_bf16) v = bf16_round(v);
    lp.logits[static_cast<int64_t>(threadIdx.x) * lp.E1 + e] = v;
  }

  // the last column to finish selects for every token
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(sp.ticket, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int s = threadIdx.x; s < sp.num_slots; s += blockDim.x) hist[s] = 0;
  __syncthreads();
  select_tokens_any(sp, 0, T, hist);
  __syncthreads();
  select_finish_one_block(sp, hist);
  if (po.send == nullptr) return;

  // The permute of the one token block (permute_rows' order: within a slot, flat
  // t*K+k order), with the rows taken from shared memory: hist holds the slot offsets,
  // phys_ids were written by this CTA above.
  __shared__ int32_t s_pos[RG * 8];
  const int ne = T * sp.K;
  __syncthreads();
  if (warp == 0) {
    for (int base = 0; base < ne; base += 32) {
      const int i = base + lane;
      const bool valid = i < ne;
      const int s = valid ? sp.phys_ids[i] : -1 - lane;
      const uint32_t peers = __match_any_sync(0xffffffffu, s);
      const int leader = __ffs(peers) - 1;
      int start = 0;
      if (valid && lane == leader) {
        start = hist[s];
        hist[s] = start + __popc(peers);
      }
      start = __shfl_sync(0xffffffffu, start, leader);
      if (valid) {
        const int d = start + __popc(peers & ((1u << lane) - 1u));
        s_pos[i] = d;
        po.pos_of[i] = d;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  const int vpr = H / V;
  for (int idx = threadIdx.x; idx < ne * vpr; idx += blockDim.x) {
    const int i = idx / vpr, v = idx - i * vpr;
    const int t = i / sp.K;
    *reinterpret_cast<uint4*>(static_cast<uint8_t*>(po.send) + static_cast<int64_t>(s_pos[i]) * po.row_bytes +
                              static_cast<int64_t>(v) * 16) =
        *reinterpret_cast<const uint4*>(xs + static_cast<int64_t>(t) * H + static_cast<int64_t>(v) * V);
  }
}

size_t router_small_fused_smem(int T, int H, int x_dtype, int num_slots, int scoring) {
  const size_t rows = (static_cast<size_t>(T) * H * dtype_bytes(x_dtype) + 15) & ~size_t(15);
  return rows + static_cast<size_t>(num_slots) * sizeof(int32_t) + (scoring == 1 ? 8 * 256 * sizeof(float) : 0);
}

bool router_small_fused_ok(int T, int H, int x_dtype, int num_slots, int scoring, bool has_norm) {
  const int V = 16 / dtype_bytes(x_dtype);
  if (T < 1 || T > RG || H % V != 0) return false;
  if (has_norm && H / V > NORM_THREADS * NORM_MAXV) return false;
  return router_small_fused_smem(T, H, x_dtype, num_slots, scoring) <= kFusedSmemMax;
}

int launch_router_small_fused(const RouterLogitsParams& lp, const RouterSelectParams& sp, const AddNormParams* np,
                              int x_dtype, cudaStream_t stream, const SmallPermuteOut* po) {
  static std::atomic<uint64_t> attr_set_mask{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set_mask.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(router_small_fused<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kFusedSmemMax)) != cudaSuccess ||
        cudaFuncSetAttribute(router_small_fused<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kFusedSmemMax)) != cudaSuccess)
      return -3;
    attr_set_mask.fetch_or(bit, std::memory_order_release);
  }
  AddNormParams none{};
  const SmallPermuteOut no_perm{};
  const size_t smem = router_small_fused_smem(lp.T, lp.H, x_dtype, sp.num_slots, sp.scoring);
  cudaError_t e;
  if (x_dtype == kDtypeBF16)
    e = launch_kernel(router_small_fused<__nv_bfloat16>, dim3(lp.E1), dim3(256), smem, stream, lp, sp,
                      np ? *np : none, np ? 1 : 0, po ? *po : no_perm);
  else
    e = launch_kernel(router_small_fused<float>, dim3(lp.E1), dim3(256), smem, stream, lp, sp, np ? *np : none,
                      np ? 1 : 0, po ? *po : no_perm);
  return e == cudaSuccess ? 0 : -2;
}

// ------------------------------------------------------------------ host launchers
// Router columns per CTA of the GEMV (1: router_logits_gemv).  Column groups need the
// token rows to fit in registers (H == NX * 256 * V, NX <= 2); the widest group that
// still gives every SM a CTA is taken.  B200MOE_ROUTER_COLS=c forces c
// (1, 2, 4, 8 or 16) for tuning.
static int router_gemv_cols(int groups, int E1, int H, int x_dtype) {
  const int V = 16 / dtype_bytes(x_dtype);
  const int nx = H / (256 * V);
  if (nx < 1 || nx > 2 || nx * 256 * V != H) return 1;
  const char* env = getenv("B200MOE_ROUTER_COLS");
  if (env != nullptr) {
    const int c = atoi(env);
    return (c == 2 || c == 4 || c == 8 || c == 16) ? c : 1;
  }
  int cg = 1;
  while (cg < 16 && static_cast<int64_t>(groups) * ((E1 + 2 * cg - 1) / (2 * cg)) >= num_sms()) cg *= 2;
  return cg;
}

template <typename E>
static void launch_gemv_cols(dim3 grid, int cg, int nx, const RouterLogitsParams& p, cudaStream_t stream) {
#define B200MOE_GEMV_COLS(NXV, CGV) \
  if (nx == NXV && cg == CGV) { launch_kernel(router_logits_gemv_cols<E, NXV, CGV>, grid, dim3(256), 0, stream, p); return; }
  B200MOE_GEMV_COLS(1, 2) B200MOE_GEMV_COLS(1, 4) B200MOE_GEMV_COLS(1, 8) B200MOE_GEMV_COLS(1, 16)
  B200MOE_GEMV_COLS(2, 2) B200MOE_GEMV_COLS(2, 4) B200MOE_GEMV_COLS(2, 8) B200MOE_GEMV_COLS(2, 16)
#undef B200MOE_GEMV_COLS
}

int launch_router_logits(const RouterLogitsParams& p, int x_dtype, cudaStream_t stream) {
  if (p.T == 0) return 0;
  // GEMV (one CTA per (8-token group, column)) up to this many tokens, tensor-core
  // tiles above; B200MOE_ROUTER_GEMV_MAX overrides it for tuning.
  static const int gemv_max = [] {
    const char* v = getenv("B200MOE_ROUTER_GEMV_MAX");
    return v ? atoi(v) : 256;
  }();
  if (p.T <= gemv_max) {
    const int groups = (p.T + RG - 1) / RG;
    const int cg = router_gemv_cols(groups, p.E1, p.H, x_dtype);
    if (cg > 1) {
      const dim3 grid(groups, (p.E1 + cg - 1) / cg);
      const int nx = p.H / (256 * (16 / dtype_bytes(x_dtype)));
      if (x_dtype == kDtypeBF16)
        launch_gemv_cols<__nv_bfloat16>(grid, cg, nx, p, stream);
      else
        launch_gemv_cols<float>(grid, cg, nx, p, stream);
      return 0;
    }
    const dim3 grid(groups, p.E1);
    if (x_dtype == kDtypeBF16)
      launch_kernel(router_logits_gemv<__nv_bfloat16>, grid, dim3(256), 0, stream, p);
    else
      launch_kernel(router_logits_gemv<float>, grid, dim3(256), 0, stream, p);
    return 0;
  }
  if (x_dtype == kDtypeBF16) {
    const int tok_blocks = (p.T + RL_TOK - 1) / RL_TOK;
    // Enough CTAs to cover the SMs: narrow column groups when the token count is small.
    // one column group when there are enough token blocks to cover the SMs (x is read
    // once); narrower groups only for short batches
    int cols = min(RL_MAXNT * 8, ((p.E1 + 7) / 8) * 8);
    while (cols > 8 && tok_blocks * ((p.E1 + cols - 1) / cols) < num_sms()) cols -= 8;
    dim3 grid(tok_blocks, (p.E1 + cols - 1) / cols);
    const size_t stage_bytes = static_cast<size_t>(RL_TOK + cols) * RL_LD * sizeof(__nv_bfloat16);
    static std::atomic<uint64_t> attr_set_mask{0};  // one bit per device ordinal
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set_mask.load(std::memory_order_acquire) & bit)) {
      auto set = [](const void* k, int bytes) {
        return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
      };
      const int b = RL_LD * sizeof(__nv_bfloat16);
      if (!set(reinterpret_cast<const void*>(router_logits_bf16<8, 1>), 8 * (RL_TOK + 8) * b) ||
          !set(reinterpret_cast<const void*>(router_logits_bf16<8, 3>), 8 * (RL_TOK + 24) * b) ||
          !set(reinterpret_cast<const void*>(router_logits_bf16<4, 8>), 4 * (RL_TOK + 64) * b) ||
          !set(reinterpret_cast<const void*>(router_logits_bf16<4, RL_MAXNT>), 4 * (RL_TOK + RL_MAXNT * 8) * b))
        return -3;
      attr_set_mask.fetch_or(bit, std::memory_order_release);
    }
    if (cols <= 8)
      launch_kernel(router_logits_bf16<8, 1>, grid, dim3(128), 8 * stage_bytes, stream, p, cols);
    else if (cols <= 24)
      launch_kernel(router_logits_bf16<8, 3>, grid, dim3(128), 8 * stage_bytes, stream, p, cols);
    else if (cols <= 64)
      launch_kernel(router_logits_bf16<4, 8>, grid, dim3(128), 4 * stage_bytes, stream, p, cols);
    else
      launch_kernel(router_logits_bf16<4, RL_MAXNT>, grid, dim3(128), 4 * stage_bytes, stream, p, cols);
  } else {
    const int grid = (p.T * 32 + 255) / 256;
    launch_kernel(router_logits_f32, dim3(grid), dim3(256), 0, stream, p);
  }
  return 0;
}

int launch_router_select(const RouterSelectParams& p, cudaStream_t stream) {
  if (p.T == 0) return 0;
  const size_t smem = static_cast<size_t>(p.num_slots) * sizeof(int32_t) +
                      (p.scoring == 1 ? 8 * 256 * sizeof(float) : 0);
  const dim3 grid(p.nblocks);
  if (p.E <= 32)
    launch_kernel(router_select<1>, grid, dim3(256), smem, stream, p);
  else if (p.E <= 64)
    launch_kernel(router_select<2>, grid, dim3(256), smem, stream, p);
  else if (p.E <= 128)
    launch_kernel(router_select<4>, grid, dim3(256), smem, stream, p);
  else
    launch_kernel(router_select<RS_MAXJ>, grid, dim3(256), smem, stream, p);
  return 0;
}

}  // namespace b200moe
