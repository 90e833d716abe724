// Kernel family (2) and (4): token permutation and the weighted unpermute.
//
// permute_rows mirrors the reference's dispatch-side permutation
//   idx          = phys_ids.view(-1).sort(stable=True).indices
//   send_indices = idx // K ; send_topk = idx % K
//   send         = x[send_indices]
// (MoeAll2AllBlock.all2all_chunk_routing_compute, easyinfra/generation/blocks/moe/
//  moe_all2all.py:345-351), without a sort: the router's last CTA already turned the
// per-block slot histograms into absolute write offsets, so each CTA ranks its own
// entries stably (flat index order within a slot) with warp match/ballot and writes
// every token row to its K destinations with 16-byte vector stores.  Rows of one
// destination rank are contiguous ([dst rank][local slot][token order]) because
// physical slot ids are rank-major.  In peer mode (fused with the expert-parallel
// dispatch) the K stores of a row go straight to the owning ranks' receive regions
// over NVLink, and the last CTA publishes the counts and raises the arrival flags
// (the protocol is described in ep_nvlink.cu).
//
// combine_rows mirrors the reference's unpermute
//   out = zeros(T, H); out.index_add_(0, send_indices, y * w[send_indices, send_topk])
// (moe_all2all.py:291-307) as a gather: one warp per token reads its K expert rows,
// accumulates w_k * y_k in fp32 and writes the token row once (no atomics).  The
// optional shared-expert term adds gate[t] * shared[t] (gate == 1 when absent).
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "kernels.cuh"

namespace b200moe {

constexpr int PM_MAX_ENTRIES = 64 * 8;  // tb * K must not exceed this

template <bool PEER>
__global__ void __launch_bounds__(256) permute_rows(const __grid_constant__ PermuteParams p) {
  extern __shared__ int32_t running[];     // [num_slots], -1 == not yet touched
  __shared__ int32_t pos[PM_MAX_ENTRIES];  // destination row of each entry of this block
  __shared__ uint8_t* dst_row[PEER ? PM_MAX_ENTRIES : 1];  // peer mode: where each entry goes
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (PEER && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x < p.ep.G)
    ep_publish_meta(p.ep, p.slot_offsets, threadIdx.x);
  const int t0 = blockIdx.x * p.tb;
  const int nt = min(p.tb, p.T - t0);
  const int ne = nt * p.K;
  const int64_t flat0 = static_cast<int64_t>(t0) * p.K;

  for (int s = threadIdx.x; s < p.num_slots; s += blockDim.x) running[s] = -1;
  __syncthreads();
  if (warp == 0) {
    // Stable rank within the block: entries in flat (t*K + k) order, 32 at a time.
    for (int base = 0; base < ne; base += 32) {
      const int i = base + lane;
      const bool valid = i < ne;
      const int s = valid ? p.phys_ids[flat0 + i] : -1 - lane;
      const uint32_t peers = __match_any_sync(0xffffffffu, s);
      const int leader = __ffs(peers) - 1;
      int start = 0;
      if (valid && lane == leader) {
        int cur = running[s];
        if (cur < 0) cur = p.block_offsets[static_cast<int64_t>(s) * p.nblocks + blockIdx.x];
        start = cur;
        running[s] = cur + __popc(peers);
      }
      start = __shfl_sync(0xffffffffu, start, leader);
      if (valid) pos[i] = start + __popc(peers & ((1u << lane) - 1u));
      __syncwarp();
    }
  }
  __syncthreads();

  for (int i = threadIdx.x; i < ne; i += blockDim.x) {
    const int d = pos[i];
    if (blockIdx.y == 0) {
      p.pos_of[flat0 + i] = d;
      if (p.send_token) p.send_token[d] = t0 + i / p.K;
      if (p.send_slot) p.send_slot[d] = i % p.K;
    }
    if (PEER) {
      // send row d of slot s -> row (rank * cap + j) of the owner's receive region,
      // j = d - (first send row of the owner rank)
      const EpParams& ep = p.ep;
      const int g = p.phys_ids[flat0 + i] / ep.P;
      const int64_t j = d - p.slot_offsets[g * ep.P];
      uint8_t* dst = nullptr;
      if (j >= 0 && j < ep.cap_rows)
        dst = ep_recv_rows(ep.peer[g], ep) + (static_cast<int64_t>(ep.rank) * ep.cap_rows + j) * p.row_bytes;
      else
        record_status(ep.status, kStatusCapacity);
      dst_row[i] = dst;
    }
  }
  if (PEER) __syncthreads();

  // Row copies: one warp per token; the token row is read once (PM_BATCH 16-byte loads
  // per lane in flight together) and written K times.  Small batches split the columns
  // over gridDim.y CTAs per token block (CTA y copies its slice of every row), so a few
  // token blocks still spread over many SMs.
  constexpr int PM_BATCH = 8;
  const int vec_total = p.row_bytes / 16;
  const int vec_slice = (vec_total + gridDim.y - 1) / gridDim.y;
  const int vec_begin = blockIdx.y * vec_slice;
  const int vec_per_row = min(vec_total, vec_begin + vec_slice);
  for (int lt = warp; lt < nt; lt += blockDim.x >> 5) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.x) +
                                                      static_cast<int64_t>(t0 + lt) * p.x_stride);
    for (int v0 = vec_begin; v0 < vec_per_row; v0 += PM_BATCH * 32) {
      uint4 val[PM_BATCH];
#pragma unroll
      for (int u = 0; u < PM_BATCH; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < vec_per_row) val[u] = __ldg(src + v);
      }
      for (int k = 0; k < p.K; ++k) {
        uint4* dst;
        if (PEER) {
          uint8_t* row = dst_row[lt * p.K + k];
          if (row == nullptr) continue;
          dst = reinterpret_cast<uint4*>(row);
        } else {
          dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.send) +
                                         static_cast<int64_t>(pos[lt * p.K + k]) * p.row_bytes);
        }
#pragma unroll
        for (int u = 0; u < PM_BATCH; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < vec_per_row) dst[v] = val[u];
        }
      }
    }
  }
  if (PEER) {
    if (last_cta(p.ep.ticket, &s_last) && threadIdx.x < p.ep.G) ep_publish_rows(p.ep, threadIdx.x);
  }
}

// 8 consecutive elements -> fp32.  L2_ONLY reads through L2 only (rows that another
// GPU wrote while this kernel was running); otherwise the read-only data path.
template <typename E, bool L2_ONLY = false>
__device__ __forceinline__ void load8(const E* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16, false>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16, true>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float, false>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<float, true>(const float* p, float (&v)[8]) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename E>
__device__ __forceinline__ void store8(E* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// One warp per (token, 256-column chunk): all K expert rows of the chunk are loaded
// before any arithmetic, so a token's gathers are in flight together.
// KT: compile-time bound on K (registers scale with it: KT rows of 8 values in flight).
template <typename E, bool PEER, int KT>
__device__ __forceinline__ void combine_body(const CombineParams& p) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int chunks = (p.H + 255) / 256;
  if (gw >= static_cast<int64_t>(p.T) * chunks) return;
  const int t = static_cast<int>(gw / chunks);
  const int c = static_cast<int>(gw - static_cast<int64_t>(t) * chunks) * 256 + lane * 8;
  if (c >= p.H) return;
  const E* y = static_cast<const E*>(p.y);
  float v[KT][8];
  float wts[KT];
#pragma unroll
  for (int k = 0; k < KT; ++k) {
    if (k < p.K) {
      const int row = p.pos_of[static_cast<int64_t>(t) * p.K + k];
      wts[k] = p.topk_w[static_cast<int64_t>(t) * p.K + k];
      load8<E, PEER>(y + static_cast<int64_t>(row) * p.ldy + c, v[k]);
    }
  }
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < KT; ++k) {
    if (k < p.K) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(wts[k], v[k][i], acc[i]);
    }
  }
  if (p.shared) {
    const float g = p.shared_gate ? p.shared_gate[t] : 1.f;
    float s[8];
    load8<E>(static_cast<const E*>(p.shared) + static_cast<int64_t>(t) * p.lds + c, s);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = fmaf(g, s[i], acc[i]);
  }
  store8<E>(static_cast<E*>(p.out) + static_cast<int64_t>(t) * p.ldo + c, acc);
}

// PEER: y is this rank's combine region, filled by the ranks that hold its experts.
// Every CTA first waits (bounded) until each of them raised its flag past the count
// this rank consumed; the last CTA to finish advances that count.
template <typename E, bool PEER, int KT>
__global__ void __launch_bounds__(256) combine_rows(const __grid_constant__ CombineParams p) {
  __shared__ uint32_t s_target;
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  if (PEER) {
    if (threadIdx.x == 0) {
      const uint32_t target = *p.wait_expect + 1u;
      bool ok = true;
      for (int d = 0; d < p.wait_n && ok; ++d) ok = wait_flag_geq(p.wait_flags + d, target, p.wait_timeout_ns, p.status);
      if (!ok) record_status(p.status, kStatusTimeout);
      s_target = target;
    }
    __syncthreads();
  }
  combine_body<E, PEER, KT>(p);
  if (PEER) {
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(p.wait_ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
      *p.wait_expect = s_target;
      *p.wait_ticket = 0u;
    }
  }
}

// Batches of prefill size: persistent CTAs stream each token's K expert rows (and its
// shared-expert row) into a ring of shared-memory stages with bulk copies that complete
// on the stage's mbarrier.  Warp 8 issues the copies; warps 0-7 reduce each token from
// shared memory in combine_body's order, so both kernels give the same bits.  A CTA
// keeps up to kCombineStageBudget bytes of row reads in flight without holding them in
// registers (the warp kernel is bound by the loads each warp can keep outstanding).
constexpr int CB_CONSUMERS = 256;
constexpr int CB_THREADS = CB_CONSUMERS + 32;
constexpr uint32_t kCombineStageBudget = 96 * 1024;
constexpr int kCombineMaxStages = 8;
constexpr int kCombineBulkMinT = 2048;

template <typename E>
__device__ __forceinline__ void lds8(const uint8_t* p, float (&v)[8]) {
  if constexpr (sizeof(E) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

template <typename E, bool PEER, int KT>
__global__ void __launch_bounds__(CB_THREADS) combine_rows_bulk(const __grid_constant__ CombineParams p, int stages) {
  extern __shared__ __align__(128) uint8_t cb_rows[];  // [stages][K (+1 shared)][H]
  __shared__ uint64_t full[kCombineMaxStages], empty[kCombineMaxStages];
  __shared__ int s_abort;
  __shared__ uint32_t s_target;
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rb = static_cast<uint32_t>(p.H) * sizeof(E);
  const uint32_t stage_bytes = rb * static_cast<uint32_t>(p.K + (p.shared ? 1 : 0));
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CB_CONSUMERS / 32);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  pdl_trigger();
  pdl_wait();
  if (PEER && threadIdx.x == 0) {
    const uint32_t target = *p.wait_expect + 1u;
    bool ok = true;
    for (int d = 0; d < p.wait_n && ok; ++d) ok = wait_flag_geq(p.wait_flags + d, target, p.wait_timeout_ns, p.status);
    if (!ok) record_status(p.status, kStatusTimeout);
    s_target = target;
  }
  __syncthreads();
  int issued = 0;  // producer: stages filled so far
  if (warp == CB_CONSUMERS / 32) {
    if (lane == 0) {
      if (PEER) {
        // rows the peers stored: acquire their flags in this thread too (thread 0 saw
        // them reach the target; they only grow), then order the bulk reads after it
        for (int d = 0; d < p.wait_n; ++d) (void)ld_acquire_sys(p.wait_flags + d);
        fence_proxy_async_global();
      }
      const E* y = static_cast<const E*>(p.y);
      const E* sh = static_cast<const E*>(p.shared);
      int& i = issued;
      for (int t = blockIdx.x; t < p.T; t += gridDim.x, ++i) {
        const int s = i % stages;
        const uint32_t ph = static_cast<uint32_t>(i / stages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, &s_abort, p.status)) break;
        uint8_t* dst = cb_rows + static_cast<size_t>(s) * stage_bytes;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        for (int k = 0; k < p.K; ++k) {
          const int row = p.pos_of[static_cast<int64_t>(t) * p.K + k];
          bulk_load(dst + k * rb, y + static_cast<int64_t>(row) * p.ldy, rb, &full[s]);
        }
        if (sh) bulk_load(dst + p.K * rb, sh + static_cast<int64_t>(t) * p.lds, rb, &full[s]);
      }
    }
  } else {
    int i = 0;
    for (int t = blockIdx.x; t < p.T; t += gridDim.x, ++i) {
      const int s = i % stages;
      const uint32_t ph = static_cast<uint32_t>(i / stages) & 1u;
      float wts[KT];
#pragma unroll
      for (int k = 0; k < KT; ++k) wts[k] = (k < p.K) ? p.topk_w[static_cast<int64_t>(t) * p.K + k] : 0.f;
      const float g = (p.shared && p.shared_gate) ? p.shared_gate[t] : 1.f;
      if (!mbar_wait(&full[s], ph, &s_abort, p.status)) break;
      const uint8_t* src = cb_rows + static_cast<size_t>(s) * stage_bytes;
      E* out = static_cast<E*>(p.out) + static_cast<int64_t>(t) * p.ldo;
      for (int c = threadIdx.x * 8; c < p.H; c += CB_CONSUMERS * 8) {
        float v[KT][8];
#pragma unroll
        for (int k = 0; k < KT; ++k)
          if (k < p.K) lds8<E>(src + k * rb + c * sizeof(E), v[k]);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int k = 0; k < KT; ++k) {
          if (k < p.K) {
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = fmaf(wts[k], v[k][e], acc[e]);
          }
        }
        if (p.shared) {
          float sv[8];
          lds8<E>(src + p.K * rb + c * sizeof(E), sv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = fmaf(g, sv[e], acc[e]);
        }
        store8<E>(out + c, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  __syncthreads();
  if (s_abort && warp == CB_CONSUMERS / 32 && lane == 0) {
    // a wait gave up: the copies already issued land before the CTA exits
    volatile int no_abort = 0;
    for (int j = max(0, issued - stages); j < issued; ++j)
      mbar_wait(&full[j % stages], static_cast<uint32_t>(j / stages) & 1u, &no_abort, p.status);
  }
  if (PEER) {
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(p.wait_ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
      *p.wait_expect = s_target;
      *p.wait_ticket = 0u;
    }
  }
}

// Column slices per token block: enough CTAs for about two per SM, each slice at least
// one 512-byte batch of a warp's 16-byte copies.
static int permute_slices(const PermuteParams& p, int nblocks) {
  const int by_sms = (2 * num_sms() + nblocks - 1) / nblocks;
  const int by_row = max64(1, p.row_bytes / 512);
  return static_cast<int>(max64(1, min64(by_sms, by_row)));
}

int launch_permute(const PermuteParams& p, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(p.num_slots) * sizeof(int32_t);
  if (p.peer_mode) {  // always launched: a rank without tokens still publishes empty counts
    const int nb = p.nblocks > 0 ? p.nblocks : 1;
    return launch_kernel(permute_rows<true>, dim3(nb, permute_slices(p, nb)), dim3(256), smem, stream, p) ==
                   cudaSuccess
               ? 0
               : -2;
  }
  if (p.T == 0) return 0;
  launch_kernel(permute_rows<false>, dim3(p.nblocks, permute_slices(p, p.nblocks)), dim3(256), smem, stream, p);
  return 0;
}

template <typename E, bool PEER>
static cudaError_t launch_combine_k(const CombineParams& p, int grid, cudaStream_t stream) {
  if (p.K <= 1) return launch_kernel(combine_rows<E, PEER, 1>, dim3(grid), dim3(256), 0, stream, p);
  if (p.K <= 2) return launch_kernel(combine_rows<E, PEER, 2>, dim3(grid), dim3(256), 0, stream, p);
  if (p.K <= 4) return launch_kernel(combine_rows<E, PEER, 4>, dim3(grid), dim3(256), 0, stream, p);
  if (p.K <= 6) return launch_kernel(combine_rows<E, PEER, 6>, dim3(grid), dim3(256), 0, stream, p);
  return launch_kernel(combine_rows<E, PEER, 8>, dim3(grid), dim3(256), 0, stream, p);
}

template <typename E, bool PEER>
static cudaError_t launch_combine_bulk_k(const CombineParams& p, int grid, int stages, size_t smem,
                                         cudaStream_t stream) {
  if (p.K <= 2) return launch_kernel(combine_rows_bulk<E, PEER, 2>, dim3(grid), dim3(CB_THREADS), smem, stream, p, stages);
  if (p.K <= 4) return launch_kernel(combine_rows_bulk<E, PEER, 4>, dim3(grid), dim3(CB_THREADS), smem, stream, p, stages);
  if (p.K <= 6) return launch_kernel(combine_rows_bulk<E, PEER, 6>, dim3(grid), dim3(CB_THREADS), smem, stream, p, stages);
  return launch_kernel(combine_rows_bulk<E, PEER, 8>, dim3(grid), dim3(CB_THREADS), smem, stream, p, stages);
}

template <typename E, bool PEER>
static bool set_combine_bulk_smem() {
  const int bytes = static_cast<int>(kCombineStageBudget);
  return cudaFuncSetAttribute(combine_rows_bulk<E, PEER, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(combine_rows_bulk<E, PEER, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(combine_rows_bulk<E, PEER, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(combine_rows_bulk<E, PEER, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
}

// Stages of the bulk kernel for this shape (0: the shape does not fit two stages).
static int combine_bulk_stages(const CombineParams& p) {
  const size_t eb = p.dtype == kDtypeBF16 ? 2 : 4;
  const size_t stage = static_cast<size_t>(p.H) * eb * static_cast<size_t>(p.K + (p.shared ? 1 : 0));
  const int stages = static_cast<int>(min64(kCombineMaxStages, static_cast<int64_t>(kCombineStageBudget / stage)));
  return stages >= 2 ? stages : 0;
}

// B200MOE_COMBINE=warp|bulk forces a combine kernel (tests and tuning); otherwise
// the bulk kernel runs from kCombineBulkMinT tokens when the shape fits its stages.
static bool use_combine_bulk(const CombineParams& p) {
  if (combine_bulk_stages(p) == 0) return false;
  const char* v = getenv("B200MOE_COMBINE");
  if (v != nullptr && strcmp(v, "warp") == 0) return false;
  if (v != nullptr && strcmp(v, "bulk") == 0) return true;
  return p.T >= kCombineBulkMinT;
}

static int launch_combine_bulk(const CombineParams& p, bool peer, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_set_mask{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set_mask.load(std::memory_order_acquire) & bit)) {
    if (!set_combine_bulk_smem<__nv_bfloat16, false>() || !set_combine_bulk_smem<__nv_bfloat16, true>() ||
        !set_combine_bulk_smem<float, false>() || !set_combine_bulk_smem<float, true>())
      return -3;
    attr_set_mask.fetch_or(bit, std::memory_order_release);
  }
  const int stages = combine_bulk_stages(p);
  const size_t eb = p.dtype == kDtypeBF16 ? 2 : 4;
  const size_t smem = static_cast<size_t>(stages) * static_cast<size_t>(p.H) * eb * (p.K + (p.shared ? 1 : 0));
  // two CTAs per SM (2 x 96 KB of stages), one token per CTA at least
  const int grid = static_cast<int>(max64(1, min64(p.T, 2 * static_cast<int64_t>(num_sms()))));
  cudaError_t e;
  if (p.dtype == kDtypeBF16)
    e = peer ? launch_combine_bulk_k<__nv_bfloat16, true>(p, grid, stages, smem, stream)
             : launch_combine_bulk_k<__nv_bfloat16, false>(p, grid, stages, smem, stream);
  else
    e = peer ? launch_combine_bulk_k<float, true>(p, grid, stages, smem, stream)
             : launch_combine_bulk_k<float, false>(p, grid, stages, smem, stream);
  return e == cudaSuccess ? 0 : -2;
}

int launch_combine(const CombineParams& p, cudaStream_t stream) {
  const bool peer = p.wait_n > 0;
  if (p.T == 0 && !peer) return 0;  // peer mode always runs: it consumes the arrival flags
  if (use_combine_bulk(p)) return launch_combine_bulk(p, peer, stream);
  const int64_t warps = static_cast<int64_t>(p.T) * ((p.H + 255) / 256);
  const int grid = static_cast<int>(max64(1, (warps * 32 + 255) / 256));
  cudaError_t e;
  if (p.dtype == kDtypeBF16)
    e = peer ? launch_combine_k<__nv_bfloat16, true>(p, grid, stream)
             : launch_combine_k<__nv_bfloat16, false>(p, grid, stream);
  else
    e = peer ? launch_combine_k<float, true>(p, grid, stream) : launch_combine_k<float, false>(p, grid, stream);
  return e == cudaSuccess ? 0 : -2;
}

}  // namespace b200moe
