// Parameter blocks and host launchers shared by the kernel translation units and
// the C-ABI layer (capi.cu).  Each struct is passed by value to its kernel.
#pragma once

#include "common.cuh"

namespace b200moe {

// ---- router (router.cu)
struct RouterLogitsParams {
  const void* x;
  int64_t ldx;         // elements
  const void* w;       // [E1, H] row-major (E routed rows, optionally + 1 shared-gate row)
  const float* bias;   // [E1] or null
  int T, H, E1;
  float* logits;       // [T, E1]
  int round_bf16 = 1;  // round bf16 logits like F.linear's bf16 output (0: keep fp32)
};

struct RouterSelectParams {
  const float* logits;  // [T, E1]
  int T, E, E1, K;
  int renorm;
  float scale;
  int round_bf16;       // round the final weights to bf16 (x.dtype == bfloat16)
  int has_shared_gate;  // logits column E is the shared-expert gate logit
  const int32_t* log2phy;    // [E, max_rep] or null (physical id == logical id)
  const int32_t* rep_count;  // [E]
  int max_rep;
  int num_slots;             // physical slots across all ranks (G * P)
  int tb;                    // tokens per CTA
  int nblocks;
  int32_t* topk_ids;     // [T, K] logical expert ids
  float* topk_w;         // [T, K]
  int32_t* phys_ids;     // [T, K]
  float* shared_gate;    // [T] sigmoid(shared-gate logit), when has_shared_gate
  int32_t* block_counts; // [num_slots, nblocks]  -> becomes absolute write offsets
  int32_t* slot_totals;  // [num_slots], zero between calls (nblocks > 16: CTAs add their counts)
  int32_t* slot_counts;  // [num_slots]
  int32_t* slot_offsets; // [num_slots + 1]
  uint32_t* ticket;      // zero before the first call; the last CTA resets it
  int* status;
  // scoring 0: softmax top-k (Qwen3MoeSparseMoeBlock._routing);
  // scoring 1: sigmoid + correction bias + group-limited top-k (DeepseekV3MoEGate)
  int scoring = 0;
  int n_group = 1, topk_group = 1;
  const float* correction_bias = nullptr;  // [E]
};

// ---- expert-parallel exchange over peer memory (ep_nvlink.cu)
constexpr int EP_MAX_RANKS = 8;

// Every rank's exchange buffer (one peer-mapped allocation per rank, same layout):
//   [0, 256)            flags: disp[G] (rows arrived), comb[G] (results returned),
//                       meta[G] (counts arrived), u32, only ever incremented
//   [256, 256 + meta)   meta: G x (P + 1) i32 — per source: rows per local slot, then
//                       the source's first send row for this rank
//   recv rows           G x cap_rows rows of row_bytes (region s written by source s)
//   comb rows           comb_rows rows (this rank's send order, written by the ranks
//                       that hold its experts)
struct EpParams {
  uint8_t* peer[EP_MAX_RANKS];  // base of every rank's buffer (peer[rank] is this rank's)
  int G, P, rank;
  int row_bytes;
  int64_t cap_rows;   // rows per source region
  int64_t comb_rows;  // rows of the combine region
  uint32_t* ticket;   // local, zero between launches
  int* status;
};

__host__ __device__ inline int64_t ep_meta_bytes(int G, int P) {
  return ((static_cast<int64_t>(G) * (P + 1) * 4 + 255) / 256) * 256;
}
__host__ __device__ inline int64_t ep_recv_offset(int G, int P) { return 256 + ep_meta_bytes(G, P); }
__host__ __device__ inline int64_t ep_comb_offset(int G, int P, int64_t cap_rows, int row_bytes) {
  return ep_recv_offset(G, P) + static_cast<int64_t>(G) * cap_rows * row_bytes;
}
__host__ __device__ inline int64_t ep_buffer_bytes(int G, int P, int64_t cap_rows, int64_t comb_rows,
                                                   int row_bytes) {
  return ep_comb_offset(G, P, cap_rows, row_bytes) + comb_rows * row_bytes;
}
__device__ __forceinline__ uint32_t* ep_flags(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }
__device__ __forceinline__ int32_t* ep_meta(uint8_t* base, const EpParams& p) {
  return reinterpret_cast<int32_t*>(base + 256);
}
__device__ __forceinline__ uint8_t* ep_recv_rows(uint8_t* base, const EpParams& p) {
  return base + ep_recv_offset(p.G, p.P);
}
__device__ __forceinline__ uint8_t* ep_comb_rows(uint8_t* base, const EpParams& p) {
  return base + ep_comb_offset(p.G, p.P, p.cap_rows, p.row_bytes);
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for *flag >= target (wrap-safe compare); false on timeout.  A zero
// timeout checks once, and so does every wait once the status word holds an error
// (a layer that already failed drains instead of waiting out every later limit).
__device__ __forceinline__ bool wait_flag_geq(const uint32_t* flag, uint32_t target, uint64_t timeout_ns,
                                              const int* status) {
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (static_cast<int32_t>(ld_acquire_sys(flag) - target) >= 0) return true;
    if (timeout_ns == 0 || globaltimer_ns() - t0 > timeout_ns) return false;
    if (status != nullptr && *reinterpret_cast<const volatile int*>(status) != 0) return false;
    __nanosleep(64);
  }
}

// One warp copies one row; L2-only loads for rows that a peer wrote.  Eight loads per
// lane are issued before their stores, so a row's reads are in flight together rather
// than one latency per 512 bytes.
template <bool FROM_PEER>
__device__ __forceinline__ void copy_row(uint8_t* dst, const uint8_t* src, int row_bytes, int lane) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  const int n = row_bytes >> 4;
  int v = lane;
  for (; v + 7 * 32 < n; v += 8 * 32) {
    uint4 t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) t[u] = FROM_PEER ? __ldcg(s + v + u * 32) : s[v + u * 32];
#pragma unroll
    for (int u = 0; u < 8; ++u) d[v + u * 32] = t[u];
  }
  for (; v < n; v += 32) d[v] = FROM_PEER ? __ldcg(s + v) : s[v];
}

// Clamp a per-slot count so that the running sum never exceeds `cap`.
__device__ __forceinline__ int clamp_run(int cnt, int run, int64_t cap) {
  const int64_t room = cap - run;
  return static_cast<int>(max64(0, min64(cnt, room)));
}

// True in the last CTA of the grid to get here (ticket), after every thread of every
// CTA fenced its stores at system scope.
__device__ __forceinline__ bool last_cta(uint32_t* ticket, int* s_last) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) *s_last = (atomicAdd(ticket, 1u) == gridDim.x * gridDim.y * gridDim.z - 1);
  __syncthreads();
  return *s_last != 0;
}

// Thread d (< G) of the dispatching kernel's first CTA, before any row moves: d's
// metadata for this source (rows per slot of d clamped to cap_rows, then this source's
// first send row for d), a system fence, then d.meta[rank] += 1 — so a consumer can
// plan its work from the counts while the rows are still in flight.
__device__ __forceinline__ void ep_publish_meta(const EpParams& p, const int32_t* slot_offsets, int d) {
  const int P = p.P;
  int32_t* meta = ep_meta(p.peer[d], p) + p.rank * (P + 1);
  int run = 0;
  for (int q = 0; q < P; ++q) {
    const int c = clamp_run(slot_offsets[d * P + q + 1] - slot_offsets[d * P + q], run, p.cap_rows);
    meta[q] = c;
    run += c;
  }
  meta[P] = slot_offsets[d * P];
  __threadfence_system();
  atomicAdd_system(ep_flags(p.peer[d]) + 2 * p.G + p.rank, 1u);
}

// Thread d (< G) of the last CTA once every row for destination d is stored and fenced:
// d.disp[rank] += 1.  Thread 0 also resets the ticket.
__device__ __forceinline__ void ep_publish_rows(const EpParams& p, int d) {
  __threadfence_system();
  atomicAdd_system(ep_flags(p.peer[d]) + p.rank, 1u);
  if (d == 0) *p.ticket = 0u;
}

// ---- permute / combine (permute.cu)
struct PermuteParams {
  const void* x;
  int64_t x_stride;       // bytes between token rows
  int row_bytes;          // H * elem bytes (multiple of 16)
  int T, K;
  const int32_t* phys_ids;       // [T, K]
  const int32_t* block_offsets;  // [num_slots, nblocks] absolute first row of (slot, block)
  int num_slots, nblocks, tb;
  void* send;                    // [T*K, H], rows packed (stride row_bytes)
  int32_t* pos_of;               // [T, K] destination row of (t, k)
  int64_t* send_token;           // [T*K] token index of each send row (nullable)
  int64_t* send_slot;            // [T*K] top-k slot of each send row (nullable)
  // Peer mode (permute fused with the expert-parallel dispatch): rows go straight to
  // the owning ranks' receive regions instead of `send`; the last CTA writes every
  // destination's metadata and raises its arrival flag.
  int peer_mode = 0;
  const int32_t* slot_offsets = nullptr;  // [num_slots + 1] (router output)
  EpParams ep;
};

struct CombineParams {
  const void* y;          // expert outputs in send order [T*K, H]
  int64_t ldy;            // elements
  int dtype;              // kDtypeBF16 / kDtypeF32 for y, shared and out
  const int32_t* pos_of;  // [T, K]
  const float* topk_w;    // [T, K]
  int T, K, H;
  const void* shared;     // [T, H] shared-expert output or null
  int64_t lds;
  const float* shared_gate;  // [T] or null (gate == 1)
  void* out;              // [T, H]
  int64_t ldo;
  // Peer mode (wait_n > 0): y is this rank's combine region; wait until the G flags
  // wait_flags[0..G) pass *wait_expect, then advance *wait_expect (last CTA, ticket).
  const uint32_t* wait_flags = nullptr;
  int wait_n = 0;
  uint32_t* wait_expect = nullptr;
  uint32_t* wait_ticket = nullptr;
  uint64_t wait_timeout_ns = 0;
  int* status = nullptr;
};

// ---- residual add + RMSNorm (norm.cu)
struct AddNormParams {
  const void* residual;   // [T, H] (row stride ld)
  const void* hidden;     // [T, H] or null (no add)
  const void* weight;     // [H] norm weight (dtype of the activations)
  float eps;
  int T, H, dtype;
  int64_t ld;             // elements, shared by residual / hidden / residual_out
  void* residual_out;     // [T, H] (may alias residual)
  void* normed;           // [T, H] or null (add only)
  int64_t ld_normed;
};

// ---- grouped GEMM (grouped_gemm.cu)
// A rows straight from this rank's exchange receive region (CTA-pair kernel, prefill
// over NVLink): groups are (source, slot) segments instead of expert-major rows, so no
// regroup copy runs, and a tile waits only for its own source's rows.  Sources are
// visited starting with this rank (its rows are local).
struct SegIn {
  const int32_t* meta = nullptr;        // this rank's meta [G][P+1]
  const uint32_t* rows_flag = nullptr;  // this rank's disp flags [G]
  const uint32_t* meta_flag = nullptr;  // this rank's meta flags [G]
  uint32_t* rows_expect = nullptr;      // arrivals consumed so far
  uint32_t* meta_expect = nullptr;
  uint32_t* ticket = nullptr;           // completion ticket of the consuming launch
  int G = 0, rank = 0;
  int64_t cap_rows = 0;
  int64_t comb_rows = 0;  // rows of every rank's combine region (bounds the return rows)
  uint64_t timeout_ns = 0;
  int consume = 0;  // 1: wait for the flags and advance the counters (first GEMM of the layer)
};

// Peer output of the down GEMM (fused combine-send): out_row_map[r] = (s << 24) | row
// sends row r to row `row` of rank s's combine region; after the last tile every CTA
// fences at system scope and the last one adds 1 to flags[G + rank] of every rank.
struct PeerOut {
  uint8_t* base[EP_MAX_RANKS];  // every rank's exchange buffer (flags at offset 0)
  uint8_t* rows[EP_MAX_RANKS];  // every rank's combine region
  int G = 0, rank = 0;
  uint32_t* ticket = nullptr;   // local, zero between launches
};
constexpr int kPeerRowBits = 24;

__device__ __forceinline__ void* peer_out_row(const PeerOut& po, int32_t v, int64_t ld_bytes) {
  return po.rows[static_cast<uint32_t>(v) >> kPeerRowBits] +
         static_cast<int64_t>(v & ((1 << kPeerRowBits) - 1)) * ld_bytes;
}

// End of a peer-output GEMM, run by every thread of every CTA.
__device__ __forceinline__ void peer_out_publish(const PeerOut& po, int* s_last) {
  if (last_cta(po.ticket, s_last) && threadIdx.x < po.G) {
    __threadfence_system();
    atomicAdd_system(ep_flags(po.base[threadIdx.x]) + po.G + po.rank, 1u);
    if (threadIdx.x == 0) *po.ticket = 0u;
  }
}

struct GemmParams {
  const int32_t* expert_offsets;  // [P+1]: rows of expert p are [off[p], off[p+1])
  int P;
  int N;        // output columns (GEMM1: I, GEMM2: H)
  int K;        // reduction length (GEMM1: H, GEMM2: I)
  int w_rows;   // weight rows per expert (GEMM1: 2I, GEMM2: H)
  int up_row;   // GEMM1: row offset of the up block inside an expert (I)
  void* out;    // bf16 [rows, ldo]
  int64_t ldo;  // elements
  const int32_t* out_row_map;  // null, or output row for every input row
  int* status;
  int peer_out = 0;            // 1: rows go to other ranks (PeerOut), out is unused
  PeerOut po;
  int seg_mode = 0;            // 1: A rows are an exchange receive region (SegIn)
  SegIn seg;
  int tile_band = 0;           // CTA-pair kernel: n-tile band of the tile order (0: m fastest)
};

// Grouped-GEMM kernel choice: automatic (by rows per slot), or forced for tests.
enum GemmVariant : int {
  kGemmAuto = 0,
  kGemmTokenMajor = 1,        // M = 128 token rows x N = 256 weight rows (prefill)
  kGemmTokenMajorSmallM = 2,  // 32 token rows per tile, N = 64
  kGemmWeightMajor = 3,       // M = 128 weight rows x N = 32 tokens (decode)
  kGemmTokenMajorPair = 4,    // CTA pairs: M = 256 token rows x N = 256 (cta_group::2)
  kGemmWeightMajorWide = 5,   // weight-major with up to 64-token tiles for slots above 32 rows
};

struct GemmLaunch {
  const void* a;        // [rows_cap, K] bf16 activations, row stride lda
  int64_t rows_cap;
  int64_t lda;
  const void* w;        // [P * w_rows, K] bf16 weights (row stride K)
  GemmParams p;
  int variant = kGemmAuto;
  int64_t rows_hint = 0;  // expected rows (kernel choice); 0: rows_cap
};

// 2D bf16 K-major TMA map (rows x cols, row stride ld elements), box box_rows x 64,
// 128-byte swizzle.  Returns 0 on success.
int make_tma_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows);
// wide: 0 = 32-token tiles, 1 = up to 64-token tiles for slots above 32 rows, -1 = by rows per slot
int launch_grouped_wm(const GemmLaunch& L, bool swiglu, int wide, cudaStream_t stream);
bool pair_gemm_supported(const GemmLaunch& L, bool swiglu);
int launch_grouped_pair(const GemmLaunch& L, bool swiglu, cudaStream_t stream);

struct GemmF32Params {
  const float* a;          // [rows, K]
  int64_t lda;
  int64_t rows_cap;
  const float* w;          // [P, w_rows, K]
  const int32_t* offsets;  // [P+1]
  int P, N, K, w_rows, up_row;
  float* out;
  int64_t ldo;
  const int32_t* out_row_map;
};

int launch_ep_dispatch(const EpParams& p, const void* send, const int32_t* slot_offsets, int64_t max_rows,
                       cudaStream_t stream);
int launch_ep_collect(const EpParams& p, void* xe, int32_t* row_map, int32_t* peer_row_map,
                      int32_t* expert_offsets, uint32_t* expect, uint32_t* meta_expect, uint64_t timeout_ns,
                      int64_t max_rows, cudaStream_t stream);
int launch_ep_combine_send(const EpParams& p, const void* y_recv, int64_t max_rows, cudaStream_t stream);
int launch_ep_wait_comb(const EpParams& p, uint32_t* expect, uint64_t timeout_ns, cudaStream_t stream);

int launch_router_logits(const RouterLogitsParams& p, int x_dtype, cudaStream_t stream);
// Small batches (T <= 8): logits, selection and optionally the block prologue in one
// launch (router.cu).  sp must describe one token block (nblocks 1).
bool router_small_fused_ok(int T, int H, int x_dtype, int num_slots, int scoring, bool has_norm);
// Optional permute outputs of the fused small-batch router (one token block): the send
// rows in (physical slot, t*K+k) order and each entry's send row, exactly as
// permute_rows writes them.
struct SmallPermuteOut {
  void* send = nullptr;       // [T*K, H], row stride row_bytes
  int32_t* pos_of = nullptr;  // [T, K]
  int row_bytes = 0;
};
int launch_router_small_fused(const RouterLogitsParams& lp, const RouterSelectParams& sp, const AddNormParams* np,
                              int x_dtype, cudaStream_t stream, const SmallPermuteOut* po = nullptr);
int launch_grouped_gemm_f32(const GemmF32Params& p, bool swiglu, cudaStream_t stream);
int launch_router_select(const RouterSelectParams& p, cudaStream_t stream);
int launch_permute(const PermuteParams& p, cudaStream_t stream);
int launch_combine(const CombineParams& p, cudaStream_t stream);
int launch_add_rmsnorm(const AddNormParams& p, cudaStream_t stream);
// Return 0, -1 (tensor map encode failed), -3 (launch failed), -4 (P too large).
int launch_grouped_swiglu(const GemmLaunch& L, cudaStream_t stream);
int launch_grouped_down(const GemmLaunch& L, cudaStream_t stream);

}  // namespace b200moe
