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
};

// Grouped-GEMM kernel choice: automatic (by rows per slot), or forced for tests.
enum GemmVariant : int {
  kGemmAuto = 0,
  kGemmTokenMajor = 1,        // M = 128 token rows x N = 256 weight rows (prefill)
  kGemmTokenMajorSmallM = 2,  // 32 token rows per tile, N = 64
  kGemmWeightMajor = 3,       // M = 128 weight rows x N = 32 tokens (decode)
};

struct GemmLaunch {
  const void* a;        // [rows_cap, K] bf16 activations, row stride lda
  int64_t rows_cap;
  int64_t lda;
  const void* w;        // [P * w_rows, K] bf16 weights (row stride K)
  GemmParams p;
  int variant = kGemmAuto;
};

// 2D bf16 K-major TMA map (rows x cols, row stride ld elements), box box_rows x 64,
// 128-byte swizzle.  Returns 0 on success.
int make_tma_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows);
int launch_grouped_wm(const GemmLaunch& L, bool swiglu, cudaStream_t stream);

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

int launch_router_logits(const RouterLogitsParams& p, int x_dtype, cudaStream_t stream);
int launch_grouped_gemm_f32(const GemmF32Params& p, bool swiglu, cudaStream_t stream);
int launch_router_select(const RouterSelectParams& p, cudaStream_t stream);
int launch_permute(const PermuteParams& p, cudaStream_t stream);
int launch_combine(const CombineParams& p, cudaStream_t stream);
int launch_add_rmsnorm(const AddNormParams& p, cudaStream_t stream);
// Return 0, -1 (tensor map encode failed), -3 (launch failed), -4 (P too large).
int launch_grouped_swiglu(const GemmLaunch& L, cudaStream_t stream);
int launch_grouped_down(const GemmLaunch& L, cudaStream_t stream);

}  // namespace b200moe
