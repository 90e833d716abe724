/*
 * b200moe — C ABI of the B200 (sm_100a) expert-parallel MoE layer forward.
 *
 * One shared library, libb200moe.so, exports the hot path of EasyInfra's
 * all-to-all MoE block as plain C entry points: device pointers, sizes and a CUDA
 * stream, no framework types.  Host code (the Python package easyinfra_b200, or a
 * ctypes stub inside EasyInfra itself) owns every buffer; no entry point allocates
 * device memory except b200moe_ep_alloc, which creates the peer-mapped exchange
 * buffer of the expert-parallel path.  Every call is asynchronous on the given stream and returns 0 on
 * success or a negative B200MOE_E* code; b200moe_last_error() describes the last
 * failure of the calling thread.  Conditions that only the device can see (an
 * out-of-range index, a bounded wait that timed out) are recorded in an optional
 * caller-owned device status word (int32, zero == fine) that the caller reads at its
 * next synchronisation point.
 *
 * Layout conventions (all row-major):
 *   x            [T, H]       activations, bf16 (B200MOE_DTYPE_BF16) or fp32
 *   gate_w       [E(+1), H]   router weight (row E = shared-expert gate, optional)
 *   w_gate_up    [P, 2I, H]   bf16, gate rows 0..I-1 then up rows I..2I-1
 *   w_down       [P, H, I]    bf16
 *   phys ids     slot s of rank g is s = g * P + local slot (rank-major)
 *
 * The reference interface each entry point replaces is cited per function
 * (paths relative to the EasyInfra repository).
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200MOE_API __attribute__((visibility("default")))
#else
#define B200MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B200MOE_ABI_VERSION 1

#define B200MOE_OK 0
#define B200MOE_EINVAL (-1)       /* bad argument (null pointer, size, alignment) */
#define B200MOE_ECUDA (-2)        /* CUDA runtime/driver error */
#define B200MOE_EUNSUPPORTED (-3) /* shape or dtype outside what the kernels cover */
#define B200MOE_ENODEVICE (-4)    /* no sm_100 device current */

#define B200MOE_DTYPE_BF16 0
#define B200MOE_DTYPE_F32 1

/* Device status word values (written by kernels, read by the caller). */
#define B200MOE_STATUS_OK 0
#define B200MOE_STATUS_TIMEOUT 1
#define B200MOE_STATUS_CAPACITY 2
#define B200MOE_STATUS_BAD_INDEX 3

/* ABI version of the loaded library (B200MOE_ABI_VERSION it was built with). */
B200MOE_API int b200moe_abi_version(void);

/* Human-readable description of the calling thread's last failed call. */
B200MOE_API const char* b200moe_last_error(void);

/* Tokens per router/permute CTA for a chunk of T tokens (the two calls must agree;
 * both derive it from T). */
B200MOE_API int b200moe_tokens_per_block(int T);

/* Bytes of workspace b200moe_router / b200moe_permute need for T tokens, E1 router
 * columns and num_slots physical slots.  The first 256 + 32768 bytes hold counters
 * (a completion ticket and per-slot totals) that must be zero before the first call
 * on a workspace; every call leaves them zero again, so zero the workspace once at
 * allocation. */
B200MOE_API size_t b200moe_router_workspace_bytes(int T, int E1, int num_slots);

/*
 * Router: logits, fp32 softmax, top-k (ties -> lowest expert id), optional renorm,
 * scaling, rounding to the activation dtype, EPLB replica pick and slot histogram.
 * Replaces Qwen3MoeSparseMoeBlock._routing (easyinfra/models/qwen3_moe/
 * modeling_qwen3_moe.py:255-266) + eplb_map_to_physical_and_record
 * (easyinfra/generation/blocks/moe/base.py:40-64) + _MoeBlock._all_expert_count_compute
 * (base.py:343-364).
 *
 *   x, ldx, x_dtype   [T, H] activations (ldx in elements, 16-byte aligned rows)
 *   gate_w            [E + has_shared_gate, H] same dtype as x
 *   gate_bias         [E + has_shared_gate] fp32 logit bias or NULL (exactly one entry
 *                     per router column: the kernel reads E + has_shared_gate floats)
 *   renorm            norm_topk_prob; scale: routed scaling factor (1.0 = none)
 *   log2phy           [E, max_rep] int32 physical slot per (logical expert, replica)
 *   rep_count         [E] int32 replica count; both NULL -> physical id = logical id
 *   num_slots         G * P physical slots over all ranks
 * Outputs (device): topk_ids [T,K] int32 logical ids, topk_w [T,K] fp32 (already
 * rounded to the activation dtype), phys_ids [T,K] int32, shared_gate [T] fp32
 * sigmoid of the shared-gate logit (only when has_shared_gate), slot_counts
 * [num_slots] int32, slot_offsets [num_slots+1] int32 (exclusive prefix; entry
 * num_slots == T*K).  logits_out [T, E1] fp32 may be NULL; when given, the logits
 * (bf16-rounded for bf16 x) are kept there.
 */
B200MOE_API int b200moe_router(const void* x, int64_t ldx, int x_dtype, const void* gate_w,
                   const float* gate_bias, int has_shared_gate, int T, int H, int E, int K,
                   int renorm, float scale, const int32_t* log2phy, const int32_t* rep_count,
                   int max_rep, int num_slots, int32_t* topk_ids, float* topk_w,
                   int32_t* phys_ids, float* shared_gate, int32_t* slot_counts,
                   int32_t* slot_offsets, float* logits_out, void* workspace,
                   size_t workspace_bytes, int* status, void* stream);

/*
 * The block's stage-1 prologue and the router in one call: residual_out = residual +
 * hidden, normed = weight * rmsnorm(residual_out) (as b200moe_add_rmsnorm, leading
 * dimension ld for residual / hidden / residual_out and ld_normed for normed), then
 * b200moe_router on normed (same remaining arguments).  For T <= 8 (decode) the whole
 * of it is one launch: every router-column CTA builds the normed rows itself and the
 * last CTA selects.  Larger batches, and an in-place add (residual_out overlapping
 * residual with hidden given), run the two calls.  Results are bit-identical to
 * calling b200moe_add_rmsnorm and b200moe_router.  Replaces the routing step of
 * MoeAll2AllBlock.all2all_chunk_routing_compute (easyinfra/generation/blocks/moe/
 * moe_all2all.py:331-343) together with Qwen3MoeSparseMoeBlock._routing
 * (modeling_qwen3_moe.py:255-266).
 */
B200MOE_API int b200moe_add_rmsnorm_router(const void* residual, const void* hidden, const void* norm_weight,
                                           float eps, int64_t ld, void* residual_out, void* normed,
                                           int64_t ld_normed, int x_dtype, const void* gate_w,
                                           const float* gate_bias, int has_shared_gate, int T, int H, int E, int K,
                                           int renorm, float scale, const int32_t* log2phy,
                                           const int32_t* rep_count, int max_rep, int num_slots,
                                           int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                                           float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets,
                                           float* logits_out, void* workspace, size_t workspace_bytes,
                                           int* status, void* stream);

/*
 * b200moe_add_rmsnorm_router followed by b200moe_permute on `normed`: additionally
 * writes send [T*K, H] (rows in (physical slot, t*K+k) order, row stride H elements)
 * and pos_of [T, K] (the send row of each (t, k)), bit-identical to calling
 * b200moe_permute after the router (send_token / send_slot are not produced).  For
 * T <= 8 on one rank it is a single launch: the router's last CTA, which holds the
 * normed rows in shared memory and every slot offset, ranks the entries and writes the
 * send rows itself.  Replaces MoeAll2AllBlock.all2all_chunk_routing_compute's
 * prologue, routing and permutation (easyinfra/generation/blocks/moe/
 * moe_all2all.py:331-356) at decode batch sizes.
 */
B200MOE_API int b200moe_add_rmsnorm_router_permute(const void* residual, const void* hidden,
                                                   const void* norm_weight, float eps, int64_t ld,
                                                   void* residual_out, void* normed, int64_t ld_normed,
                                                   int x_dtype, const void* gate_w, const float* gate_bias,
                                                   int has_shared_gate, int T, int H, int E, int K, int renorm,
                                                   float scale, const int32_t* log2phy, const int32_t* rep_count,
                                                   int max_rep, int num_slots, int32_t* topk_ids, float* topk_w,
                                                   int32_t* phys_ids, float* shared_gate, int32_t* slot_counts,
                                                   int32_t* slot_offsets, float* logits_out, void* send,
                                                   int32_t* pos_of, void* workspace, size_t workspace_bytes,
                                                   int* status, void* stream);

/*
 * Router of the DeepSeek-V3 family: fp32 logits x·W_gᵀ, sigmoid scores, choice =
 * score + correction_bias, keep the topk_group groups (E / n_group consecutive
 * experts each) with the largest sum of their two best choices, top-K over the
 * choices of the kept groups (others count as 0.0), weights = the chosen experts'
 * sigmoid scores, renormalised (+1e-20) when renorm, times scale, rounded to the
 * activation dtype; then the same replica pick, histogram and offsets as
 * b200moe_router.  Replaces DeepseekV3MoEGate.forward (easyinfra/models/deepseek_v3/
 * modeling_deepseek_v3.py:151-203, scoring_func "sigmoid", topk_method "noaux_tc").
 * Ties go to the lowest group / expert id.  Requires E % n_group == 0,
 * n_group <= 32, at least 2 experts per group.  Workspace: b200moe_router_workspace_bytes(T, E, num_slots).
 */
B200MOE_API int b200moe_router_sigmoid_grouped(const void* x, int64_t ldx, int x_dtype, const void* gate_w,
                                               const float* correction_bias, int T, int H, int E, int K,
                                               int n_group, int topk_group, int renorm, float scale,
                                               const int32_t* log2phy, const int32_t* rep_count, int max_rep,
                                               int num_slots, int32_t* topk_ids, float* topk_w,
                                               int32_t* phys_ids, int32_t* slot_counts, int32_t* slot_offsets,
                                               float* logits_out, void* workspace, size_t workspace_bytes,
                                               int* status, void* stream);

/*
 * b200moe_router without a workspace argument: it allocates nothing and takes no
 * caller scratch.  No counterpart in the reference (EasyInfra allocates everything
 * through PyTorch).  For callers that cannot allocate device memory: a plugin handed
 * only input/output device pointers by a host runtime that owns the allocator, or a
 * caller on a latency path where a cudaMalloc (which can synchronise the device) is
 * not acceptable.  The caller still passes every input and output.
 * Scratch is a built-in device array of 8 MiB (ticket + per-block slot counts +
 * logits), held by every GPU that loads the library until the process exits; calls
 * needing more (see b200moe_router_workspace_bytes) return B200MOE_EUNSUPPORTED.
 * The first call on a device looks the array's address up (cudaGetSymbolAddress), so
 * make that first call before any stream capture; the lookup is repeated when the
 * calling thread's current context changes (after cudaDeviceReset, for example), so
 * the first call after such a change must also come before any capture.  All calls share the array and it
 * keeps the last call's contents (each call clears the counter it needs zeroed first):
 * calls that overlap on the GPU race, so serialise them (one stream, or events).
 * It is not usable with b200moe_permute, which needs the workspace of its router call.
 */
B200MOE_API int b200moe_router_noalloc(const void* x, int64_t ldx, int x_dtype, const void* gate_w,
                                       const float* gate_bias, int has_shared_gate, int T, int H, int E,
                                       int K, int renorm, float scale, const int32_t* log2phy,
                                       const int32_t* rep_count, int max_rep, int num_slots,
                                       int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                                       float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets,
                                       float* logits_out, int* status, void* stream);

/*
 * The selection half of b200moe_router on caller-provided logits [T, E1] (fp32,
 * holding bf16-rounded values for a bf16 model).  Used to pin the selection against
 * the reference's own logits bit for bit.  round_bf16 rounds the final weights to
 * bf16 (x.dtype == bfloat16 in the reference).
 */
B200MOE_API int b200moe_router_from_logits(const float* logits, int has_shared_gate, int T, int E, int K,
                               int renorm, float scale, int round_bf16, const int32_t* log2phy,
                               const int32_t* rep_count, int max_rep, int num_slots,
                               int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                               float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets,
                               void* workspace, size_t workspace_bytes, int* status,
                               void* stream);

/*
 * Permute: writes every (token, k) row of x into send [T*K, H] in the order
 * (physical slot, flat index t*K+k) — the reference's stable sort of the physical
 * ids followed by x[send_indices] (easyinfra/generation/blocks/moe/
 * moe_all2all.py:345-351).  Needs the workspace of the b200moe_router call that
 * produced phys_ids (same T, E1, num_slots).  pos_of [T,K] int32 receives the send row
 * of each (t, k); send_token / send_slot [T*K] int64 (nullable) receive the
 * reference's send_indices and send_weight_top_k.
 */
B200MOE_API int b200moe_permute(const void* x, int64_t ldx, int x_dtype, int T, int H, int K, int E1,
                    const int32_t* phys_ids, int num_slots, void* send, int32_t* pos_of,
                    int64_t* send_token, int64_t* send_slot, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * Grouped gate/up GEMM with SwiGLU: act[r, :] = silu(x[r] Wg_e^T) * (x[r] Wu_e^T) for
 * every row r of expert e, rows of expert e being [offsets[e], offsets[e+1]) of x
 * (expert-major).  bf16 in/out, fp32 accumulation, one rounding.  rows_cap is the
 * allocated row count of x and act (>= offsets[P]).
 * Replaces the gate_up projection + act_fn(gate) * up of NativeMoE / TritonExperts
 * (easyinfra/generation/modules/moe/native_moe.py:56-103, base.py:39-42,
 * fused_moe.py:443-459).
 */
B200MOE_API int b200moe_grouped_swiglu(const void* x, int64_t ldx, int64_t rows_cap,
                           const int32_t* expert_offsets, int P, int H, int I,
                           const void* w_gate_up, void* act, int64_t ld_act, int* status,
                           void* stream);

/*
 * Grouped down GEMM: out[map(r), :] = act[r] Wd_e^T (map = identity when out_row_map is
 * NULL).  Replaces the down projection of NativeMoE / TritonExperts
 * (native_moe.py:56-103, fused_moe.py:462-476).
 */
B200MOE_API int b200moe_grouped_down(const void* act, int64_t ld_act, int64_t rows_cap,
                         const int32_t* expert_offsets, int P, int H, int I,
                         const void* w_down, void* out, int64_t ldo,
                         const int32_t* out_row_map, int* status, void* stream);

/*
 * fp32 versions of the two grouped GEMMs (same arguments, fp32 activations, weights
 * and outputs; CUDA-core fp32 arithmetic, no tensor-core rounding of the inputs).
 * For fp32 models, whose reference path (NativeMoE.forward_ep,
 * native_moe.py:56-103) multiplies in fp32.
 */
B200MOE_API int b200moe_grouped_swiglu_f32(const float* x, int64_t ldx, int64_t rows_cap,
                                           const int32_t* expert_offsets, int P, int H, int I,
                                           const float* w_gate_up, float* act, int64_t ld_act,
                                           void* stream);
B200MOE_API int b200moe_grouped_down_f32(const float* act, int64_t ld_act, int64_t rows_cap,
                                         const int32_t* expert_offsets, int P, int H, int I,
                                         const float* w_down, float* out, int64_t ldo,
                                         const int32_t* out_row_map, void* stream);

/*
 * Combine / weighted unpermute: out[t] = sum_k topk_w[t,k] * y[pos_of[t,k]]
 * (+ shared_gate[t] * shared[t] when shared != NULL; gate 1 when shared_gate == NULL),
 * fp32 accumulation, one rounding to the output dtype.  Replaces
 * MoeAll2AllBlock._all2all_chunk_output_compute (easyinfra/generation/blocks/moe/
 * moe_all2all.py:291-307) and the shared-expert residual add (:536-537).
 */
B200MOE_API int b200moe_combine(const void* y, int64_t ldy, int dtype, const int32_t* pos_of,
                    const float* topk_w, int T, int K, int H, const void* shared, int64_t lds,
                    const float* shared_gate, void* out, int64_t ldo, void* stream);

/*
 * MoE block prologue: residual_out = residual + hidden (rounded to the dtype; hidden
 * may be NULL: no add), normed = weight * rmsnorm(residual_out) with the reference's
 * rounding points (fp32 statistics, rounded before and after the weight multiply;
 * normed may be NULL: add only).  Replaces _add_to_residual + post_attention_layernorm
 * in MoeAll2AllBlock.all2all_chunk_routing_compute (easyinfra/generation/blocks/moe/
 * moe_all2all.py:331-335; _rmsnorm at generation/modules/rmsnorm/base_rmsnorm.py:6-12).
 * residual_out may alias residual.
 */
B200MOE_API int b200moe_add_rmsnorm(const void* residual, const void* hidden, const void* weight,
                                    float eps, int T, int H, int dtype, int64_t ld,
                                    void* residual_out, void* normed, int64_t ld_normed,
                                    void* stream);

/*
 * Row-segment gather used around the expert-parallel all-to-all: for each segment i,
 * copies rows [src_start[i], src_start[i] + len[i]) of src to rows
 * [dst_start[i], ...) of dst (row_bytes each, multiple of 16).  Segment tables are
 * device int32 arrays; max_rows bounds every len[i].  dst_to_src (nullable, int32)
 * receives, for every written dst row, the src row it came from.  Turns the received
 * [source rank][local expert] layout (moe_all2all.py:441-444) into the expert-major
 * layout the grouped GEMMs read; dst_to_src then serves as b200moe_grouped_down's
 * out_row_map to write results back in received order.
 */
B200MOE_API int b200moe_gather_segments(const void* src, void* dst, int64_t row_bytes,
                            const int32_t* src_start, const int32_t* dst_start,
                            const int32_t* len, int nseg, int64_t max_rows,
                            int32_t* dst_to_src, void* stream);

/*
 * Grouped GEMMs with a row-count hint: as b200moe_grouped_swiglu / b200moe_grouped_down,
 * but the kernel (weight-major for decode, token-major for prefill) is chosen from
 * rows_hint, the expected row count, instead of rows_cap.  For callers whose
 * activation buffer is sized for the worst case while the rows live on the device
 * (the peer exchange below).  rows_hint 0 behaves like the plain entry points.
 * No counterpart in the reference (its all-to-all path knows the row count on the host).
 */
B200MOE_API int b200moe_grouped_swiglu_ex(const void* x, int64_t ldx, int64_t rows_cap, int64_t rows_hint,
                                          const int32_t* expert_offsets, int P, int H, int I,
                                          const void* w_gate_up, void* act, int64_t ld_act, int* status,
                                          void* stream);
B200MOE_API int b200moe_grouped_down_ex(const void* act, int64_t ld_act, int64_t rows_cap, int64_t rows_hint,
                                        const int32_t* expert_offsets, int P, int H, int I,
                                        const void* w_down, void* out, int64_t ldo,
                                        const int32_t* out_row_map, int* status, void* stream);

/*
 * Expert-parallel token exchange over NVLink peer memory (one process per GPU).
 *
 * Replaces the count all-gather, the host synchronisation and the two NCCL
 * all_to_all_single calls of MoeAll2AllBlock (easyinfra/generation/blocks/moe/
 * moe_all2all.py:397-444 dispatch, :560-591 combine; GroupCommunicator.all_to_all_single,
 * easyinfra/generation/parallel/communicator.py:269) with four stream-ordered launches that need
 * no host round trip and can be captured in a CUDA graph:
 *   b200moe_ep_dispatch      send rows (router send order, rank-major slots) -> the
 *                            owning ranks' buffers, then raise their arrival flags;
 *   b200moe_ep_collect       wait for every rank's rows, regroup them expert-major
 *                            (x for the grouped GEMMs), write expert_offsets [P+1] and
 *                            row_map (the down GEMM's out_row_map);
 *   b200moe_ep_combine_send  down-GEMM rows (arrival order, y_recv) -> the sources'
 *                            combine regions at their send positions, raise flags;
 *   b200moe_ep_wait_combine  wait until every rank returned this rank's rows; the
 *                            combine region (b200moe_ep_layout comb_offset) then holds
 *                            the expert outputs in send order for b200moe_combine.
 * Each rank creates one buffer with b200moe_ep_alloc, exchanges the 64-byte handles
 * (any host collective), maps every peer's with b200moe_ep_open and fills a
 * b200moe_ep_desc.  counters (16 x uint32, device, zeroed once) hold the kernels'
 * tickets and how many arrivals this rank consumed; every rank must issue the four
 * calls in the same order.  Every wait is bounded by timeout_ns; on timeout the
 * status word gets B200MOE_STATUS_TIMEOUT and the kernel proceeds with what arrived
 * (the caller must treat the layer output as invalid).  timeout_ns == 0 checks each
 * flag once without waiting: for running all ranks' launches in stream order on a
 * single device.
 */
#define B200MOE_EP_MAX_RANKS 8
#define B200MOE_EP_HANDLE_BYTES 64

typedef struct b200moe_ep_desc {
  void* peer[B200MOE_EP_MAX_RANKS]; /* every rank's exchange buffer, as mapped in this process */
  int world_size;                   /* G <= B200MOE_EP_MAX_RANKS */
  int rank;
  int slots_per_rank;               /* P */
  int row_bytes;                    /* H * element bytes, multiple of 16 */
  int64_t cap_rows;                 /* rows one source may send to one rank */
  int64_t comb_rows;                /* rows this rank sends per layer at most (T * K) */
  uint32_t* counters;               /* device, 16 x uint32, zero before the first call */
  int* status;                      /* device status word (nullable) */
  uint64_t timeout_ns;
} b200moe_ep_desc;

/* Byte offsets inside every rank's exchange buffer and its total size. */
B200MOE_API int b200moe_ep_layout(int world_size, int slots_per_rank, int64_t cap_rows, int64_t comb_rows,
                                  int row_bytes, int64_t* recv_offset, int64_t* comb_offset,
                                  int64_t* total_bytes);
/* Allocate and zero this rank's exchange buffer on the current device; writes its
 * inter-process handle (B200MOE_EP_HANDLE_BYTES). */
B200MOE_API int b200moe_ep_alloc(size_t bytes, void** buffer, void* handle);
/* Map a peer's buffer from its handle (enables peer access on first use). */
B200MOE_API int b200moe_ep_open(const void* handle, void** peer_buffer);
B200MOE_API int b200moe_ep_close(void* peer_buffer);
B200MOE_API int b200moe_ep_free(void* buffer);

B200MOE_API int b200moe_ep_dispatch(const b200moe_ep_desc* ep, const void* send, const int32_t* slot_offsets,
                                    int64_t send_rows, void* stream);
/* row_map (nullable): arrival row of every expert-major row, for b200moe_grouped_down's
 * out_row_map; peer_row_map (nullable): (source rank << 24) | row in that rank's
 * combine region, for b200moe_ep_grouped_down_send.  At least one of the two. */
B200MOE_API int b200moe_ep_collect(const b200moe_ep_desc* ep, void* x_expert, int32_t* row_map,
                                   int32_t* peer_row_map, int32_t* expert_offsets, int64_t rows_hint,
                                   void* stream);
B200MOE_API int b200moe_ep_combine_send(const b200moe_ep_desc* ep, const void* y_recv, int64_t rows_hint,
                                        void* stream);
B200MOE_API int b200moe_ep_wait_combine(const b200moe_ep_desc* ep, void* stream);

/*
 * Fused forms of the exchange (same protocol, fewer launches and HBM passes):
 *   b200moe_ep_permute_dispatch   b200moe_permute + b200moe_ep_dispatch: each token row
 *                                 is read once and stored straight into the owning
 *                                 ranks' receive regions (no send buffer); pos_of as in
 *                                 b200moe_permute (send positions, for the combine).
 *                                 slot_offsets and workspace are the router call's.
 *                                 Launched even when T == 0 (it publishes empty counts).
 *   b200moe_ep_grouped_down_send  b200moe_grouped_down + b200moe_ep_combine_send: the
 *                                 epilogue stores each output row into the combine
 *                                 region of the rank that sent it (peer_row_map from
 *                                 b200moe_ep_collect), so the NVLink stores overlap the
 *                                 tensor-core work; the last CTA raises the flags.
 *   b200moe_ep_combine            b200moe_ep_wait_combine + b200moe_combine on this rank's
 *                                 combine region: every CTA waits (bounded) for the
 *                                 flags, then gathers; always launched (it consumes the
 *                                 flags even when T == 0).
 */
B200MOE_API int b200moe_ep_permute_dispatch(const b200moe_ep_desc* ep, const void* x, int64_t ldx, int x_dtype,
                                            int T, int H, int K, int E1, const int32_t* phys_ids,
                                            const int32_t* slot_offsets, int32_t* pos_of, void* workspace,
                                            size_t workspace_bytes, void* stream);
B200MOE_API int b200moe_ep_grouped_down_send(const b200moe_ep_desc* ep, const void* act, int64_t ld_act,
                                             int64_t rows_cap, int64_t rows_hint, const int32_t* expert_offsets,
                                             int P, int H, int I, const void* w_down,
                                             const int32_t* peer_row_map, int* status, void* stream);
/*
 * Prefill without the regroup copy: the CTA-pair grouped GEMMs read this rank's
 * receive region directly, one tile group per (source rank, local slot) segment,
 * sources visited from this rank onwards.  b200moe_ep_grouped_swiglu_recv waits
 * (bounded) for every source's counts, plans its tiles from them, and lets each tile
 * wait only for its own source's rows — so the GEMM starts on local rows while the
 * other ranks' rows are still crossing NVLink; act gets the SwiGLU rows in
 * receive-region order (world_size * cap_rows rows).  b200moe_ep_grouped_down_send_recv
 * then returns every down-projection row straight into the combine region of the rank
 * that sent it (as b200moe_ep_grouped_down_send).  Use in place of b200moe_ep_collect
 * + the two GEMMs, after b200moe_ep_permute_dispatch; needs I % 128 == 0,
 * H % 256 == 0 and world_size * slots_per_rank <= 512.
 */
B200MOE_API int b200moe_ep_grouped_swiglu_recv(const b200moe_ep_desc* ep, const void* w_gate_up, int P, int H,
                                               int I, void* act, int64_t ld_act, int* status, void* stream);
B200MOE_API int b200moe_ep_grouped_down_send_recv(const b200moe_ep_desc* ep, const void* act, int64_t ld_act,
                                                  const void* w_down, int P, int H, int I, int* status,
                                                  void* stream);
B200MOE_API int b200moe_ep_combine(const b200moe_ep_desc* ep, const int32_t* pos_of, const float* topk_w, int T,
                                   int K, int H, int dtype, const void* shared, int64_t lds,
                                   const float* shared_gate, void* out, int64_t ldo, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
