// C-ABI entry points of libb200moe.so (declared in include/b200moe.h).
//
// This layer validates arguments, lays out the router workspace, picks kernel
// configurations and launches on the caller's stream.  It never throws across the
// ABI and allocates device memory only in b200moe_ep_alloc (the exchange buffer).
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/b200moe.h"
#include "kernels.cuh"

namespace b200moe {

bool pdl_enabled() {
  static const bool enabled = [] {
    const char* v = getenv("B200MOE_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return enabled;
}

int num_sms() {
  static std::atomic<int> cached[64];  // zero-initialised (static storage)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int gemm_grid_limit() {
  const int n = num_sms();
  const char* v = getenv("B200MOE_GEMM_MAX_CTAS");
  if (v == nullptr) return n;
  const int cap = atoi(v);
  return (cap >= 2 && cap < n) ? cap : n;
}

// ------------------------------------------------------------------ segment gather
__global__ void __launch_bounds__(256) gather_segments_kernel(const uint8_t* src, uint8_t* dst,
                                                              int64_t row_bytes,
                                                              const int32_t* src_start,
                                                              const int32_t* dst_start,
                                                              const int32_t* len, int rows_per_cta,
                                                              int32_t* dst_to_src) {
  pdl_trigger();
  pdl_wait();
  const int seg = blockIdx.y;
  const int n = len[seg];
  const int r0 = blockIdx.x * rows_per_cta;
  if (r0 >= n) return;
  const int r1 = min(n, r0 + rows_per_cta);
  const int64_t vec = row_bytes / 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = r0 + warp; r < r1; r += blockDim.x >> 5) {
    const uint4* s = reinterpret_cast<const uint4*>(src + (static_cast<int64_t>(src_start[seg]) + r) * row_bytes);
    uint4* d = reinterpret_cast<uint4*>(dst + (static_cast<int64_t>(dst_start[seg]) + r) * row_bytes);
    int64_t v = lane;
    for (; v + 7 * 32 < vec; v += 8 * 32) {  // eight loads in flight per lane
      uint4 t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = __ldg(s + v + u * 32);
#pragma unroll
      for (int u = 0; u < 8; ++u) d[v + u * 32] = t[u];
    }
    for (; v < vec; v += 32) d[v] = __ldg(s + v);
    if (dst_to_src != nullptr && lane == 0) dst_to_src[dst_start[seg] + r] = src_start[seg] + r;
  }
}

}  // namespace b200moe

using namespace b200moe;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B200MOE_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return B200MOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// B200MOE_GEMM_VARIANT=token|token_small|weight|weight_wide|pair forces one grouped-GEMM kernel
// (tuning and tests); unset or "auto" picks by rows per slot.
int gemm_variant_from_env() {
  const char* v = getenv("B200MOE_GEMM_VARIANT");
  if (v == nullptr || strcmp(v, "auto") == 0) return kGemmAuto;
  if (strcmp(v, "token") == 0) return kGemmTokenMajor;
  if (strcmp(v, "token_small") == 0) return kGemmTokenMajorSmallM;
  if (strcmp(v, "weight") == 0) return kGemmWeightMajor;
  if (strcmp(v, "weight_wide") == 0) return kGemmWeightMajorWide;
  if (strcmp(v, "pair") == 0) return kGemmTokenMajorPair;
  return kGemmAuto;
}

constexpr size_t kTicketBytes = 256;
constexpr int kMaxSlots = 8192;
constexpr size_t kTotalsBytes = kMaxSlots * sizeof(int32_t);
// Counters at the start of a router workspace that must be zero before a call (every
// call leaves them zero again).
constexpr size_t kCounterBytes = kTicketBytes + kTotalsBytes;

int tokens_per_block(int T) {
  if (T > 32768) return 64;  // at most 1024 token blocks up to 65536 tokens
  if (T >= 16384) return 32;
  if (T >= 4096) return 16;
  return 8;
}

int nblocks_for(int T) {
  const int tb = tokens_per_block(T);
  return (T + tb - 1) / tb;
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct RouterWs {
  uint32_t* ticket;
  int32_t* slot_totals;
  int32_t* block_counts;
  float* logits;
  size_t bytes;
};

RouterWs router_ws_layout(void* base, int T, int E1, int num_slots) {
  RouterWs w;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  w.ticket = reinterpret_cast<uint32_t*>(p);
  off += kTicketBytes;
  w.slot_totals = reinterpret_cast<int32_t*>(p + off);  // fixed place and size: always zero between calls
  off += kTotalsBytes;
  w.block_counts = reinterpret_cast<int32_t*>(p + off);
  off += align256(static_cast<size_t>(num_slots) * nblocks_for(T) * sizeof(int32_t));
  w.logits = reinterpret_cast<float*>(p + off);
  off += align256(static_cast<size_t>(T) * E1 * sizeof(float));
  w.bytes = off;
  return w;
}

int device_ok() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(B200MOE_ENODEVICE, "no CUDA device");
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return fail(B200MOE_ENODEVICE, "device %d is sm_%d0, this library is built for sm_100a", dev, major);
  return B200MOE_OK;
}

int select_common(const float* logits, int has_shared_gate, int T, int E, int K, int renorm,
                  float scale, int round_bf16, const int32_t* log2phy, const int32_t* rep_count,
                  int max_rep, int num_slots, int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                  float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets,
                  const RouterWs& ws, int* status, cudaStream_t stream, int scoring = 0,
                  int n_group = 1, int topk_group = 1, const float* correction_bias = nullptr,
                  const RouterLogitsParams* fuse_lp = nullptr, const AddNormParams* fuse_np = nullptr,
                  int x_dtype = 0, const SmallPermuteOut* fuse_po = nullptr) {
  RouterSelectParams s;
  s.scoring = scoring;
  s.n_group = n_group;
  s.topk_group = topk_group;
  s.correction_bias = correction_bias;
  s.logits = logits;
  s.T = T;
  s.E = E;
  s.E1 = E + (has_shared_gate ? 1 : 0);
  s.K = K;
  s.renorm = renorm;
  s.scale = scale;
  s.round_bf16 = round_bf16;
  s.has_shared_gate = has_shared_gate;
  s.log2phy = log2phy;
  s.rep_count = rep_count;
  s.max_rep = max_rep;
  s.num_slots = num_slots;
  s.tb = tokens_per_block(T);
  s.nblocks = nblocks_for(T);
  s.topk_ids = topk_ids;
  s.topk_w = topk_w;
  s.phys_ids = phys_ids;
  s.shared_gate = shared_gate;
  s.block_counts = ws.block_counts;
  s.slot_totals = ws.slot_totals;
  s.slot_counts = slot_counts;
  s.slot_offsets = slot_offsets;
  s.ticket = ws.ticket;
  s.status = status;
  if (fuse_lp != nullptr) {
    // logits (and the prologue) fused with the selection: one launch for small batches
    if (launch_router_small_fused(*fuse_lp, s, fuse_np, x_dtype, stream, fuse_po))
      return fail(B200MOE_ECUDA, "router_small_fused: %s", cudaGetErrorString(cudaGetLastError()));
    return check_launch("router_small_fused");
  }
  launch_router_select(s, stream);
  return check_launch("router_select");
}

int check_select_args(int T, int E, int K, int num_slots, const int32_t* log2phy,
                      const int32_t* rep_count, int max_rep, const void* topk_ids,
                      const void* topk_w, const void* phys_ids, const void* slot_counts,
                      const void* slot_offsets, int has_shared_gate, const void* shared_gate) {
  if (T < 0) return fail(B200MOE_EINVAL, "T=%d < 0", T);
  if (T > 65536) return fail(B200MOE_EUNSUPPORTED, "T=%d above 65536 tokens per call", T);
  if (E < 1 || E > 256) return fail(B200MOE_EUNSUPPORTED, "E=%d outside [1, 256]", E);
  if (K < 1 || K > 8 || K > E) return fail(B200MOE_EUNSUPPORTED, "K=%d outside [1, min(8, E)]", K);
  if (num_slots < 1 || num_slots > kMaxSlots) return fail(B200MOE_EUNSUPPORTED, "num_slots=%d", num_slots);
  if ((log2phy == nullptr) != (rep_count == nullptr))
    return fail(B200MOE_EINVAL, "log2phy and rep_count must both be given or both be NULL");
  if (log2phy == nullptr && num_slots < E)
    return fail(B200MOE_EINVAL, "num_slots=%d < E=%d without a placement map", num_slots, E);
  if (log2phy != nullptr && max_rep < 1) return fail(B200MOE_EINVAL, "max_rep=%d", max_rep);
  if (!slot_counts || !slot_offsets) return fail(B200MOE_EINVAL, "null slot_counts/slot_offsets");
  if (T > 0 && (!topk_ids || !topk_w || !phys_ids)) return fail(B200MOE_EINVAL, "null output pointer");
  if (T > 0 && has_shared_gate && !shared_gate) return fail(B200MOE_EINVAL, "shared_gate output is NULL");
  return B200MOE_OK;
}

// A chunk without tokens still reports (zero) counts and offsets: a rank with no
// tokens takes part in the count exchange like any other.
int zero_counts(int32_t* slot_counts, int32_t* slot_offsets, int num_slots, cudaStream_t stream) {
  if (cudaMemsetAsync(slot_counts, 0, sizeof(int32_t) * num_slots, stream) != cudaSuccess ||
      cudaMemsetAsync(slot_offsets, 0, sizeof(int32_t) * (num_slots + 1), stream) != cudaSuccess)
    return fail(B200MOE_ECUDA, "zeroing slot counts: %s", cudaGetErrorString(cudaGetLastError()));
  return B200MOE_OK;
}

}  // namespace

extern "C" {

int b200moe_abi_version(void) { return B200MOE_ABI_VERSION; }

const char* b200moe_last_error(void) { return g_err; }

int b200moe_tokens_per_block(int T) { return tokens_per_block(T); }

size_t b200moe_router_workspace_bytes(int T, int E1, int num_slots) {
  if (T < 0 || E1 < 0 || num_slots < 0) return 0;
  return router_ws_layout(nullptr, T, E1, num_slots).bytes;
}

int b200moe_router(const void* x, int64_t ldx, int x_dtype, const void* gate_w,
                   const float* gate_bias, int has_shared_gate, int T, int H, int E, int K,
                   int renorm, float scale, const int32_t* log2phy, const int32_t* rep_count,
                   int max_rep, int num_slots, int32_t* topk_ids, float* topk_w,
                   int32_t* phys_ids, float* shared_gate, int32_t* slot_counts,
                   int32_t* slot_offsets, float* logits_out, void* workspace,
                   size_t workspace_bytes, int* status, void* stream) {
  int rc = check_select_args(T, E, K, num_slots, log2phy, rep_count, max_rep, topk_ids, topk_w,
                             phys_ids, slot_counts, slot_offsets, has_shared_gate, shared_gate);
  if (rc) return rc;
  if ((rc = device_ok())) return rc;
  if (x_dtype != B200MOE_DTYPE_BF16 && x_dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "x_dtype=%d", x_dtype);
  if (T == 0) return zero_counts(slot_counts, slot_offsets, num_slots, static_cast<cudaStream_t>(stream));
  if (!x || !gate_w || !workspace) return fail(B200MOE_EINVAL, "null input or workspace");
  if (H <= 0 || H % 8 != 0) return fail(B200MOE_EUNSUPPORTED, "H=%d must be a positive multiple of 8", H);
  if (ldx < H || (ldx * dtype_bytes(x_dtype)) % 16 != 0 || !aligned16(x) || !aligned16(gate_w))
    return fail(B200MOE_EINVAL, "x/gate_w must be 16-byte aligned with 16-byte row stride (ldx=%lld)",
                static_cast<long long>(ldx));
  const int E1 = E + (has_shared_gate ? 1 : 0);
  const RouterWs ws = router_ws_layout(workspace, T, E1, num_slots);
  if (workspace_bytes < ws.bytes)
    return fail(B200MOE_EINVAL, "workspace too small: %zu < %zu", workspace_bytes, ws.bytes);
  if (T == 0) return B200MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RouterLogitsParams lp;
  lp.x = x;
  lp.ldx = ldx;
  lp.w = gate_w;
  lp.bias = gate_bias;
  lp.T = T;
  lp.H = H;
  lp.E1 = E1;
  lp.logits = logits_out ? logits_out : ws.logits;
  const bool fuse = router_small_fused_ok(T, H, x_dtype, num_slots, 0, false);
  if (!fuse) {
    if (launch_router_logits(lp, x_dtype, st)) return fail(B200MOE_ECUDA, "router_logits: kernel setup failed");
    if ((rc = check_launch("router_logits"))) return rc;
  }
  return select_common(lp.logits, has_shared_gate, T, E, K, renorm, scale,
                       x_dtype == B200MOE_DTYPE_BF16, log2phy, rep_count, max_rep, num_slots,
                       topk_ids, topk_w, phys_ids, shared_gate, slot_counts, slot_offsets, ws,
                       status, st, 0, 1, 1, nullptr, fuse ? &lp : nullptr, nullptr, x_dtype);
}

}  // extern "C"

namespace {

// b200moe_add_rmsnorm_router, and with `send` / `pos_of` also the permute of the routed
// rows (b200moe_add_rmsnorm_router_permute): fused into the one launch for T <= 8,
// otherwise b200moe_permute after the router.
int add_rmsnorm_router_impl(const void* residual, const void* hidden, const void* norm_weight, float eps,
                            int64_t ld, void* residual_out, void* normed, int64_t ld_normed, int x_dtype,
                            const void* gate_w, const float* gate_bias, int has_shared_gate, int T, int H, int E,
                            int K, int renorm, float scale, const int32_t* log2phy, const int32_t* rep_count,
                            int max_rep, int num_slots, int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                            float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets, float* logits_out,
                            void* workspace, size_t workspace_bytes, int* status, void* stream, void* send,
                            int32_t* pos_of) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (x_dtype != B200MOE_DTYPE_BF16 && x_dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "x_dtype=%d", x_dtype);
  const int eb = dtype_bytes(x_dtype);
  if (T > 0 && (!residual || !norm_weight || !residual_out || !normed))
    return fail(B200MOE_EINVAL, "null prologue pointer");
  if (T > 0 && (!aligned16(residual) || !aligned16(residual_out) || !aligned16(normed) ||
                (hidden && !aligned16(hidden)) || !aligned16(norm_weight) || (ld * eb) % 16 != 0 ||
                (ld_normed * eb) % 16 != 0 || ld < H || ld_normed < H))
    return fail(B200MOE_EINVAL, "prologue rows must be 16-byte aligned with 16-byte strides");
  const bool with_permute = send != nullptr || pos_of != nullptr;
  if (with_permute && (!send || !pos_of || !aligned16(send) || (static_cast<int64_t>(H) * eb) % 16 != 0))
    return fail(B200MOE_EINVAL, "send and pos_of must both be given, send 16-byte aligned with 16-byte rows");
  // The fused kernel writes residual_out from its first CTA while the others still read
  // residual: an in-place add runs the separate kernels (one CTA per row) instead.
  const int64_t span = T > 0 ? ((T - 1) * ld + H) * eb : 0;
  const char* r0 = static_cast<const char*>(residual);
  const char* o0 = static_cast<const char*>(residual_out);
  const bool in_place = hidden != nullptr && T > 0 && o0 < r0 + span && r0 < o0 + span;
  const bool fuse = !in_place && router_small_fused_ok(T, H, x_dtype, num_slots, 0, true);
  if (!fuse) {
    // the prologue kernel, then the router on its output (then the permute)
    if ((rc = b200moe_add_rmsnorm(residual, hidden, norm_weight, eps, T, H, x_dtype, ld, residual_out, normed,
                                  ld_normed, stream)))
      return rc;
    if ((rc = b200moe_router(normed, ld_normed, x_dtype, gate_w, gate_bias, has_shared_gate, T, H, E, K, renorm,
                             scale, log2phy, rep_count, max_rep, num_slots, topk_ids, topk_w, phys_ids, shared_gate,
                             slot_counts, slot_offsets, logits_out, workspace, workspace_bytes, status, stream)))
      return rc;
    if (!with_permute) return B200MOE_OK;
    return b200moe_permute(normed, ld_normed, x_dtype, T, H, K, E + (has_shared_gate ? 1 : 0), phys_ids, num_slots,
                           send, pos_of, nullptr, nullptr, workspace, workspace_bytes, stream);
  }
  rc = check_select_args(T, E, K, num_slots, log2phy, rep_count, max_rep, topk_ids, topk_w, phys_ids, slot_counts,
                         slot_offsets, has_shared_gate, shared_gate);
  if (rc) return rc;
  if (!gate_w || !workspace || !aligned16(gate_w)) return fail(B200MOE_EINVAL, "null or misaligned gate_w / workspace");
  const int E1 = E + (has_shared_gate ? 1 : 0);
  const RouterWs ws = router_ws_layout(workspace, T, E1, num_slots);
  if (workspace_bytes < ws.bytes)
    return fail(B200MOE_EINVAL, "workspace too small: %zu < %zu", workspace_bytes, ws.bytes);
  AddNormParams np;
  np.residual = residual;
  np.hidden = hidden;
  np.weight = norm_weight;
  np.eps = eps;
  np.T = T;
  np.H = H;
  np.dtype = x_dtype;
  np.ld = ld;
  np.residual_out = residual_out;
  np.normed = normed;
  np.ld_normed = ld_normed;
  RouterLogitsParams lp;
  lp.x = normed;
  lp.ldx = ld_normed;
  lp.w = gate_w;
  lp.bias = gate_bias;
  lp.T = T;
  lp.H = H;
  lp.E1 = E1;
  lp.logits = logits_out ? logits_out : ws.logits;
  SmallPermuteOut po;
  po.send = send;
  po.pos_of = pos_of;
  po.row_bytes = H * eb;
  return select_common(lp.logits, has_shared_gate, T, E, K, renorm, scale, x_dtype == B200MOE_DTYPE_BF16, log2phy,
                       rep_count, max_rep, num_slots, topk_ids, topk_w, phys_ids, shared_gate, slot_counts,
                       slot_offsets, ws, status, static_cast<cudaStream_t>(stream), 0, 1, 1, nullptr, &lp, &np,
                       x_dtype, with_permute ? &po : nullptr);
}

}  // namespace

extern "C" {

int b200moe_add_rmsnorm_router(const void* residual, const void* hidden, const void* norm_weight, float eps,
                               int64_t ld, void* residual_out, void* normed, int64_t ld_normed, int x_dtype,
                               const void* gate_w, const float* gate_bias, int has_shared_gate, int T, int H, int E,
                               int K, int renorm, float scale, const int32_t* log2phy, const int32_t* rep_count,
                               int max_rep, int num_slots, int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                               float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets, float* logits_out,
                               void* workspace, size_t workspace_bytes, int* status, void* stream) {
  return add_rmsnorm_router_impl(residual, hidden, norm_weight, eps, ld, residual_out, normed, ld_normed, x_dtype,
                                 gate_w, gate_bias, has_shared_gate, T, H, E, K, renorm, scale, log2phy, rep_count,
                                 max_rep, num_slots, topk_ids, topk_w, phys_ids, shared_gate, slot_counts,
                                 slot_offsets, logits_out, workspace, workspace_bytes, status, stream, nullptr,
                                 nullptr);
}

int b200moe_add_rmsnorm_router_permute(const void* residual, const void* hidden, const void* norm_weight, float eps,
                                       int64_t ld, void* residual_out, void* normed, int64_t ld_normed, int x_dtype,
                                       const void* gate_w, const float* gate_bias, int has_shared_gate, int T, int H,
                                       int E, int K, int renorm, float scale, const int32_t* log2phy,
                                       const int32_t* rep_count, int max_rep, int num_slots, int32_t* topk_ids,
                                       float* topk_w, int32_t* phys_ids, float* shared_gate, int32_t* slot_counts,
                                       int32_t* slot_offsets, float* logits_out, void* send, int32_t* pos_of,
                                       void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (T > 0 && (send == nullptr || pos_of == nullptr)) return fail(B200MOE_EINVAL, "null send / pos_of");
  return add_rmsnorm_router_impl(residual, hidden, norm_weight, eps, ld, residual_out, normed, ld_normed, x_dtype,
                                 gate_w, gate_bias, has_shared_gate, T, H, E, K, renorm, scale, log2phy, rep_count,
                                 max_rep, num_slots, topk_ids, topk_w, phys_ids, shared_gate, slot_counts,
                                 slot_offsets, logits_out, workspace, workspace_bytes, status, stream, send, pos_of);
}


int b200moe_router_sigmoid_grouped(const void* x, int64_t ldx, int x_dtype, const void* gate_w,
                                   const float* correction_bias, int T, int H, int E, int K,
                                   int n_group, int topk_group, int renorm, float scale,
                                   const int32_t* log2phy, const int32_t* rep_count, int max_rep,
                                   int num_slots, int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                                   int32_t* slot_counts, int32_t* slot_offsets, float* logits_out,
                                   void* workspace, size_t workspace_bytes, int* status, void* stream) {
  int rc = check_select_args(T, E, K, num_slots, log2phy, rep_count, max_rep, topk_ids, topk_w,
                             phys_ids, slot_counts, slot_offsets, 0, nullptr);
  if (rc) return rc;
  if ((rc = device_ok())) return rc;
  if (n_group < 1 || n_group > 32 || E % n_group != 0 || E / n_group < 2 || topk_group < 1 ||
      topk_group > n_group || K > topk_group * (E / n_group))
    return fail(B200MOE_EUNSUPPORTED, "E=%d n_group=%d topk_group=%d K=%d: need E %% n_group == 0, "
                "n_group <= 32, >= 2 experts per group, K <= kept experts", E, n_group, topk_group, K);
  if (x_dtype != B200MOE_DTYPE_BF16 && x_dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "x_dtype=%d", x_dtype);
  if (T == 0) return zero_counts(slot_counts, slot_offsets, num_slots, static_cast<cudaStream_t>(stream));
  if (!x || !gate_w || !workspace || !correction_bias) return fail(B200MOE_EINVAL, "null input or workspace");
  if (H <= 0 || H % 8 != 0) return fail(B200MOE_EUNSUPPORTED, "H=%d must be a positive multiple of 8", H);
  if (ldx < H || (ldx * dtype_bytes(x_dtype)) % 16 != 0 || !aligned16(x) || !aligned16(gate_w))
    return fail(B200MOE_EINVAL, "x/gate_w must be 16-byte aligned with 16-byte row stride");
  const RouterWs ws = router_ws_layout(workspace, T, E, num_slots);
  if (workspace_bytes < ws.bytes)
    return fail(B200MOE_EINVAL, "workspace too small: %zu < %zu", workspace_bytes, ws.bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RouterLogitsParams lp;
  lp.x = x;
  lp.ldx = ldx;
  lp.w = gate_w;
  lp.bias = nullptr;
  lp.T = T;
  lp.H = H;
  lp.E1 = E;
  lp.logits = logits_out ? logits_out : ws.logits;
  lp.round_bf16 = 0;  // the reference computes these logits in fp32
  const bool fuse = router_small_fused_ok(T, H, x_dtype, num_slots, 1, false);
  if (!fuse) {
    if (launch_router_logits(lp, x_dtype, st)) return fail(B200MOE_ECUDA, "router_logits: kernel setup failed");
    if ((rc = check_launch("router_logits"))) return rc;
  }
  return select_common(lp.logits, 0, T, E, K, renorm && K > 1, scale, x_dtype == B200MOE_DTYPE_BF16,
                       log2phy, rep_count, max_rep, num_slots, topk_ids, topk_w, phys_ids, nullptr,
                       slot_counts, slot_offsets, ws, status, st, 1, n_group, topk_group, correction_bias,
                       fuse ? &lp : nullptr, nullptr, x_dtype);
}

int b200moe_router_from_logits(const float* logits, int has_shared_gate, int T, int E, int K,
                               int renorm, float scale, int round_bf16, const int32_t* log2phy,
                               const int32_t* rep_count, int max_rep, int num_slots,
                               int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                               float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets,
                               void* workspace, size_t workspace_bytes, int* status,
                               void* stream) {
  int rc = check_select_args(T, E, K, num_slots, log2phy, rep_count, max_rep, topk_ids, topk_w,
                             phys_ids, slot_counts, slot_offsets, has_shared_gate, shared_gate);
  if (rc) return rc;
  if ((rc = device_ok())) return rc;
  if (T == 0) return zero_counts(slot_counts, slot_offsets, num_slots, static_cast<cudaStream_t>(stream));
  if (!logits || !workspace) return fail(B200MOE_EINVAL, "null logits or workspace");
  const int E1 = E + (has_shared_gate ? 1 : 0);
  const RouterWs ws = router_ws_layout(workspace, T, E1, num_slots);
  if (workspace_bytes < ws.bytes)
    return fail(B200MOE_EINVAL, "workspace too small: %zu < %zu", workspace_bytes, ws.bytes);
  if (T == 0) return B200MOE_OK;
  return select_common(logits, has_shared_gate, T, E, K, renorm, scale, round_bf16, log2phy,
                       rep_count, max_rep, num_slots, topk_ids, topk_w, phys_ids, shared_gate,
                       slot_counts, slot_offsets, ws, status, static_cast<cudaStream_t>(stream));
}

int b200moe_permute(const void* x, int64_t ldx, int x_dtype, int T, int H, int K, int E1,
                    const int32_t* phys_ids, int num_slots, void* send, int32_t* pos_of,
                    int64_t* send_token, int64_t* send_slot, void* workspace,
                    size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (x_dtype != B200MOE_DTYPE_BF16 && x_dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "x_dtype=%d", x_dtype);
  if (T < 0 || K < 1 || K > 8 || H <= 0) return fail(B200MOE_EINVAL, "T=%d K=%d H=%d", T, K, H);
  const int row_bytes = H * dtype_bytes(x_dtype);
  if (row_bytes % 16 != 0) return fail(B200MOE_EUNSUPPORTED, "row bytes %d not a multiple of 16", row_bytes);
  if (T == 0) return B200MOE_OK;
  if (!x || !phys_ids || !send || !pos_of || !workspace) return fail(B200MOE_EINVAL, "null pointer");
  if (!aligned16(x) || !aligned16(send) || (ldx * dtype_bytes(x_dtype)) % 16 != 0)
    return fail(B200MOE_EINVAL, "x/send must be 16-byte aligned with 16-byte row stride");
  if (tokens_per_block(T) * K > 512) return fail(B200MOE_EUNSUPPORTED, "tokens per block * K > 512");
  const RouterWs ws = router_ws_layout(workspace, T, E1, num_slots);
  if (workspace_bytes < ws.bytes)
    return fail(B200MOE_EINVAL, "workspace too small: %zu < %zu", workspace_bytes, ws.bytes);
  if (T == 0) return B200MOE_OK;
  PermuteParams p;
  p.x = x;
  p.x_stride = ldx * dtype_bytes(x_dtype);
  p.row_bytes = row_bytes;
  p.T = T;
  p.K = K;
  p.phys_ids = phys_ids;
  p.block_offsets = ws.block_counts;
  p.num_slots = num_slots;
  p.nblocks = nblocks_for(T);
  p.tb = tokens_per_block(T);
  p.send = send;
  p.pos_of = pos_of;
  p.send_token = send_token;
  p.send_slot = send_slot;
  launch_permute(p, static_cast<cudaStream_t>(stream));
  return check_launch("permute");
}

int b200moe_grouped_swiglu(const void* x, int64_t ldx, int64_t rows_cap,
                           const int32_t* expert_offsets, int P, int H, int I,
                           const void* w_gate_up, void* act, int64_t ld_act, int* status,
                           void* stream) {
  return b200moe_grouped_swiglu_ex(x, ldx, rows_cap, 0, expert_offsets, P, H, I, w_gate_up, act, ld_act,
                                   status, stream);
}

int b200moe_grouped_swiglu_ex(const void* x, int64_t ldx, int64_t rows_cap, int64_t rows_hint,
                              const int32_t* expert_offsets, int P, int H, int I,
                              const void* w_gate_up, void* act, int64_t ld_act, int* status,
                              void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (P < 1 || H <= 0 || I <= 0 || rows_cap < 0) return fail(B200MOE_EINVAL, "P=%d H=%d I=%d", P, H, I);
  if (rows_cap == 0) return B200MOE_OK;  // a rank may receive no rows at all
  if (!x || !expert_offsets || !w_gate_up || !act) return fail(B200MOE_EINVAL, "null pointer");
  if (H % 64 != 0 || I % 32 != 0)
    return fail(B200MOE_EUNSUPPORTED, "grouped_swiglu needs H %% 64 == 0 and I %% 32 == 0 (H=%d I=%d)", H, I);
  if (ldx < H || ldx % 8 != 0 || ld_act < I || ld_act % 8 != 0 || !aligned16(x) || !aligned16(act) ||
      !aligned16(w_gate_up))
    return fail(B200MOE_EINVAL, "bad leading dimension or alignment");
  GemmLaunch L;
  L.a = x;
  L.rows_cap = rows_cap;
  L.lda = ldx;
  L.w = w_gate_up;
  L.p.expert_offsets = expert_offsets;
  L.p.P = P;
  L.p.N = I;
  L.p.K = H;
  L.p.w_rows = 2 * I;
  L.p.up_row = I;
  L.p.out = act;
  L.p.ldo = ld_act;
  L.p.out_row_map = nullptr;
  L.p.status = status;
  L.variant = gemm_variant_from_env();
  L.rows_hint = rows_hint < 0 ? 0 : rows_hint;
  rc = launch_grouped_swiglu(L, static_cast<cudaStream_t>(stream));
  if (rc == -4) return fail(B200MOE_EUNSUPPORTED, "P=%d exceeds the kernel's slot limit", P);
  if (rc == -1) return fail(B200MOE_ECUDA, "cuTensorMapEncodeTiled failed (gate_up)");
  if (rc) return fail(B200MOE_ECUDA, "grouped_swiglu launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("grouped_swiglu");
}

int b200moe_grouped_down(const void* act, int64_t ld_act, int64_t rows_cap,
                         const int32_t* expert_offsets, int P, int H, int I,
                         const void* w_down, void* out, int64_t ldo,
                         const int32_t* out_row_map, int* status, void* stream) {
  return b200moe_grouped_down_ex(act, ld_act, rows_cap, 0, expert_offsets, P, H, I, w_down, out, ldo,
                                 out_row_map, status, stream);
}

int b200moe_grouped_down_ex(const void* act, int64_t ld_act, int64_t rows_cap, int64_t rows_hint,
                            const int32_t* expert_offsets, int P, int H, int I,
                            const void* w_down, void* out, int64_t ldo,
                            const int32_t* out_row_map, int* status, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (P < 1 || H <= 0 || I <= 0 || rows_cap < 0) return fail(B200MOE_EINVAL, "P=%d H=%d I=%d", P, H, I);
  if (rows_cap == 0) return B200MOE_OK;
  if (!act || !expert_offsets || !w_down || !out) return fail(B200MOE_EINVAL, "null pointer");
  if (H % 32 != 0 || I % 64 != 0)
    return fail(B200MOE_EUNSUPPORTED, "grouped_down needs H %% 32 == 0 and I %% 64 == 0 (H=%d I=%d)", H, I);
  if (ld_act < I || ld_act % 8 != 0 || ldo < H || ldo % 8 != 0 || !aligned16(act) || !aligned16(out) ||
      !aligned16(w_down))
    return fail(B200MOE_EINVAL, "bad leading dimension or alignment");
  GemmLaunch L;
  L.a = act;
  L.rows_cap = rows_cap;
  L.lda = ld_act;
  L.w = w_down;
  L.p.expert_offsets = expert_offsets;
  L.p.P = P;
  L.p.N = H;
  L.p.K = I;
  L.p.w_rows = H;
  L.p.up_row = 0;
  L.p.out = out;
  L.p.ldo = ldo;
  L.p.out_row_map = out_row_map;
  L.p.status = status;
  L.variant = gemm_variant_from_env();
  L.rows_hint = rows_hint < 0 ? 0 : rows_hint;
  rc = launch_grouped_down(L, static_cast<cudaStream_t>(stream));
  if (rc == -4) return fail(B200MOE_EUNSUPPORTED, "P=%d exceeds the kernel's slot limit", P);
  if (rc == -1) return fail(B200MOE_ECUDA, "cuTensorMapEncodeTiled failed (down)");
  if (rc) return fail(B200MOE_ECUDA, "grouped_down launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("grouped_down");
}

int b200moe_grouped_swiglu_f32(const float* x, int64_t ldx, int64_t rows_cap,
                               const int32_t* expert_offsets, int P, int H, int I,
                               const float* w_gate_up, float* act, int64_t ld_act, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (P < 1 || H <= 0 || I <= 0 || rows_cap < 0) return fail(B200MOE_EINVAL, "P=%d H=%d I=%d", P, H, I);
  if (rows_cap == 0) return B200MOE_OK;
  if (!x || !expert_offsets || !w_gate_up || !act) return fail(B200MOE_EINVAL, "null pointer");
  if (ldx < H || ld_act < I) return fail(B200MOE_EINVAL, "bad leading dimension");
  GemmF32Params p{x, ldx, rows_cap, w_gate_up, expert_offsets, P, I, H, 2 * I, I, act, ld_act, nullptr};
  launch_grouped_gemm_f32(p, true, static_cast<cudaStream_t>(stream));
  return check_launch("grouped_swiglu_f32");
}

int b200moe_grouped_down_f32(const float* act, int64_t ld_act, int64_t rows_cap,
                             const int32_t* expert_offsets, int P, int H, int I, const float* w_down,
                             float* out, int64_t ldo, const int32_t* out_row_map, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (P < 1 || H <= 0 || I <= 0 || rows_cap < 0) return fail(B200MOE_EINVAL, "P=%d H=%d I=%d", P, H, I);
  if (rows_cap == 0) return B200MOE_OK;
  if (!act || !expert_offsets || !w_down || !out) return fail(B200MOE_EINVAL, "null pointer");
  if (ld_act < I || ldo < H) return fail(B200MOE_EINVAL, "bad leading dimension");
  GemmF32Params p{act, ld_act, rows_cap, w_down, expert_offsets, P, H, I, H, 0, out, ldo, out_row_map};
  launch_grouped_gemm_f32(p, false, static_cast<cudaStream_t>(stream));
  return check_launch("grouped_down_f32");
}

int b200moe_combine(const void* y, int64_t ldy, int dtype, const int32_t* pos_of,
                    const float* topk_w, int T, int K, int H, const void* shared, int64_t lds,
                    const float* shared_gate, void* out, int64_t ldo, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (dtype != B200MOE_DTYPE_BF16 && dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "dtype=%d", dtype);
  if (T < 0 || K < 1 || K > 8 || H <= 0 || H % 8 != 0) return fail(B200MOE_EINVAL, "T=%d K=%d H=%d", T, K, H);
  if (T == 0) return B200MOE_OK;
  if (!y || !pos_of || !topk_w || !out) return fail(B200MOE_EINVAL, "null pointer");
  const int eb = dtype_bytes(dtype);
  if (!aligned16(y) || !aligned16(out) || (ldy * eb) % 16 || (ldo * eb) % 16 ||
      (shared && (!aligned16(shared) || (lds * eb) % 16)))
    return fail(B200MOE_EINVAL, "y/out/shared must be 16-byte aligned with 16-byte row strides");
  CombineParams p;
  p.y = y;
  p.ldy = ldy;
  p.dtype = dtype;
  p.pos_of = pos_of;
  p.topk_w = topk_w;
  p.T = T;
  p.K = K;
  p.H = H;
  p.shared = shared;
  p.lds = lds;
  p.shared_gate = shared_gate;
  p.out = out;
  p.ldo = ldo;
  launch_combine(p, static_cast<cudaStream_t>(stream));
  return check_launch("combine");
}

int b200moe_add_rmsnorm(const void* residual, const void* hidden, const void* weight, float eps,
                        int T, int H, int dtype, int64_t ld, void* residual_out, void* normed,
                        int64_t ld_normed, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (dtype != B200MOE_DTYPE_BF16 && dtype != B200MOE_DTYPE_F32) return fail(B200MOE_EUNSUPPORTED, "dtype=%d", dtype);
  if (T < 0 || H <= 0) return fail(B200MOE_EINVAL, "T=%d H=%d", T, H);
  if (T == 0) return B200MOE_OK;
  const int eb = dtype_bytes(dtype);
  if (!residual || !residual_out || (normed && !weight)) return fail(B200MOE_EINVAL, "null pointer");
  if ((H * eb) % 16 || (ld * eb) % 16 || ld < H || !aligned16(residual) || !aligned16(residual_out) ||
      (hidden && !aligned16(hidden)) || (normed && (!aligned16(normed) || !aligned16(weight) ||
                                                    (ld_normed * eb) % 16 || ld_normed < H)))
    return fail(B200MOE_EINVAL, "rows must be 16-byte aligned multiples of 16 bytes");
  AddNormParams p;
  p.residual = residual;
  p.hidden = hidden;
  p.weight = weight;
  p.eps = eps;
  p.T = T;
  p.H = H;
  p.dtype = dtype;
  p.ld = ld;
  p.residual_out = residual_out;
  p.normed = normed;
  p.ld_normed = ld_normed;
  if (launch_add_rmsnorm(p, static_cast<cudaStream_t>(stream)) != 0)
    return fail(B200MOE_EUNSUPPORTED, "add_rmsnorm supports rows up to 32 KB (H=%d)", H);
  return check_launch("add_rmsnorm");
}

int b200moe_gather_segments(const void* src, void* dst, int64_t row_bytes,
                            const int32_t* src_start, const int32_t* dst_start,
                            const int32_t* len, int nseg, int64_t max_rows,
                            int32_t* dst_to_src, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (nseg < 0 || nseg > 65535 || max_rows < 0) return fail(B200MOE_EINVAL, "nseg=%d max_rows=%lld", nseg, static_cast<long long>(max_rows));
  if (nseg == 0 || max_rows == 0) return B200MOE_OK;
  if (!src || !dst || !src_start || !dst_start || !len) return fail(B200MOE_EINVAL, "null pointer");
  if (row_bytes <= 0 || row_bytes % 16 != 0 || !aligned16(src) || !aligned16(dst))
    return fail(B200MOE_EINVAL, "row_bytes=%lld must be a positive multiple of 16 with aligned buffers",
                static_cast<long long>(row_bytes));
  const int rows_per_cta = 16;
  dim3 grid(static_cast<unsigned>((max_rows + rows_per_cta - 1) / rows_per_cta), static_cast<unsigned>(nseg));
  launch_kernel(gather_segments_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream),
                static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), row_bytes, src_start, dst_start,
                len, rows_per_cta, dst_to_src);
  return check_launch("gather_segments");
}

// ------------------------------------------------------------------ peer exchange
// counters[0..2]: tickets of dispatch (or permute-dispatch) / collect / combine_send;
// counters[3]: dispatch arrivals consumed; counters[4]: combine arrivals consumed;
// counters[5]: ticket of the combine that waits itself; counters[6]: ticket of the down
// GEMM that sends its rows; counters[7]: metadata arrivals consumed; counters[8]: ticket
// of the GEMM that reads the receive region directly.
static_assert(sizeof(cudaIpcMemHandle_t) == B200MOE_EP_HANDLE_BYTES, "IPC handle size");

}  // extern "C"

namespace {

int ep_params(const b200moe_ep_desc* ep, EpParams* p) {
  if (ep == nullptr) return fail(B200MOE_EINVAL, "null exchange descriptor");
  const int G = ep->world_size;
  if (G < 1 || G > B200MOE_EP_MAX_RANKS || ep->rank < 0 || ep->rank >= G)
    return fail(B200MOE_EINVAL, "world_size=%d rank=%d (at most %d ranks)", G, ep->rank, B200MOE_EP_MAX_RANKS);
  const int P = ep->slots_per_rank;
  if (P < 1 || ep->row_bytes <= 0 || ep->row_bytes % 16 != 0 || ep->cap_rows < 0 || ep->comb_rows < 0)
    return fail(B200MOE_EINVAL, "P=%d row_bytes=%d cap_rows=%lld comb_rows=%lld", P, ep->row_bytes,
                static_cast<long long>(ep->cap_rows), static_cast<long long>(ep->comb_rows));
  if (static_cast<int64_t>(G) * ep->cap_rows > INT32_MAX || ep->comb_rows > INT32_MAX)
    return fail(B200MOE_EUNSUPPORTED, "exchange regions above 2^31 rows");
  if (sizeof(int32_t) * (2 * G * P + G + 1 + P + 1) > 48 * 1024)
    return fail(B200MOE_EUNSUPPORTED, "G*P=%d too large for the collect kernel's tables", G * P);
  if (ep->counters == nullptr) return fail(B200MOE_EINVAL, "null counters");
  for (int g = 0; g < G; ++g) {
    if (ep->peer[g] == nullptr || !aligned16(ep->peer[g])) return fail(B200MOE_EINVAL, "peer buffer %d", g);
    p->peer[g] = static_cast<uint8_t*>(ep->peer[g]);
  }
  for (int g = G; g < EP_MAX_RANKS; ++g) p->peer[g] = nullptr;
  p->G = G;
  p->P = P;
  p->rank = ep->rank;
  p->row_bytes = ep->row_bytes;
  p->cap_rows = ep->cap_rows;
  p->comb_rows = ep->comb_rows;
  p->ticket = ep->counters;
  p->status = ep->status;
  return B200MOE_OK;
}

}  // namespace

extern "C" {

int b200moe_ep_layout(int world_size, int slots_per_rank, int64_t cap_rows, int64_t comb_rows, int row_bytes,
                      int64_t* recv_offset, int64_t* comb_offset, int64_t* total_bytes) {
  if (world_size < 1 || world_size > B200MOE_EP_MAX_RANKS || slots_per_rank < 1 || cap_rows < 0 ||
      comb_rows < 0 || row_bytes <= 0 || row_bytes % 16 != 0)
    return fail(B200MOE_EINVAL, "world_size=%d P=%d row_bytes=%d", world_size, slots_per_rank, row_bytes);
  if (recv_offset) *recv_offset = ep_recv_offset(world_size, slots_per_rank);
  if (comb_offset) *comb_offset = ep_comb_offset(world_size, slots_per_rank, cap_rows, row_bytes);
  if (total_bytes) *total_bytes = ep_buffer_bytes(world_size, slots_per_rank, cap_rows, comb_rows, row_bytes);
  return B200MOE_OK;
}

int b200moe_ep_alloc(size_t bytes, void** buffer, void* handle) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (bytes == 0 || buffer == nullptr || handle == nullptr) return fail(B200MOE_EINVAL, "ep_alloc arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(B200MOE_ECUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(B200MOE_ECUDA, "exchange buffer setup: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *buffer = p;
  return B200MOE_OK;
}

int b200moe_ep_open(const void* handle, void** peer_buffer) {
  int rc;
  if ((rc = device_ok())) return rc;
  if (handle == nullptr || peer_buffer == nullptr) return fail(B200MOE_EINVAL, "ep_open arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(B200MOE_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return B200MOE_OK;
}

int b200moe_ep_close(void* peer_buffer) {
  if (peer_buffer == nullptr) return B200MOE_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buffer);
  if (e != cudaSuccess) return fail(B200MOE_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return B200MOE_OK;
}

int b200moe_ep_free(void* buffer) {
  if (buffer == nullptr) return B200MOE_OK;
  const cudaError_t e = cudaFree(buffer);
  if (e != cudaSuccess) return fail(B200MOE_ECUDA, "cudaFree: %s", cudaGetErrorString(e));
  return B200MOE_OK;
}

int b200moe_ep_dispatch(const b200moe_ep_desc* ep, const void* send, const int32_t* slot_offsets,
                        int64_t send_rows, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams p;
  if ((rc = ep_params(ep, &p))) return rc;
  if (slot_offsets == nullptr || send_rows < 0 || (send_rows > 0 && (send == nullptr || !aligned16(send))))
    return fail(B200MOE_EINVAL, "dispatch: send/slot_offsets");
  if (send_rows > ep->comb_rows)
    return fail(B200MOE_EINVAL, "send_rows=%lld exceeds comb_rows=%lld", static_cast<long long>(send_rows),
                static_cast<long long>(ep->comb_rows));
  p.ticket = ep->counters + 0;
  if (launch_ep_dispatch(p, send, slot_offsets, send_rows, static_cast<cudaStream_t>(stream)))
    return fail(B200MOE_ECUDA, "ep_dispatch launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_dispatch");
}

int b200moe_ep_collect(const b200moe_ep_desc* ep, void* x_expert, int32_t* row_map, int32_t* peer_row_map,
                       int32_t* expert_offsets, int64_t rows_hint, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams p;
  if ((rc = ep_params(ep, &p))) return rc;
  if (x_expert == nullptr || !aligned16(x_expert) || (row_map == nullptr && peer_row_map == nullptr) ||
      expert_offsets == nullptr)
    return fail(B200MOE_EINVAL, "collect: null or misaligned output");
  if (peer_row_map != nullptr && ep->comb_rows > (int64_t(1) << kPeerRowBits))
    return fail(B200MOE_EUNSUPPORTED, "peer row map holds at most 2^%d rows per rank", kPeerRowBits);
  p.ticket = ep->counters + 1;
  const int64_t rows = rows_hint > 0 ? rows_hint : static_cast<int64_t>(p.G) * p.cap_rows;
  if (launch_ep_collect(p, x_expert, row_map, peer_row_map, expert_offsets, ep->counters + 3, ep->counters + 7,
                        ep->timeout_ns, rows, static_cast<cudaStream_t>(stream)))
    return fail(B200MOE_ECUDA, "ep_collect launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_collect");
}

int b200moe_ep_combine_send(const b200moe_ep_desc* ep, const void* y_recv, int64_t rows_hint, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams p;
  if ((rc = ep_params(ep, &p))) return rc;
  if (y_recv == nullptr || !aligned16(y_recv)) return fail(B200MOE_EINVAL, "combine_send: y_recv");
  p.ticket = ep->counters + 2;
  const int64_t rows = rows_hint > 0 ? rows_hint : static_cast<int64_t>(p.G) * p.cap_rows;
  if (launch_ep_combine_send(p, y_recv, rows, static_cast<cudaStream_t>(stream)))
    return fail(B200MOE_ECUDA, "ep_combine_send launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_combine_send");
}

int b200moe_ep_permute_dispatch(const b200moe_ep_desc* ep, const void* x, int64_t ldx, int x_dtype, int T, int H,
                                int K, int E1, const int32_t* phys_ids, const int32_t* slot_offsets,
                                int32_t* pos_of, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams e;
  if ((rc = ep_params(ep, &e))) return rc;
  if (x_dtype != B200MOE_DTYPE_BF16 && x_dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "x_dtype=%d", x_dtype);
  if (T < 0 || K < 1 || K > 8 || H <= 0) return fail(B200MOE_EINVAL, "T=%d K=%d H=%d", T, K, H);
  const int row_bytes = H * dtype_bytes(x_dtype);
  if (row_bytes != ep->row_bytes) return fail(B200MOE_EINVAL, "row bytes %d != exchange row bytes %d", row_bytes,
                                              ep->row_bytes);
  if (static_cast<int64_t>(T) * K > ep->comb_rows)
    return fail(B200MOE_EINVAL, "T*K=%lld exceeds comb_rows=%lld", static_cast<long long>(T) * K,
                static_cast<long long>(ep->comb_rows));
  if (!slot_offsets || !workspace || (T > 0 && (!x || !phys_ids || !pos_of)))
    return fail(B200MOE_EINVAL, "null pointer");
  if (T > 0 && (!aligned16(x) || (ldx * dtype_bytes(x_dtype)) % 16 != 0))
    return fail(B200MOE_EINVAL, "x must be 16-byte aligned with a 16-byte row stride");
  if (tokens_per_block(T) * K > 512) return fail(B200MOE_EUNSUPPORTED, "tokens per block * K > 512");
  const int num_slots = ep->world_size * ep->slots_per_rank;
  const RouterWs ws = router_ws_layout(workspace, T, E1, num_slots);
  if (workspace_bytes < ws.bytes)
    return fail(B200MOE_EINVAL, "workspace too small: %zu < %zu", workspace_bytes, ws.bytes);
  PermuteParams p;
  p.x = x;
  p.x_stride = ldx * dtype_bytes(x_dtype);
  p.row_bytes = row_bytes;
  p.T = T;
  p.K = K;
  p.phys_ids = phys_ids;
  p.block_offsets = ws.block_counts;
  p.num_slots = num_slots;
  p.nblocks = nblocks_for(T);
  p.tb = tokens_per_block(T);
  p.send = nullptr;
  p.pos_of = pos_of;
  p.send_token = nullptr;
  p.send_slot = nullptr;
  p.peer_mode = 1;
  p.slot_offsets = slot_offsets;
  p.ep = e;
  p.ep.ticket = ep->counters + 0;
  if (launch_permute(p, static_cast<cudaStream_t>(stream)))
    return fail(B200MOE_ECUDA, "ep_permute_dispatch launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_permute_dispatch");
}

int b200moe_ep_grouped_down_send(const b200moe_ep_desc* ep, const void* act, int64_t ld_act, int64_t rows_cap,
                                 int64_t rows_hint, const int32_t* expert_offsets, int P, int H, int I,
                                 const void* w_down, const int32_t* peer_row_map, int* status, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams e;
  if ((rc = ep_params(ep, &e))) return rc;
  if (P != ep->slots_per_rank || H <= 0 || I <= 0 || rows_cap <= 0)
    return fail(B200MOE_EINVAL, "P=%d H=%d I=%d rows_cap=%lld", P, H, I, static_cast<long long>(rows_cap));
  if (H * 2 != ep->row_bytes) return fail(B200MOE_EINVAL, "bf16 rows of H=%d do not match the exchange", H);
  if (!act || !expert_offsets || !w_down || !peer_row_map) return fail(B200MOE_EINVAL, "null pointer");
  if (H % 32 != 0 || I % 64 != 0)
    return fail(B200MOE_EUNSUPPORTED, "grouped_down needs H %% 32 == 0 and I %% 64 == 0 (H=%d I=%d)", H, I);
  if (ld_act < I || ld_act % 8 != 0 || !aligned16(act) || !aligned16(w_down))
    return fail(B200MOE_EINVAL, "bad leading dimension or alignment");
  GemmLaunch L;
  L.a = act;
  L.rows_cap = rows_cap;
  L.lda = ld_act;
  L.w = w_down;
  L.p.expert_offsets = expert_offsets;
  L.p.P = P;
  L.p.N = H;
  L.p.K = I;
  L.p.w_rows = H;
  L.p.up_row = 0;
  L.p.out = nullptr;
  L.p.ldo = H;
  L.p.out_row_map = peer_row_map;
  L.p.status = status;
  L.p.peer_out = 1;
  for (int g = 0; g < EP_MAX_RANKS; ++g) {
    L.p.po.base[g] = g < e.G ? e.peer[g] : nullptr;
    L.p.po.rows[g] = g < e.G ? e.peer[g] + ep_comb_offset(e.G, e.P, e.cap_rows, e.row_bytes) : nullptr;
  }
  L.p.po.G = e.G;
  L.p.po.rank = e.rank;
  L.p.po.ticket = ep->counters + 6;
  L.variant = gemm_variant_from_env();
  L.rows_hint = rows_hint < 0 ? 0 : rows_hint;
  rc = launch_grouped_down(L, static_cast<cudaStream_t>(stream));
  if (rc == -4) return fail(B200MOE_EUNSUPPORTED, "P=%d exceeds the kernel's slot limit", P);
  if (rc == -1) return fail(B200MOE_ECUDA, "cuTensorMapEncodeTiled failed (down)");
  if (rc) return fail(B200MOE_ECUDA, "ep_grouped_down_send launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_grouped_down_send");
}

int b200moe_ep_combine(const b200moe_ep_desc* ep, const int32_t* pos_of, const float* topk_w, int T, int K,
                       int H, int dtype, const void* shared, int64_t lds, const float* shared_gate, void* out,
                       int64_t ldo, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams e;
  if ((rc = ep_params(ep, &e))) return rc;
  if (dtype != B200MOE_DTYPE_BF16 && dtype != B200MOE_DTYPE_F32)
    return fail(B200MOE_EUNSUPPORTED, "dtype=%d", dtype);
  if (T < 0 || K < 1 || K > 8 || H <= 0 || H % 8 != 0) return fail(B200MOE_EINVAL, "T=%d K=%d H=%d", T, K, H);
  const int eb = dtype_bytes(dtype);
  if (H * eb != ep->row_bytes) return fail(B200MOE_EINVAL, "rows of H=%d do not match the exchange", H);
  if (T > 0 && (!pos_of || !topk_w || !out)) return fail(B200MOE_EINVAL, "null pointer");
  if ((T > 0 && !aligned16(out)) || (ldo * eb) % 16 || (shared && (!aligned16(shared) || (lds * eb) % 16)))
    return fail(B200MOE_EINVAL, "out/shared must be 16-byte aligned with 16-byte row strides");
  CombineParams p;
  p.y = e.peer[e.rank] + ep_comb_offset(e.G, e.P, e.cap_rows, e.row_bytes);
  p.ldy = H;
  p.dtype = dtype;
  p.pos_of = pos_of;
  p.topk_w = topk_w;
  p.T = T;
  p.K = K;
  p.H = H;
  p.shared = shared;
  p.lds = lds;
  p.shared_gate = shared_gate;
  p.out = out;
  p.ldo = ldo;
  p.wait_flags = reinterpret_cast<const uint32_t*>(e.peer[e.rank]) + e.G;
  p.wait_n = e.G;
  p.wait_expect = ep->counters + 4;
  p.wait_ticket = ep->counters + 5;
  p.wait_timeout_ns = ep->timeout_ns;
  p.status = ep->status;
  if (launch_combine(p, static_cast<cudaStream_t>(stream)))
    return fail(B200MOE_ECUDA, "ep_combine launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_combine");
}

// The two prefill GEMMs reading this rank's receive region directly (no collect).
static int recv_gemm_launch(const b200moe_ep_desc* ep, const EpParams& e, const void* a, int64_t lda,
                            const void* w, int P, int N, int K, int w_rows, int up_row, void* out, int64_t ldo,
                            bool swiglu, int consume, int* status, cudaStream_t st) {
  GemmLaunch L;
  L.a = a;
  L.rows_cap = static_cast<int64_t>(e.G) * e.cap_rows;
  L.lda = lda;
  L.w = w;
  L.p.expert_offsets = nullptr;
  L.p.P = P;
  L.p.N = N;
  L.p.K = K;
  L.p.w_rows = w_rows;
  L.p.up_row = up_row;
  L.p.out = out;
  L.p.ldo = ldo;
  L.p.out_row_map = nullptr;
  L.p.status = status;
  L.p.seg_mode = 1;
  uint8_t* mine = e.peer[e.rank];
  L.p.seg.meta = reinterpret_cast<const int32_t*>(mine + 256);
  L.p.seg.rows_flag = reinterpret_cast<const uint32_t*>(mine);
  L.p.seg.meta_flag = reinterpret_cast<const uint32_t*>(mine) + 2 * e.G;
  L.p.seg.rows_expect = ep->counters + 3;
  L.p.seg.meta_expect = ep->counters + 7;
  L.p.seg.ticket = ep->counters + 8;
  L.p.seg.G = e.G;
  L.p.seg.rank = e.rank;
  L.p.seg.cap_rows = e.cap_rows;
  L.p.seg.comb_rows = e.comb_rows;
  L.p.seg.timeout_ns = ep->timeout_ns;
  L.p.seg.consume = consume;
  if (!swiglu) {
    L.p.peer_out = 1;
    for (int g = 0; g < EP_MAX_RANKS; ++g) {
      L.p.po.base[g] = g < e.G ? e.peer[g] : nullptr;
      L.p.po.rows[g] = g < e.G ? e.peer[g] + ep_comb_offset(e.G, e.P, e.cap_rows, e.row_bytes) : nullptr;
    }
    L.p.po.G = e.G;
    L.p.po.rank = e.rank;
    L.p.po.ticket = ep->counters + 6;
  }
  if (!pair_gemm_supported(L, swiglu))
    return fail(B200MOE_EUNSUPPORTED, "receive-region GEMMs need I %% 128 == 0, H %% 256 == 0, G*P <= 512");
  if (launch_grouped_pair(L, swiglu, st))
    return fail(B200MOE_ECUDA, "receive-region GEMM launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch(swiglu ? "ep_grouped_swiglu_recv" : "ep_grouped_down_send_recv");
}

int b200moe_ep_grouped_swiglu_recv(const b200moe_ep_desc* ep, const void* w_gate_up, int P, int H, int I, void* act,
                                   int64_t ld_act, int* status, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams e;
  if ((rc = ep_params(ep, &e))) return rc;
  if (P != ep->slots_per_rank || H * 2 != ep->row_bytes || I <= 0 || !w_gate_up || !act || ld_act < I ||
      ld_act % 8 != 0 || !aligned16(act) || !aligned16(w_gate_up))
    return fail(B200MOE_EINVAL, "ep_grouped_swiglu_recv: P=%d H=%d I=%d (bf16 rows of the exchange)", P, H, I);
  return recv_gemm_launch(ep, e, e.peer[e.rank] + ep_recv_offset(e.G, e.P), H, w_gate_up, P, I, H, 2 * I, I, act,
                          ld_act, true, 1, status, static_cast<cudaStream_t>(stream));
}

int b200moe_ep_grouped_down_send_recv(const b200moe_ep_desc* ep, const void* act, int64_t ld_act, const void* w_down,
                                      int P, int H, int I, int* status, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams e;
  if ((rc = ep_params(ep, &e))) return rc;
  if (P != ep->slots_per_rank || H * 2 != ep->row_bytes || I <= 0 || !w_down || !act || ld_act < I ||
      ld_act % 8 != 0 || !aligned16(act) || !aligned16(w_down))
    return fail(B200MOE_EINVAL, "ep_grouped_down_send_recv: P=%d H=%d I=%d (bf16 rows of the exchange)", P, H, I);
  if (ep->comb_rows > (int64_t(1) << kPeerRowBits))
    return fail(B200MOE_EUNSUPPORTED, "peer rows hold at most 2^%d rows per rank", kPeerRowBits);
  return recv_gemm_launch(ep, e, act, ld_act, w_down, P, H, I, H, 0, nullptr, H, false, 0, status,
                          static_cast<cudaStream_t>(stream));
}

int b200moe_ep_wait_combine(const b200moe_ep_desc* ep, void* stream) {
  int rc;
  if ((rc = device_ok())) return rc;
  EpParams p;
  if ((rc = ep_params(ep, &p))) return rc;
  if (launch_ep_wait_comb(p, ep->counters + 4, ep->timeout_ns, static_cast<cudaStream_t>(stream)))
    return fail(B200MOE_ECUDA, "ep_wait_combine launch: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch("ep_wait_combine");
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free router
// Scratch of b200moe_router_noalloc: one file-scope device array.  Every GPU on which
// this library is loaded holds these bytes until the process exits.  Calls share it
// and it keeps the last call's contents, so calls that overlap on the GPU race.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
}  // namespace

static __device__ __align__(256) uint8_t g_router_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};
CUcontext g_scratch_ctx[64] = {nullptr};

// The calling thread's current CUDA context (driver entry point, no libcuda link).
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static const Fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<Fn>(p);
    return static_cast<Fn>(nullptr);
  }();
  CUcontext c = nullptr;
  if (fn != nullptr && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

// Device address of g_router_scratch on the current device.  Looked up with that
// device current, on the first call there, and again whenever the thread's current
// context is no longer the one the address was taken in (a context created anew,
// e.g. after cudaDeviceReset, loads the module again and may place the array
// elsewhere).  In host code the symbol itself is only a host-side stand-in, never a
// device address.
int router_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(B200MOE_ENODEVICE, "no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr || current_context() != g_scratch_ctx[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(B200MOE_ECUDA, "cudaGetSymbolAddress(router scratch) on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = current_context();  // the lookup made the primary context current
  }
  *out = g_scratch_ptr[dev];
  return B200MOE_OK;
}

}  // namespace

extern "C" int b200moe_router_noalloc(const void* x, int64_t ldx, int x_dtype, const void* gate_w,
                                      const float* gate_bias, int has_shared_gate, int T, int H, int E,
                                      int K, int renorm, float scale, const int32_t* log2phy,
                                      const int32_t* rep_count, int max_rep, int num_slots,
                                      int32_t* topk_ids, float* topk_w, int32_t* phys_ids,
                                      float* shared_gate, int32_t* slot_counts, int32_t* slot_offsets,
                                      float* logits_out, int* status, void* stream) {
  if (T < 0 || E < 1 || num_slots < 1) return fail(B200MOE_EINVAL, "T=%d E=%d num_slots=%d", T, E, num_slots);
  const int E1 = E + (has_shared_gate ? 1 : 0);
  const size_t need = router_ws_layout(nullptr, T, E1, num_slots).bytes;
  if (need > kNoAllocScratchBytes)
    return fail(B200MOE_EUNSUPPORTED,
                "b200moe_router_noalloc: T=%d, %d router columns and %d slots need %zu bytes of scratch; "
                "the built-in scratch holds %zu bytes (use b200moe_router with a caller workspace)",
                T, E1, num_slots, need, kNoAllocScratchBytes);
  int rc = device_ok();  // a clear error on a device without an sm_100a image, before any lookup
  if (rc) return rc;
  void* ws = nullptr;
  if ((rc = router_scratch_address(&ws))) return rc;
  // The completion counter must read zero when the kernels start; a call that was cut
  // short could have left it set, so clear it on the caller's stream every time.
  const cudaError_t e = cudaMemsetAsync(ws, 0, kCounterBytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(B200MOE_ECUDA, "clearing the router scratch counter: %s", cudaGetErrorString(e));
  return b200moe_router(x, ldx, x_dtype, gate_w, gate_bias, has_shared_gate, T, H, E, K, renorm, scale,
                        log2phy, rep_count, max_rep, num_slots, topk_ids, topk_w, phys_ids, shared_gate,
                        slot_counts, slot_offsets, logits_out, ws, kNoAllocScratchBytes, status, stream);
}
