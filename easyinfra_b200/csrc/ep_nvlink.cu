// Expert-parallel token exchange over NVLink peer memory, without host round trips.
//
// The reference moves tokens with two NCCL all_to_all_single calls whose split sizes
// come from a device->host copy of the all-gathered counts
// (easyinfra/generation/blocks/moe/moe_all2all.py:397-444 dispatch, :560-591 combine).
// Here every rank owns one peer-mapped buffer (layout in kernels.cuh, EpParams) and the
// exchange is four kernels that store into peers and wait only on their own flags:
//   ep_dispatch      sender r: the rows for destination d -> d.recv[r]; r's row count
//                    per slot of d and r's first send row for d -> d.meta[r]; the last
//                    CTA fences at system scope and adds 1 to d.disp[r] for every d;
//   ep_collect       receiver: bounded wait until every disp flag passed the expected
//                    count, then expert offsets, expert-major regroup of the received
//                    rows and the row map that sends the down GEMM's rows back to
//                    arrival order;
//   ep_combine_send  receiver: expert outputs of source s -> s.comb at s's own send
//                    positions; the last CTA adds 1 to s.comb[r];
//   ep_wait_comb     sender: bounded wait until every comb flag passed its count; the
//                    combine kernel that follows reads s.comb in send order.
// Flags only grow; each rank keeps device-side counts of the arrivals it consumed, so
// the same launches replay unchanged inside a CUDA graph.  A wait that passes its limit
// records B200MOE_STATUS_TIMEOUT and the kernel carries on with what it has.
//
// Buffer reuse is safe without further waits: a source writes d.recv[s] and d.meta[s]
// for the next layer only after its own ep_wait_comb saw d's ep_combine_send, which
// runs after d's ep_collect finished reading both; a destination writes s.comb for the
// next layer only after s's next ep_dispatch, which follows s's combine.
//
// Peers are reached with plain 16-byte stores, acquire loads and system-scope atomics;
// no TMA or cluster-shared load ever reads peer memory.
#include "kernels.cuh"

namespace b200moe {

// ------------------------------------------------------------------ dispatch
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __grid_constant__ EpParams p, const uint8_t* send,
                                                          const int32_t* slot_offsets) {
  __shared__ int s_off[EP_MAX_RANKS + 1];  // first send row per destination
  __shared__ int s_n[EP_MAX_RANKS];        // rows sent per destination (clamped to cap_rows)
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int G = p.G, P = p.P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x <= G) s_off[threadIdx.x] = slot_offsets[threadIdx.x * P];  // first send row per rank
  __syncthreads();
  if (threadIdx.x < G) {
    const int n = s_off[threadIdx.x + 1] - s_off[threadIdx.x];
    if (n > p.cap_rows) record_status(p.status, kStatusCapacity);
    s_n[threadIdx.x] = static_cast<int>(min64(n, p.cap_rows));
    if (blockIdx.x == 0) ep_publish_meta(p, slot_offsets, threadIdx.x);
  }
  __syncthreads();
  const int total = s_off[G];
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int i = blockIdx.x * (blockDim.x >> 5) + warp; i < total; i += nwarps) {
    int d = 0;
    while (d + 1 < G && i >= s_off[d + 1]) ++d;
    const int j = i - s_off[d];
    if (j >= s_n[d]) continue;
    copy_row<false>(ep_recv_rows(p.peer[d], p) + (static_cast<int64_t>(p.rank) * p.cap_rows + j) * p.row_bytes,
                    send + static_cast<int64_t>(i) * p.row_bytes, p.row_bytes, lane);
  }
  if (last_cta(p.ticket, &s_last) && threadIdx.x < G) ep_publish_rows(p, threadIdx.x);
}

// ------------------------------------------------------------------ collect
// Dynamic shared memory: cnt[G*P], base[G*P], srow[G+1], eoff[P+1] (int32).
__global__ void __launch_bounds__(256) ep_collect_kernel(const __grid_constant__ EpParams p, uint8_t* xe, int32_t* row_map,
                                                         int32_t* peer_row_map, int32_t* expert_offsets,
                                                         uint32_t* expect, uint32_t* meta_expect,
                                                         uint64_t timeout_ns) {
  extern __shared__ int32_t sm[];
  __shared__ int s_last;
  __shared__ uint32_t s_target;
  __shared__ int s_dst[EP_MAX_RANKS];  // first combine row at each source (peer_row_map)
  pdl_trigger();
  pdl_wait();
  const int G = p.G, P = p.P;
  int32_t* cnt = sm;
  int32_t* base = cnt + G * P;
  int32_t* srow = base + G * P;
  int32_t* eoff = srow + G + 1;
  uint8_t* mine = p.peer[p.rank];
  if (threadIdx.x == 0) {
    const uint32_t target = *expect + 1u;
    bool ok = true;
    for (int s = 0; s < G && ok; ++s) ok = wait_flag_geq(ep_flags(mine) + s, target, timeout_ns, p.status);
    if (!ok) record_status(p.status, kStatusTimeout);
    s_target = target;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    // per-source counts, re-clamped so that no region is read past cap_rows
    const int s = threadIdx.x;
    const volatile int32_t* meta = ep_meta(mine, p) + s * (P + 1);
    int run = 0;
    for (int q = 0; q < P; ++q) {
      const int c = clamp_run(meta[q], run, p.cap_rows);
      cnt[s * P + q] = c;
      run += c;
    }
    int dst = meta[P];
    if (dst < 0 || static_cast<int64_t>(dst) + run > p.comb_rows) {
      if (peer_row_map != nullptr) record_status(p.status, kStatusBadIndex);
      dst = 0;  // keeps every store in bounds; the status word reports the fault
    }
    s_dst[s] = dst;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // base[s*P+q]: first expert-major row of (source s, slot q); srow[s]: first arrival row
    int run = 0;
    for (int q = 0; q < P; ++q) {
      eoff[q] = run;
      for (int s = 0; s < G; ++s) {
        base[s * P + q] = run;
        run += cnt[s * P + q];
      }
    }
    eoff[P] = run;
    int r2 = 0;
    for (int s = 0; s < G; ++s) {
      srow[s] = r2;
      for (int q = 0; q < P; ++q) r2 += cnt[s * P + q];
    }
    srow[G] = r2;
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int q = threadIdx.x; q <= P; q += blockDim.x) expert_offsets[q] = eoff[q];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int total = srow[G];
  for (int i = blockIdx.x * (blockDim.x >> 5) + warp; i < total; i += nwarps) {
    int s = 0;
    while (s + 1 < G && i >= srow[s + 1]) ++s;
    const int j = i - srow[s];  // row within source s's region (< cap_rows by the clamp)
    int q = 0, acc = 0;
    while (q + 1 < P && j >= acc + cnt[s * P + q]) acc += cnt[s * P + q++];
    const int dst = base[s * P + q] + (j - acc);
    const int64_t src = static_cast<int64_t>(s) * p.cap_rows + j;
    copy_row<true>(xe + static_cast<int64_t>(dst) * p.row_bytes, ep_recv_rows(mine, p) + src * p.row_bytes,
                   p.row_bytes, lane);
    if (lane == 0) {
      if (row_map != nullptr) row_map[dst] = static_cast<int32_t>(src);
      if (peer_row_map != nullptr) {
        const int64_t crow = min64(s_dst[s] + static_cast<int64_t>(j), p.comb_rows - 1);
        peer_row_map[dst] = (s << kPeerRowBits) | static_cast<int32_t>(crow);
      }
    }
  }
  if (last_cta(p.ticket, &s_last) && threadIdx.x == 0) {
    *expect = s_target;
    *meta_expect += 1u;  // the counts arrived with the rows; keep the meta count in step
    *p.ticket = 0u;
  }
}

// ------------------------------------------------------------------ combine send
// y_recv holds the expert outputs in arrival order: row s*cap_rows + j is row j of
// source s.  They go back to s.comb starting at s's first send row for this rank.
__global__ void __launch_bounds__(256) ep_combine_send_kernel(const __grid_constant__ EpParams p, const uint8_t* y_recv) {
  __shared__ int s_row[EP_MAX_RANKS + 1];  // first packed row per source
  __shared__ int s_dst[EP_MAX_RANKS];      // first comb row at the source
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int G = p.G, P = p.P;
  if (threadIdx.x < G) {
    const int s = threadIdx.x;
    const volatile int32_t* meta = ep_meta(p.peer[p.rank], p) + s * (P + 1);
    int run = 0;
    for (int q = 0; q < P; ++q) run += clamp_run(meta[q], run, p.cap_rows);
    int dst = meta[P];
    if (dst < 0 || dst > p.comb_rows) {
      record_status(p.status, kStatusBadIndex);
      dst = 0;
      run = 0;
    }
    s_row[s + 1] = static_cast<int>(min64(run, p.comb_rows - dst));  // count; prefix below
    s_dst[s] = dst;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_row[0] = 0;
    for (int s = 0; s < G; ++s) s_row[s + 1] += s_row[s];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int i = blockIdx.x * (blockDim.x >> 5) + warp; i < s_row[G]; i += nwarps) {
    int s = 0;
    while (s + 1 < G && i >= s_row[s + 1]) ++s;
    const int j = i - s_row[s];
    copy_row<false>(ep_comb_rows(p.peer[s], p) + (static_cast<int64_t>(s_dst[s]) + j) * p.row_bytes,
                    y_recv + (static_cast<int64_t>(s) * p.cap_rows + j) * p.row_bytes, p.row_bytes, lane);
  }
  if (last_cta(p.ticket, &s_last) && threadIdx.x < G) {
    __threadfence_system();
    atomicAdd_system(ep_flags(p.peer[threadIdx.x]) + G + p.rank, 1u);  // s.comb[rank] += 1
    if (threadIdx.x == 0) *p.ticket = 0u;
  }
}

// ------------------------------------------------------------------ wait for combine rows
__global__ void ep_wait_comb_kernel(const __grid_constant__ EpParams p, uint32_t* expect, uint64_t timeout_ns) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0) return;
  const uint32_t target = *expect + 1u;
  const uint32_t* flags = ep_flags(p.peer[p.rank]) + p.G;
  bool ok = true;
  for (int d = 0; d < p.G && ok; ++d) ok = wait_flag_geq(flags + d, target, timeout_ns, p.status);
  if (!ok) record_status(p.status, kStatusTimeout);
  *expect = target;
}

// One warp per row in flight; up to 6 CTAs of 8 warps per SM so that large copies keep
// enough loads outstanding to stream at HBM / NVLink speed.
static int grid_for_rows(int64_t rows) {
  return static_cast<int>(max64(1, min64(6 * num_sms(), (rows + 7) / 8)));
}

int launch_ep_dispatch(const EpParams& p, const void* send, const int32_t* slot_offsets, int64_t max_rows,
                       cudaStream_t stream) {
  return launch_kernel(ep_dispatch_kernel, dim3(grid_for_rows(max_rows)), dim3(256), 0, stream, p,
                       static_cast<const uint8_t*>(send), slot_offsets) == cudaSuccess
             ? 0
             : -2;
}

int launch_ep_collect(const EpParams& p, void* xe, int32_t* row_map, int32_t* peer_row_map,
                      int32_t* expert_offsets, uint32_t* expect, uint32_t* meta_expect, uint64_t timeout_ns,
                      int64_t max_rows, cudaStream_t stream) {
  const size_t smem = sizeof(int32_t) * (2 * p.G * p.P + p.G + 1 + p.P + 1);
  return launch_kernel(ep_collect_kernel, dim3(grid_for_rows(max_rows)), dim3(256), smem, stream, p,
                       static_cast<uint8_t*>(xe), row_map, peer_row_map, expert_offsets, expect, meta_expect,
                       timeout_ns) == cudaSuccess
             ? 0
             : -2;
}

int launch_ep_combine_send(const EpParams& p, const void* y_recv, int64_t max_rows, cudaStream_t stream) {
  return launch_kernel(ep_combine_send_kernel, dim3(grid_for_rows(max_rows)), dim3(256), 0, stream, p,
                       static_cast<const uint8_t*>(y_recv)) == cudaSuccess
             ? 0
             : -2;
}

int launch_ep_wait_comb(const EpParams& p, uint32_t* expect, uint64_t timeout_ns, cudaStream_t stream) {
  return launch_kernel(ep_wait_comb_kernel, dim3(1), dim3(32), 0, stream, p, expect, timeout_ns) == cudaSuccess
             ? 0
             : -2;
}

}  // namespace b200moe
