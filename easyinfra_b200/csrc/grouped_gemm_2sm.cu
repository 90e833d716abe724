// Kernel family (3), prefill form on CTA pairs: grouped expert GEMMs with
// tcgen05.mma.cta_group::2 (M = 256 rows per MMA across the two CTAs of a cluster).
//
// Same contract as grouped_gemm.cu (rows of expert e are [off[e], off[e+1]) of A,
// weights [P, w_rows, K], SwiGLU fused, optional row scatter / peer output), same
// arithmetic (bf16 operands, fp32 accumulation, one rounding).  What changes is how
// the operands reach the tensor cores: a pair tile is 256 activation rows x 256
// weight rows; CTA r of the pair loads activation rows [128r, 128r + 128) and weight
// rows [128r, 128r + 128) of the tile (for SwiGLU: CTA 0 the gate rows, CTA 1 the up
// rows of the same 128 intermediate columns), and the even CTA issues one M = 256,
// N = 256 MMA that reads both CTAs' shared memory.  Each CTA therefore stages 32 KB
// per k-block instead of 48 KB for the same FLOPs, which leaves room for 6 stages.
//
// Roles (192 threads per CTA):
//   warp 0   TMA producer in both CTAs; loads complete on the even CTA's full barrier;
//   warp 1   TMEM allocation (both CTAs, cta_group::2) and, in the even CTA, the MMA
//            issuer, whose commits arrive on the empty / accumulator-full barriers of
//            both CTAs at once (tcgen05.commit to the pair);
//   warps 2-5 epilogue in both CTAs (each drains its own 128 accumulator rows and
//            arrives on the even CTA's accumulator-empty barrier).
// Every mbarrier wait is bounded (kWaitLimitNs); both CTAs meet at a cluster barrier
// after initialisation and before TMEM is freed.  No load is shared across CTAs:
// each CTA's TMA writes only its own shared memory.
#include <atomic>
#include <cstdlib>

#include "kernels.cuh"

namespace b200moe {

constexpr int G2_ROWS = 128;  // activation rows per CTA (pair tile: 256)
constexpr int G2_BK = 64;
constexpr int G2_UMMA_K = 16;
constexpr int G2_MAXP = 512;
constexpr int G2_THREADS = 192;
constexpr uint16_t G2_PAIR_MASK = 0x3;  // both CTAs of the cluster

template <int STAGES, bool SWIGLU>
struct PairShape {
  static constexpr int A_BYTES = G2_ROWS * G2_BK * 2;  // 16 KB
  static constexpr int B_BYTES = 128 * G2_BK * 2;      // this CTA's 128 of the tile's 256 weight rows
  static constexpr int N = 256;                        // accumulator columns
  static constexpr int OUT_COLS = SWIGLU ? 128 : 256;  // output columns per tile
  static constexpr int TMEM_COLS = 2 * N;              // two fp32 accumulators
  static constexpr int CTRL_BYTES = 512 + 3 * (G2_MAXP + 1) * 4 + 64;  // + segment lengths, dst rows
  // down GEMM, rows sent to peers: per epilogue warp, 32 output rows x 64 columns
  // staged in shared memory (144-byte rows: 128 bytes + 16 of padding)
  static constexpr int STG_LD = 144;
  static constexpr int STG_BYTES = SWIGLU ? 0 : 4 * 32 * STG_LD;
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + STG_BYTES + CTRL_BYTES;
};

// tile -> (group, n-tile, m-tile) with 256-row m-tiles, m fastest.  A group is an
// expert (rows off[g] .. off[g+1]) or, reading a receive region, a (source, slot)
// segment (rows off[g] .. off[g] + len[g]).
__device__ __forceinline__ int group_rows(const int32_t* off, const int32_t* len, bool seg, int g) {
  return seg ? len[g] : off[g + 1] - off[g];
}

// ng > 0: n-tiles are visited in bands of ng, and inside a band the tiles of one
// m-tile are consecutive — a wave of concurrent tiles then covers a compact block of
// m x n tiles, so both operands are reused from L2 (ng = 0: m fastest).
__device__ __forceinline__ void pair_decode_tile(const int* prefix, const int32_t* off, const int32_t* len, bool seg,
                                                 int ngroups, int tile, int nt, int ng, int& e, int& m, int& n) {
  int lo = 0, hi = ngroups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int local = tile - prefix[e];
  const int rows = group_rows(off, len, seg, e);
  const int mt = (rows + 2 * G2_ROWS - 1) / (2 * G2_ROWS);
  if (ng <= 0) {
    n = local / mt;
    m = local - n * mt;
    return;
  }
  const int band = local / (mt * ng);
  const int nb = min(ng, nt - band * ng);  // n-tiles in this band
  const int li = local - band * mt * ng;
  m = li / nb;
  n = band * ng + (li - m * nb);
}

__device__ __forceinline__ float pair_silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

template <int STAGES, bool SWIGLU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(G2_THREADS, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                             const __grid_constant__ GemmParams p) {
  using S = PairShape<STAGES, SWIGLU>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * S::A_BYTES;
  uint8_t* stg = sb + STAGES * S::B_BYTES;  // epilogue staging (down GEMM, peer rows)
  uint64_t* full = reinterpret_cast<uint64_t*>(stg + S::STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* prefix = reinterpret_cast<int*>(tmem_holder + 2);  // [groups+1] tile prefix
  int32_t* off = prefix + (G2_MAXP + 1);                   // [groups+1] first row of each group
  int32_t* glen = off + (G2_MAXP + 1);                     // [groups] segment rows (receive region)
  int32_t* s_dst = glen + (G2_MAXP + 1);                   // [G] first combine row at each source
  volatile uint32_t* s_target = reinterpret_cast<volatile uint32_t*>(s_dst + EP_MAX_RANKS);  // rows, meta

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nt = (p.N + S::OUT_COLS - 1) / S::OUT_COLS;
  const bool seg = p.seg_mode != 0;
  const int ngroups = seg ? p.seg.G * p.P : p.P;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // even CTA: its producer's arrive + both CTAs' bytes
      mbar_init(&empty[s], 1);  // the MMA commit, in both CTAs
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);   // the MMA commit, in both CTAs
      mbar_init(&tempty[a], 8);  // even CTA: 4 epilogue warps of each CTA
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive / load
  pdl_wait();
  if (warp == 2) {
    if (!seg) {
      for (int base = 0; base <= p.P; base += 32) {
        const int e = base + lane;
        if (e <= p.P) off[e] = p.expert_offsets[e];
      }
    } else {
      // receive-region groups: (source, slot) segments, sources from this rank onwards
      const SegIn& sg = p.seg;
      if (lane == 0) {
        const uint32_t mt = *sg.meta_expect + (sg.consume ? 1u : 0u);
        const uint32_t rt = *sg.rows_expect + (sg.consume ? 1u : 0u);
        if (sg.consume) {
          bool ok = true;
          for (int s = 0; s < sg.G && ok; ++s) ok = wait_flag_geq(sg.meta_flag + s, mt, sg.timeout_ns, p.status);
          if (!ok) record_status(p.status, kStatusTimeout);
        }
        s_target[0] = rt;
        s_target[1] = mt;
      }
      __syncwarp();
      if (lane < sg.G) {
        const int src = (sg.rank + lane) % sg.G;
        const volatile int32_t* meta = sg.meta + src * (p.P + 1);
        int run = 0;
        for (int q = 0; q < p.P; ++q) {
          const int c = clamp_run(meta[q], run, sg.cap_rows);
          off[lane * p.P + q] = static_cast<int32_t>(src * sg.cap_rows + run);
          glen[lane * p.P + q] = c;
          run += c;
        }
        int dst = meta[p.P];
        if (dst < 0 || static_cast<int64_t>(dst) + run > sg.comb_rows) {
          if (p.peer_out) record_status(p.status, kStatusBadIndex);
          dst = 0;  // keeps every return row inside the source's combine region
        }
        s_dst[src] = dst;
      }
    }
    __syncwarp();
    int run = 0;
    for (int base = 0; base < ngroups; base += 32) {
      const int e = base + lane;
      int c = 0;
      if (e < ngroups) c = ((group_rows(off, glen, seg, e) + 2 * G2_ROWS - 1) / (2 * G2_ROWS)) * nt;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < ngroups) prefix[e] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[ngroups] = run;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = prefix[ngroups];
  const int num_kb = (p.K + G2_BK - 1) / G2_BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // the even CTA's full barriers
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t ready = 0;  // receive region: sources whose rows have arrived
      for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
        int g, m, n;
        pair_decode_tile(prefix, off, glen, seg, ngroups, tile, nt, p.tile_band, g, m, n);
        const int e = seg ? g % p.P : g;  // weight slot
        if (seg && p.seg.consume && !((ready >> (g / p.P)) & 1u)) {
          // this tile's rows come from one source: wait (bounded) for its rows flag,
          // then order the tensor loads after that acquire
          const int src = (p.seg.rank + g / p.P) % p.seg.G;
          if (!wait_flag_geq(p.seg.rows_flag + src, s_target[0], p.seg.timeout_ns, p.status))
            record_status(p.status, kStatusTimeout);
          asm volatile("fence.proxy.async.global;" ::: "memory");
          ready |= 1u << (g / p.P);
        }
        const int row_a = off[g] + m * 2 * G2_ROWS + static_cast<int>(crank) * G2_ROWS;
        const int row_b = e * p.w_rows + n * S::OUT_COLS +
                          (SWIGLU ? (crank ? p.up_row : 0) : static_cast<int>(crank) * 128);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (S::A_BYTES + S::B_BYTES));
          const uint32_t fb = full0 + stage * 8;
          tma_load_2d_pair(sa + stage * S::A_BYTES, &map_a, fb, kb * G2_BK, row_a);
          tma_load_2d_pair(sb + stage * S::B_BYTES, &map_b, fb, kb * G2_BK, row_b);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      // ------------------------------------------------ MMA issuer (even CTA)
      constexpr uint32_t idesc = make_idesc_bf16_f32(2 * G2_ROWS, S::N);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * S::N);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(sa + stage * S::A_BYTES));
          const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sb + stage * S::B_BYTES));
#pragma unroll
          for (int k = 0; k < G2_BK / G2_UMMA_K; ++k)
            umma_bf16_pair(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&empty[stage], G2_PAIR_MASK);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], G2_PAIR_MASK);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // -------------------------------------------------- epilogue (warps 2..5, both CTAs)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
    for (int tile = pair; tile < total_tiles; tile += npairs) {
      int g, m, n;
      pair_decode_tile(prefix, off, glen, seg, ngroups, tile, nt, p.tile_band, g, m, n);
      const int rows = group_rows(off, glen, seg, g);
      const int r = m * 2 * G2_ROWS + static_cast<int>(crank) * G2_ROWS + row_in_tile;
      const bool valid = r < rows;
      const int64_t grow = static_cast<int64_t>(off[g]) + r;
      int64_t orow = grow;
      __nv_bfloat16* peer_row = nullptr;
      if (valid && p.peer_out) {
        int32_t v;
        if (seg) {
          // row j of source src's region returns to row s_dst[src] + j of src's combine region
          const int src = (p.seg.rank + g / p.P) % p.seg.G;
          const int64_t j = grow - static_cast<int64_t>(src) * p.seg.cap_rows;
          v = (src << kPeerRowBits) | static_cast<int32_t>(s_dst[src] + j);
        } else {
          v = p.out_row_map[grow];
        }
        peer_row = static_cast<__nv_bfloat16*>(peer_out_row(p.po, v, p.ldo * 2));
      } else if (valid && p.out_row_map != nullptr) {
        orow = p.out_row_map[grow];
      }
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * S::N);
      __nv_bfloat16* orow_ptr = p.peer_out ? peer_row : out + orow * p.ldo;
      if (SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < S::N / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + c, g);
          tmem_ld_32x32b_x32(tbase + S::N / 2 + c, u);
          tmem_ld_wait();
          const int col = n * S::OUT_COLS + c;
          if (valid) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float h0 = pair_silu_mul(__uint_as_float(g[2 * j]), __uint_as_float(u[2 * j]));
              const float h1 = pair_silu_mul(__uint_as_float(g[2 * j + 1]), __uint_as_float(u[2 * j + 1]));
              packed[j] = pack_bf16x2(h0, h1);
            }
            if (col + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(orow_ptr + col);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            } else {
              const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(packed);
              for (int j = 0; j < 32 && col + j < p.N; ++j) orow_ptr[col + j] = hb[j];
            }
          }
        }
      } else if (p.peer_out) {
        // Rows go to other GPUs: a thread holds one output row, so storing straight from
        // registers would scatter 16-byte pieces over 32 rows per warp instruction, each
        // a separate small NVLink write.  Stage the warp's 32 rows x 64 columns in shared
        // memory and store whole 128-byte row segments instead (8 lanes per row, 4 rows
        // per instruction).
        uint8_t* my = stg + quarter * (32 * S::STG_LD);
        const unsigned long long rp = reinterpret_cast<unsigned long long>(orow_ptr);
        const int vflag = valid ? 1 : 0;
#pragma unroll 1
        for (int c = 0; c < S::N; c += 64) {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(tbase + c, v0);
          tmem_ld_32x32b_x32(tbase + c + 32, v1);
          tmem_ld_wait();
          uint4* srow = reinterpret_cast<uint4*>(my + lane * S::STG_LD);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            srow[q] = make_uint4(pack_bf16x2(__uint_as_float(v0[8 * q]), __uint_as_float(v0[8 * q + 1])),
                                 pack_bf16x2(__uint_as_float(v0[8 * q + 2]), __uint_as_float(v0[8 * q + 3])),
                                 pack_bf16x2(__uint_as_float(v0[8 * q + 4]), __uint_as_float(v0[8 * q + 5])),
                                 pack_bf16x2(__uint_as_float(v0[8 * q + 6]), __uint_as_float(v0[8 * q + 7])));
            srow[4 + q] = make_uint4(pack_bf16x2(__uint_as_float(v1[8 * q]), __uint_as_float(v1[8 * q + 1])),
                                     pack_bf16x2(__uint_as_float(v1[8 * q + 2]), __uint_as_float(v1[8 * q + 3])),
                                     pack_bf16x2(__uint_as_float(v1[8 * q + 4]), __uint_as_float(v1[8 * q + 5])),
                                     pack_bf16x2(__uint_as_float(v1[8 * q + 6]), __uint_as_float(v1[8 * q + 7])));
          }
          __syncwarp();
          const int col = n * S::OUT_COLS + c;  // a multiple of 64; the pair down GEMM has N % 256 == 0
#pragma unroll
          for (int pass = 0; pass < 8; ++pass) {
            const int row = pass * 4 + (lane >> 3), piece = lane & 7;
            const unsigned long long dst = __shfl_sync(0xffffffffu, rp, row);
            const int vrow = __shfl_sync(0xffffffffu, vflag, row);
            if (vrow) {
              const uint4 val = reinterpret_cast<const uint4*>(my + row * S::STG_LD)[piece];
              reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + col)[piece] = val;
            }
          }
          __syncwarp();
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < S::N; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + c, v);
          tmem_ld_wait();
          const int col = n * S::OUT_COLS + c;
          if (valid) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
              packed[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
            if (col + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(orow_ptr + col);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            } else {
              const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(packed);
              for (int j = 0; j < 32 && col + j < p.N; ++j) orow_ptr[col + j] = hb[j];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (crank == 0)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_remote(tempty0 + acc * 8);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or exits while the pair still works
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
  if (p.peer_out) {
    __shared__ int s_last;
    peer_out_publish(p.po, &s_last);
  }
  if (seg && p.seg.consume) {
    // the last CTA records the arrivals this launch consumed
    __shared__ int s_seg_last;
    __syncthreads();
    if (threadIdx.x == 0) s_seg_last = (atomicAdd(p.seg.ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (s_seg_last && threadIdx.x == 0) {
      *p.seg.rows_expect = s_target[0];
      *p.seg.meta_expect = s_target[1];
      *p.seg.ticket = 0u;
    }
  }
}

template <int STAGES, bool SWIGLU>
static int run_pair(const GemmLaunch& L0, cudaStream_t stream) {
  using S = PairShape<STAGES, SWIGLU>;
  // B200MOE_PAIR_BAND=k visits n-tiles in bands of k (0 / unset: m fastest)
  static const int band = [] {
    const char* v = getenv("B200MOE_PAIR_BAND");
    return v ? atoi(v) : 0;
  }();
  GemmLaunch L = L0;
  L.p.tile_band = band;
  static_assert(S::SMEM_BYTES <= 232448, "shared memory");
  CUtensorMap ma, mb;
  if (make_tma_map_2d(&ma, L.a, L.rows_cap, L.p.K, L.lda, G2_ROWS) != 0) return -1;
  if (make_tma_map_2d(&mb, L.w, static_cast<int64_t>(L.p.P) * L.p.w_rows, L.p.K, L.p.K, 128) != 0) return -1;
  static std::atomic<uint64_t> attr_set_mask{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set_mask.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(grouped_gemm_pair_kernel<STAGES, SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             S::SMEM_BYTES) != cudaSuccess)
      return -3;
    attr_set_mask.fetch_or(bit, std::memory_order_release);
  }
  const int nt = (L.p.N + S::OUT_COLS - 1) / S::OUT_COLS;
  const int groups = L.p.seg_mode ? L.p.seg.G * L.p.P : L.p.P;
  const int64_t bound = ((L.rows_cap + 2 * G2_ROWS - 1) / (2 * G2_ROWS) + groups) * static_cast<int64_t>(nt);
  const int limit = gemm_grid_limit() / 2;
  const int pairs = static_cast<int>(bound < limit ? bound : limit);
  if (pairs <= 0) return 0;
  launch_kernel(grouped_gemm_pair_kernel<STAGES, SWIGLU>, dim3(2 * pairs), dim3(G2_THREADS), S::SMEM_BYTES,
                stream, ma, mb, L.p);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// The SwiGLU form needs the 128 gate and 128 up rows of a tile to be separate boxes
// (I % 128 == 0); the down form needs H % 256 == 0.  Callers fall back to the
// single-CTA kernel otherwise.
bool pair_gemm_supported(const GemmLaunch& L, bool swiglu) {
  if ((L.p.seg_mode ? L.p.seg.G * L.p.P : L.p.P) > G2_MAXP) return false;
  return swiglu ? (L.p.N % 128 == 0) : (L.p.N % 256 == 0);
}

int launch_grouped_pair(const GemmLaunch& L, bool swiglu, cudaStream_t stream) {
  return swiglu ? run_pair<6, true>(L, stream) : run_pair<6, false>(L, stream);
}

}  // namespace b200moe
