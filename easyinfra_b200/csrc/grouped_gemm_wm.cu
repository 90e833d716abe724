// Kernel family (3), decode regime: "weight-major" grouped expert GEMMs.
//
// Same contract as grouped_gemm.cu (expert-major rows, stacked weights, fused
// SwiGLU, optional output row map) with the operands swapped for few tokens per
// expert: the streamed weights are the MMA's A operand (M = 128 weight rows) and
// the expert's token rows are B (N = NTOK), so every byte of shared memory in the
// pipeline carries weights and ~10 stages of 16 KB stay in flight per SM — the
// regime is HBM-bound and bytes in flight are what sustain bandwidth.
//   * tile = (expert, feature block, token block): 128 output features (SwiGLU:
//     64 gate + 64 up rows of the same 64 features) x NTOK tokens;
//   * accumulator D[features, tokens] in TMEM (lane = feature), double-buffered;
//   * epilogue: a warp holds 32 consecutive features of every token, so each token's
//     store is one coalesced 64-byte run; for SwiGLU the up half (lanes 64..127) is
//     handed to the gate warps through shared memory;
//   * per-CTA TMA loads only (no clusters), bounded mbarrier waits.
#include <atomic>

#include "kernels.cuh"

namespace b200moe {

constexpr int WM_M = 128;    // weight rows per tile (UMMA M)
constexpr int WM_BK = 64;
constexpr int WM_MAXP = 512;
constexpr int WM_THREADS = 192;

// WIDE: slots with more than NTOK rows get token tiles of 2 * NTOK rows (one N = 64
// MMA per k step), so a heavily routed slot re-reads each weight tile half as often;
// slots with at most NTOK rows keep NTOK-row tiles.  The stage's token buffer is
// sized for the wide tile (fewer stages fit).
template <int NTOK, int STAGES, bool SWIGLU, bool WIDE = false>
struct WmShape {
  static constexpr int TT = WIDE ? 2 * NTOK : NTOK;     // largest token tile
  static constexpr int A_BYTES = WM_M * WM_BK * 2;      // 16 KB of weights per stage
  static constexpr int B_BYTES = TT * WM_BK * 2;        // token rows per stage
  static constexpr int FEAT = SWIGLU ? WM_M / 2 : WM_M; // output features per tile
  static constexpr int TMEM_COLS = (2 * TT < 32) ? 32 : 2 * TT;
  static constexpr int UP_LD = NTOK + 1;                // padded row of the up exchange buffer
  static constexpr int XCHG_BYTES = SWIGLU ? 64 * UP_LD * 4 : 0;
  // down GEMM, rows sent to peers: one epilogue pass (NTOK tokens x 128 features,
  // bf16) staged in shared memory, rows padded to 272 bytes
  static constexpr int STG_LD = WM_M + 8;  // elements
  static constexpr int STG_BYTES = SWIGLU ? 0 : NTOK * STG_LD * 2;
  static constexpr int CTRL_BYTES = 512 + 2 * (WM_MAXP + 1) * 4;
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + XCHG_BYTES + STG_BYTES + CTRL_BYTES;
  static_assert(NTOK % 16 == 0 && NTOK >= 16 && TT <= 256, "UMMA N for M = 128");
  static_assert(NTOK <= 32, "epilogue loads NTOK columns per 32x32b.x32 load");
  static_assert(B_BYTES % 1024 == 0, "token buffers keep the 1024-byte swizzle alignment");
};

// Token rows per tile of a slot with `rows` rows.
template <int NTOK, bool WIDE>
__device__ __forceinline__ int wm_tile_rows(int rows) {
  return (WIDE && rows > NTOK) ? 2 * NTOK : NTOK;
}

// tile -> (expert e, token tile m of tt rows, feature tile n); m is fastest, so the
// token tiles of one weight tile run side by side and share it through L2.
template <int NTOK, bool WIDE>
__device__ __forceinline__ void wm_decode_tile(const int* prefix, const int32_t* off, int P, int tile, int& e,
                                               int& m, int& n, int& tt) {
  int lo = 0, hi = P - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int local = tile - prefix[e];
  const int rows = off[e + 1] - off[e];
  tt = wm_tile_rows<NTOK, WIDE>(rows);
  const int mt = (rows + tt - 1) / tt;
  n = local / mt;
  m = local - n * mt;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int NTOK, int STAGES, bool SWIGLU, bool WIDE>
__global__ void __launch_bounds__(WM_THREADS, 1)
    grouped_gemm_wm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                           const __grid_constant__ CUtensorMap map_x2, const __grid_constant__ GemmParams p) {
  using S = WmShape<NTOK, STAGES, SWIGLU, WIDE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;                                   // weights
  uint8_t* sb = smem + STAGES * S::A_BYTES;             // tokens
  float* up_buf = reinterpret_cast<float*>(sb + STAGES * S::B_BYTES);
  __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(sb + STAGES * S::B_BYTES + S::XCHG_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + STAGES * S::B_BYTES + S::XCHG_BYTES + S::STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* tile_ok = reinterpret_cast<volatile int*>(tmem_holder + 2);  // epilogue handshake
  int* prefix = reinterpret_cast<int*>(tmem_holder + 4);
  int32_t* off = prefix + (WM_MAXP + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (p.N + S::FEAT - 1) / S::FEAT;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
    if (WIDE) tma_prefetch_desc(&map_x2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::TMEM_COLS);
    tmem_relinquish();
  }
  pdl_wait();  // inputs of this launch are complete and visible from here on
  if (warp == 2) {
    for (int base = 0; base <= p.P; base += 32) {
      const int e = base + lane;
      if (e <= p.P) off[e] = p.expert_offsets[e];
    }
    __syncwarp();
    int run = 0;
    for (int base = 0; base < p.P; base += 32) {
      const int e = base + lane;
      int c = 0;
      if (e < p.P) {
        const int rows = off[e + 1] - off[e];
        const int tt = wm_tile_rows<NTOK, WIDE>(rows);
        c = ((rows + tt - 1) / tt) * nt;
      }
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < p.P) prefix[e] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[p.P] = run;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = prefix[p.P];
  const int num_kb = (p.K + WM_BK - 1) / WM_BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const uint64_t stream_once = l2_policy_evict_first();  // weights are read once
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        int e, m, n, tt;
        wm_decode_tile<NTOK, WIDE>(prefix, off, p.P, tile, e, m, n, tt);
        const int row_w = e * p.w_rows + n * S::FEAT;
        const int row_x = off[e] + m * tt;
        const CUtensorMap* mx = (WIDE && tt > NTOK) ? &map_x2 : &map_x;
        const uint32_t tx = S::A_BYTES + static_cast<uint32_t>(tt) * WM_BK * 2;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], tx);
          uint8_t* dst = sa + stage * S::A_BYTES;
          if (SWIGLU) {
            tma_load_2d_hint(dst, &map_w, &full[stage], kb * WM_BK, row_w, stream_once);
            tma_load_2d_hint(dst + 64 * 128, &map_w, &full[stage], kb * WM_BK, row_w + p.up_row, stream_once);
          } else {
            tma_load_2d_hint(dst, &map_w, &full[stage], kb * WM_BK, row_w, stream_once);
          }
          tma_load_2d(sb + stage * S::B_BYTES, mx, &full[stage], kb * WM_BK, row_x);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        int e, m, n, tt;
        wm_decode_tile<NTOK, WIDE>(prefix, off, p.P, tile, e, m, n, tt);
        const uint32_t idesc = make_idesc_bf16_f32(WM_M, tt);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * S::TT);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(sa + stage * S::A_BYTES));
          const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sb + stage * S::B_BYTES));
#pragma unroll
          for (int k = 0; k < WM_BK / 16; ++k)
            umma_bf16(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
    __syncwarp();
  } else {
    // -------------------------------------------------- epilogue (warps 2..5)
    const int quarter = warp & 3;          // TMEM lanes = tile rows (features) 32q..32q+31
    const int feat = quarter * 32 + lane;  // row of the weight tile this thread holds
    int acc = 0;
    uint32_t acc_phase = 0;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int e, m, n, tt;
      wm_decode_tile<NTOK, WIDE>(prefix, off, p.P, tile, e, m, n, tt);
      const int rows = off[e + 1] - off[e];
      const int tok0 = m * tt;
      const int ntok = min(tt, rows - tok0);
      // One thread waits (bounded); the outcome reaches all four epilogue warps through
      // shared memory and the named barrier, so they all continue or all stop together
      // and no warp can be left waiting at a later barrier.
      if (warp == 2 && lane == 0) *tile_ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status) ? 1 : 0;
      epi_bar();
      if (*tile_ok == 0) break;
      // NTOK accumulator columns (tokens) per pass; two passes for a wide tile
      const int passes = (ntok + NTOK - 1) / NTOK;
      for (int h = 0; h < passes; ++h) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(acc * S::TT + h * NTOK),
                           v);
        tmem_ld_wait();
        tc_fence_before();
        if (h == passes - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);  // accumulator copied to registers
        }
        const int t0 = tok0 + h * NTOK;
        const int nt_h = min(NTOK, ntok - h * NTOK);
        if (SWIGLU) {
          if (quarter >= 2) {
            float* u = up_buf + (feat - 64) * S::UP_LD;
#pragma unroll
            for (int j = 0; j < NTOK; ++j) u[j] = __uint_as_float(v[j]);
          }
          epi_bar();
          if (quarter < 2) {
            const int col = n * S::FEAT + feat;
            const float* u = up_buf + feat * S::UP_LD;
            if (col < p.N) {
              for (int j = 0; j < nt_h; ++j) {
                const int64_t grow = static_cast<int64_t>(off[e]) + t0 + j;
                const float g = __uint_as_float(v[j]);
                out[grow * p.ldo + col] = __float2bfloat16_rn(g / (1.f + expf(-g)) * u[j]);
              }
            }
          }
          if (h + 1 < passes) epi_bar();  // up_buf is rewritten by the next pass
        } else if (p.peer_out) {
          // Rows go to other GPUs.  A thread holds one feature of every token, so each
          // warp store would carry only 64 bytes of a row over NVLink; stage the pass as
          // [token][128 features] and store whole 256-byte token rows (16 lanes per row).
          const int col = n * S::FEAT + feat;
          if (col < p.N)
            for (int j = 0; j < nt_h; ++j) stg[j * S::STG_LD + feat] = __float2bfloat16_rn(__uint_as_float(v[j]));
          epi_bar();
          const int nfeat = min(S::FEAT, p.N - n * S::FEAT);
          const int l16 = lane & 15;
          for (int j = quarter * 2 + (lane >> 4); j < nt_h; j += 8) {
            const int64_t grow = static_cast<int64_t>(off[e]) + t0 + j;
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(peer_out_row(p.po, p.out_row_map[grow], p.ldo * 2)) +
                                 n * S::FEAT;
            const __nv_bfloat16* src = stg + j * S::STG_LD;
            if (l16 * 8 + 8 <= nfeat) {
              *reinterpret_cast<uint4*>(dst + l16 * 8) = *reinterpret_cast<const uint4*>(src + l16 * 8);
            } else {
              for (int f = l16 * 8; f < nfeat; ++f) dst[f] = src[f];
            }
          }
          epi_bar();  // the staging buffer is rewritten by the next pass or tile
        } else {
          const int col = n * S::FEAT + feat;
          if (col < p.N) {
            for (int j = 0; j < nt_h; ++j) {
              int64_t grow = static_cast<int64_t>(off[e]) + t0 + j;
              if (p.out_row_map != nullptr) grow = p.out_row_map[grow];
              out[grow * p.ldo + col] = __float2bfloat16_rn(__uint_as_float(v[j]));
            }
          }
        }
      }
      epi_bar();  // tile_ok and up_buf are rewritten for the next tile
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
  if (p.peer_out) {
    __shared__ int s_last;
    peer_out_publish(p.po, &s_last);
  }
}

template <int NTOK, int STAGES, bool SWIGLU, bool WIDE>
static int run_wm(const GemmLaunch& L, cudaStream_t stream) {
  using S = WmShape<NTOK, STAGES, SWIGLU, WIDE>;
  static_assert(S::SMEM_BYTES <= 232448, "shared memory");
  CUtensorMap mw, mx, mx2;
  if (make_tma_map_2d(&mw, L.w, static_cast<int64_t>(L.p.P) * L.p.w_rows, L.p.K, L.p.K,
                      SWIGLU ? WM_M / 2 : WM_M) != 0)
    return -1;
  if (make_tma_map_2d(&mx, L.a, L.rows_cap, L.p.K, L.lda, NTOK) != 0) return -1;
  if (WIDE) {
    if (make_tma_map_2d(&mx2, L.a, L.rows_cap, L.p.K, L.lda, 2 * NTOK) != 0) return -1;
  } else {
    mx2 = mx;
  }
  const int smem = S::SMEM_BYTES > 120 * 1024 ? S::SMEM_BYTES : 120 * 1024;
  static std::atomic<uint64_t> attr_set_mask{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set_mask.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(grouped_gemm_wm_kernel<NTOK, STAGES, SWIGLU, WIDE>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return -3;
    attr_set_mask.fetch_or(bit, std::memory_order_release);
  }
  const int nt = (L.p.N + S::FEAT - 1) / S::FEAT;
  const int64_t bound = ((L.rows_cap + NTOK - 1) / NTOK + L.p.P) * static_cast<int64_t>(nt);
  const int limit = gemm_grid_limit();
  const int grid = static_cast<int>(bound < limit ? bound : limit);
  if (grid <= 0) return 0;
  launch_kernel(grouped_gemm_wm_kernel<NTOK, STAGES, SWIGLU, WIDE>, dim3(grid), dim3(WM_THREADS), smem, stream,
                mw, mx, mx2, L.p);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Wide token tiles (up to 64 rows) pay off when slots carry more than 32 rows: many
// slots and at least 8 rows per slot on average (skewed routing then puts 32+ rows
// on the hot slots).  With fewer rows the 10-stage narrow kernel keeps more weight
// bytes in flight.  wide: 0 = narrow, 1 = wide, -1 = choose.
int launch_grouped_wm(const GemmLaunch& L, bool swiglu, int wide, cudaStream_t stream) {
  if (L.p.P > WM_MAXP) return -4;
  if (wide < 0) {
    const int64_t rows = L.rows_hint > 0 ? L.rows_hint : L.rows_cap;
    wide = (L.p.P >= 32 && rows >= 8 * static_cast<int64_t>(L.p.P)) ? 1 : 0;
  }
  if (wide) return swiglu ? run_wm<32, 8, true, true>(L, stream) : run_wm<32, 8, false, true>(L, stream);
  return swiglu ? run_wm<32, 10, true, false>(L, stream) : run_wm<32, 10, false, false>(L, stream);
}

}  // namespace b200moe
