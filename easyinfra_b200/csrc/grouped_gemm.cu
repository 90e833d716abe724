// Kernel family (3): grouped expert GEMMs on 5th-generation tensor cores.
//
// Replaces the reference's expert FFN (NativeMoE.forward_ep, easyinfra/generation/
// modules/moe/native_moe.py:56-103; TritonExperts.forward_ep + fused_moe_kernel,
// modules/moe/fused_moe.py:213-296, 379-478):
//   for every local expert e and its rows X_e:
//     H_e = silu(X_e W_gate,e^T) * (X_e W_up,e^T)     (GEMM1, SwiGLU fused in epilogue)
//     Y_e = H_e W_down,e^T                             (GEMM2)
// Weights keep the reference's stacked layout: gate_up [P, 2I, H] (gate rows 0..I-1,
// up rows I..2I-1, MergedColumnParallelLinear order) and down [P, H, I].
//
// Design (sm_100a):
//   * persistent kernel, one CTA per SM, static round-robin over a device-side tile
//     list (expert, n-tile, m-tile) with m fastest so that all m-tiles of one weight
//     n-tile run concurrently and share it through L2;
//   * warp 0 = TMA producer (128B-swizzled K-major tiles, STAGES-deep ring),
//     warp 1 = TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16),
//     warps 2..5 = epilogue (tcgen05.ld 32x32b from a double-buffered fp32
//     accumulator, SwiGLU in fp32, bf16 rounding once, optional row scatter);
//   * GEMM1 loads the gate and up rows of the same intermediate columns into one
//     B tile (two TMA boxes) so the accumulator holds [gate | up] side by side and
//     the intermediate never round-trips through HBM in fp32 or unfused form;
//   * no cluster launch: every CTA loads its own tiles with plain TMA loads.
// Every mbarrier wait is bounded; on timeout the CTA records kStatusTimeout, drains
// and frees its TMEM.
#include <atomic>

#include "kernels.cuh"

namespace b200moe {

constexpr int GM_BM = 128;
constexpr int GM_BK = 64;  // 64 bf16 = 128 B = one swizzle row
constexpr int GM_UMMA_K = 16;
constexpr int GM_MAXP = 512;
constexpr int GM_THREADS = 192;

// BMA = activation rows loaded per tile (GM_BM for prefill; fewer for decode, where an
// expert sees only a few rows: the MMA still runs M = 128 and the accumulator rows
// past BMA are never stored, but only BMA rows cross L2 per k-block).
template <int BN, int STAGES, bool SWIGLU, int BMA = GM_BM>
struct GemmShape {
  static constexpr int A_BYTES = GM_BM * GM_BK * 2;     // smem per A stage (MMA reads 128 rows)
  static constexpr int A_LOAD_BYTES = BMA * GM_BK * 2;  // bytes TMA writes per A stage
  static constexpr int B_BYTES = BN * GM_BK * 2;
  static constexpr int OUT_COLS = SWIGLU ? BN / 2 : BN;
  static constexpr int TMEM_COLS = 2 * BN;  // two fp32 accumulators
  static constexpr int CTRL_BYTES = 512 + 2 * (GM_MAXP + 1) * 4;  // barriers, flags, prefix, offsets
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + CTRL_BYTES;
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM columns");
  static_assert(BN % 32 == 0 && BN <= 256, "BN");
  static_assert(BMA % 32 == 0 && BMA <= GM_BM, "BMA");
};

template <int BMA>
__device__ __forceinline__ void decode_tile(const int* prefix, const int32_t* off, int P, int tile,
                                            int& e, int& m, int& n) {
  int lo = 0, hi = P - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  e = lo;
  const int local = tile - prefix[e];
  const int rows = off[e + 1] - off[e];
  const int mt = (rows + BMA - 1) / BMA;
  n = local / mt;
  m = local - n * mt;
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

template <int BN, int STAGES, bool SWIGLU, int BMA>
__global__ void __launch_bounds__(GM_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_b, const __grid_constant__ GemmParams p) {
  using S = GemmShape<BN, STAGES, SWIGLU, BMA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + STAGES * S::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* prefix = reinterpret_cast<int*>(tmem_holder + 2);  // [P+1] tile prefix
  int32_t* off = prefix + (GM_MAXP + 1);                   // [P+1] expert row offsets (copy)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (p.N + S::OUT_COLS - 1) / S::OUT_COLS;
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
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::TMEM_COLS);
    tmem_relinquish();
  }
  pdl_wait();  // inputs of this launch are complete and visible from here on
  if (warp == 2) {
    int run = 0;
    for (int base = 0; base <= p.P; base += 32) {
      const int e = base + lane;
      if (e <= p.P) off[e] = p.expert_offsets[e];
    }
    __syncwarp();
    for (int base = 0; base < p.P; base += 32) {
      const int e = base + lane;
      int c = 0;
      if (e < p.P) {
        const int rows = off[e + 1] - off[e];
        c = ((rows + BMA - 1) / BMA) * nt;
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
  const int num_kb = (p.K + GM_BK - 1) / GM_BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        int e, m, n;
        decode_tile<BMA>(prefix, off, p.P, tile, e, m, n);
        const int row_a = off[e] + m * BMA;
        const int row_b = e * p.w_rows + n * S::OUT_COLS;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], S::A_LOAD_BYTES + S::B_BYTES);
          tma_load_2d(sa + stage * S::A_BYTES, &map_a, &full[stage], kb * GM_BK, row_a);
          if (SWIGLU) {
            uint8_t* dst = sb + stage * S::B_BYTES;
            tma_load_2d(dst, &map_b, &full[stage], kb * GM_BK, row_b);
            tma_load_2d(dst + (BN / 2) * 128, &map_b, &full[stage], kb * GM_BK, row_b + p.up_row);
          } else {
            tma_load_2d(sb + stage * S::B_BYTES, &map_b, &full[stage], kb * GM_BK, row_b);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16_f32(GM_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(sa + stage * S::A_BYTES));
          const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sb + stage * S::B_BYTES));
#pragma unroll
          for (int k = 0; k < GM_BK / GM_UMMA_K; ++k) {
            // advance the start address by k * 16 elements * 2 B = 32 B (encoded >> 4)
            umma_bf16(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
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
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row_in_tile = quarter * 32 + lane;
    const bool warp_has_rows = quarter * 32 < BMA;  // lanes past BMA hold no loaded rows
    int acc = 0;
    uint32_t acc_phase = 0;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      int e, m, n;
      decode_tile<BMA>(prefix, off, p.P, tile, e, m, n);
      const int rows = off[e + 1] - off[e];
      const int r = m * BMA + row_in_tile;
      const bool valid = warp_has_rows && r < rows;
      const int64_t grow = static_cast<int64_t>(off[e]) + r;
      int64_t orow = grow;
      __nv_bfloat16* peer_row = nullptr;
      if (valid && p.peer_out)
        peer_row = static_cast<__nv_bfloat16*>(peer_out_row(p.po, p.out_row_map[grow], p.ldo * 2));
      else if (valid && p.out_row_map != nullptr)
        orow = p.out_row_map[grow];
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      __nv_bfloat16* orow_ptr = p.peer_out ? peer_row : out + orow * p.ldo;
      if (!warp_has_rows) {
        // nothing of this tile lives in this warp's TMEM lanes
      } else if (SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + c, g);
          tmem_ld_32x32b_x32(tbase + BN / 2 + c, u);
          tmem_ld_wait();
          const int col = n * S::OUT_COLS + c;
          if (valid) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float h0 = silu_mul(__uint_as_float(g[2 * j]), __uint_as_float(u[2 * j]));
              const float h1 = silu_mul(__uint_as_float(g[2 * j + 1]), __uint_as_float(u[2 * j + 1]));
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
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
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
      if (lane == 0) mbar_arrive(&tempty[acc]);
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

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static const EncodeTiledFn fn = [] {  // looked up once, thread-safe initialisation
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(ptr);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

// 2D bf16 K-major map: rows x cols (cols contiguous, row stride ld elements), box
// box_rows x 64 with the 128-byte swizzle.
int make_tma_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(GM_BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <int BN, int STAGES, bool SWIGLU, int BMA>
static int run_gemm(const GemmLaunch& L, cudaStream_t stream) {
  using S = GemmShape<BN, STAGES, SWIGLU, BMA>;
  static_assert(S::SMEM_BYTES <= 232448, "shared memory");
  CUtensorMap ma, mb;
  if (make_tma_map_2d(&ma, L.a, L.rows_cap, L.p.K, L.lda, BMA) != 0) return -1;
  if (make_tma_map_2d(&mb, L.w, static_cast<int64_t>(L.p.P) * L.p.w_rows, L.p.K, L.p.K,
                  SWIGLU ? BN / 2 : BN) != 0)
    return -1;
  // Request at least half the SM's shared memory so two CTAs never share one SM
  // (each holds TMEM_COLS of the 512 TMEM columns for its whole lifetime).
  const int smem = S::SMEM_BYTES > 120 * 1024 ? S::SMEM_BYTES : 120 * 1024;
  static std::atomic<uint64_t> attr_set_mask{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set_mask.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(grouped_gemm_kernel<BN, STAGES, SWIGLU, BMA>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return -3;
    attr_set_mask.fetch_or(bit, std::memory_order_release);
  }
  const int nt = (L.p.N + S::OUT_COLS - 1) / S::OUT_COLS;
  const int64_t bound = ((L.rows_cap + BMA - 1) / BMA + L.p.P) * static_cast<int64_t>(nt);
  const int limit = gemm_grid_limit();
  const int grid = static_cast<int>(bound < limit ? bound : limit);
  if (grid <= 0) return 0;
  launch_kernel(grouped_gemm_kernel<BN, STAGES, SWIGLU, BMA>, dim3(grid), dim3(GM_THREADS), smem, stream, ma, mb,
                L.p);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Decode regime: the GEMM streams weights and is HBM-bound, and the weight-major
// kernel (grouped_gemm_wm.cu) keeps the most weight bytes in flight — when slots have
// few rows on average, and, for the down GEMM, also when its token-major tiles (128
// rows x 256 output columns) are too few to give every SM one: a shared expert over a
// decode batch, or one expert per rank, would otherwise stream its long-K weights with
// a tenth of the SMs (measured with 128 rows: Mixtral's down GEMM 92 -> 71 us, Qwen1.5's
// shared down 39 -> 32 us; the SwiGLU GEMM at those shapes is faster token-major).
// The token-major kernel with 32-row activation tiles remains available
// (GemmVariant::kTokenMajorSmallM) for comparison.
static bool decode_regime(const GemmLaunch& L) {
  const int64_t rows = L.rows_hint > 0 ? L.rows_hint : L.rows_cap;
  if (rows <= 48 * static_cast<int64_t>(L.p.P)) return true;
  if (L.p.w_rows == 2 * L.p.N) return false;  // SwiGLU
  const int64_t token_tiles = ((rows + GM_BM - 1) / GM_BM + L.p.P - 1) * ((L.p.N + 2 * GM_BM - 1) / (2 * GM_BM));
  return token_tiles < num_sms();
}

// Prefill regime with full 256-row pair tiles on average: the CTA-pair kernel
// (grouped_gemm_2sm.cu), which stages a third fewer shared-memory bytes per FLOP.
static bool pair_regime(const GemmLaunch& L) {
  const int64_t rows = L.rows_hint > 0 ? L.rows_hint : L.rows_cap;
  return rows >= 256 * static_cast<int64_t>(L.p.P);
}

int launch_grouped_swiglu(const GemmLaunch& L, cudaStream_t stream) {
  if (L.p.P > GM_MAXP) return -4;
  const int v = L.variant;
  if (v == kGemmWeightMajor || v == kGemmWeightMajorWide || (v == kGemmAuto && decode_regime(L)))
    return launch_grouped_wm(L, true, v == kGemmAuto ? -1 : (v == kGemmWeightMajorWide ? 1 : 0), stream);
  if (v == kGemmTokenMajorSmallM) return run_gemm<64, 9, true, 32>(L, stream);
  if ((v == kGemmTokenMajorPair || (v == kGemmAuto && pair_regime(L))) && pair_gemm_supported(L, true))
    return launch_grouped_pair(L, true, stream);
  return run_gemm<256, 4, true, GM_BM>(L, stream);
}

int launch_grouped_down(const GemmLaunch& L, cudaStream_t stream) {
  if (L.p.P > GM_MAXP) return -4;
  const int v = L.variant;
  if (v == kGemmWeightMajor || v == kGemmWeightMajorWide || (v == kGemmAuto && decode_regime(L)))
    return launch_grouped_wm(L, false, v == kGemmAuto ? -1 : (v == kGemmWeightMajorWide ? 1 : 0), stream);
  if (v == kGemmTokenMajorSmallM) return run_gemm<64, 9, false, 32>(L, stream);
  if ((v == kGemmTokenMajorPair || (v == kGemmAuto && pair_regime(L))) && pair_gemm_supported(L, false))
    return launch_grouped_pair(L, false, stream);
  return run_gemm<256, 4, false, GM_BM>(L, stream);
}

}  // namespace b200moe
