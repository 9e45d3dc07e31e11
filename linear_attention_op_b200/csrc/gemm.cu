// tcgen05 GEMM for sm_100a: C = A * B^T with A [M, K] and B [N, K] bf16 K-major, fp32 accumulators in
// TMEM.  One CTA computes one 128 x BN tile (or one K-slice of it):
//   warp 0      TMA producer (one elected lane), STAGES-deep ring of 128B-swizzled A/B tiles
//   warp 1      TMEM allocator and UMMA issuer (one elected lane), commits free stages back to warp 0
//   warps 2..5  epilogue: tcgen05.ld of the 32-lane TMEM quarter (warp % 4) -> fused epilogue -> global
// Split-K (skinny decode GEMMs) runs the K-slices of a tile as one thread-block cluster; each slice parks
// its fp32 partial tile in shared memory and then sums a share of the tile's column chunks over all slices
// through distributed shared memory, so the reduction and the epilogue are spread over the cluster.
//
// The two GEMMs of the layer use it as:
//   in_proj  (9B/gdn_layer.py:255-259: ttnn.linear for qkv+z and for a,b) fused into ONE weight
//            [q | k | v | z | a | b] x hidden; decode swaps the operands (weights are A) and fuses the
//            causal conv, the conv-state roll and the gating scalars into the epilogue;
//   out_proj (9B/gdn_layer.py:272-276).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "gemm.cuh"
#include "ptx.cuh"

namespace gdn {

__device__ int g_device_error = 0;

static std::atomic<uint64_t> g_launches{0};
uint64_t launch_count() { return g_launches.load(); }
void count_launch() { g_launches.fetch_add(1); }

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kGemmThreads = 192;

template <int BN, int STAGES>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // barriers + 1 KB alignment slack
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M = 128");
  static_assert(BN * kBM * 4 <= STAGES * kStageBytes, "split-K partial tile must fit in the stage ring");
};

template <int EPI>
__device__ __forceinline__ void epilogue16(const GemmEpiArgs& ep, int m, int n0, int M, int N,
                                           const float (&v)[16]) {
  if constexpr (EPI == kEpiSwiGLUT) {
    // Rows 2j (gate) and 2j + 1 (up) sit in neighbouring lanes: every lane of the warp takes part in the
    // exchange (M is even, so both rows of a pair are in range or neither is).
    float u[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) u[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
    if (m >= M || (m & 1)) return;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(ep.out);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (n0 + j < N) out[static_cast<int64_t>(n0 + j) * ep.ld + (m >> 1)] = __float2bfloat16_rn(silu_fast(v[j]) * u[j]);
    return;
  }
  if (m >= M) return;
  if constexpr (EPI == kEpiStoreF32) {
    float* row = static_cast<float*>(ep.out) + static_cast<int64_t>(m) * ep.ld + n0;
    if (n0 + 16 <= N && (ep.ld & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(row)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) row[j] = v[j];
    }
  } else if constexpr (EPI == kEpiStoreBF16) {
    __nv_bfloat16* row = static_cast<__nv_bfloat16*>(ep.out) + static_cast<int64_t>(m) * ep.ld + n0;
    if (n0 + 16 <= N && (ep.ld & 7) == 0) {
      uint4 pk[2];
      uint32_t* w = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      }
      reinterpret_cast<uint4*>(row)[0] = pk[0];
      reinterpret_cast<uint4*>(row)[1] = pk[1];
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) row[j] = __float2bfloat16_rn(v[j]);
    }
  } else if constexpr (EPI == kEpiStoreF32T) {
    float* out = static_cast<float*>(ep.out);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (n0 + j < N) out[static_cast<int64_t>(n0 + j) * ep.ld + m] = v[j];
  } else if constexpr (EPI == kEpiStoreBF16T) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(ep.out);
    if (ep.residual) {
      const __nv_bfloat16* res = static_cast<const __nv_bfloat16*>(ep.residual);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N)
          out[static_cast<int64_t>(n0 + j) * ep.ld + m] =
              __float2bfloat16_rn(v[j] + __bfloat162float(res[static_cast<int64_t>(n0 + j) * ep.res_ld + m]));
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (n0 + j < N) out[static_cast<int64_t>(n0 + j) * ep.ld + m] = __float2bfloat16_rn(v[j]);
    }
  }
}

// Row and column scales of the fp8 operands (per weight row, per activation row), applied before the
// epilogue proper.
__device__ __forceinline__ void apply_scales(const GemmEpiArgs& ep, int m, int n0, int M, int N, float (&v)[16]) {
  if (!ep.row_scale || m >= M) return;
  const float rs = ep.row_scale[m];
  if (!ep.col_scale) {  // weight-only quantisation: the activations are bf16
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (v[j] * ep.acc_scale) * rs;
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] *= rs * (n0 + j < N ? ep.col_scale[n0 + j] : 0.f);
}

template <int BN, int EPI>
__device__ __forceinline__ void tn_epilogue(uint32_t tmem, uint8_t* smem, const GemmEpiArgs& ep, int m_tile, int n_tile,
                                            int M, int N, int ksplit, int split, int warp, int lane, uint64_t* accum);

// One CTA of the tcgen05 GEMM.  F8: A and B are fp8 e4m3 (kind::f8f6f4, 32-deep MMAs) and a 128-byte
// stage row holds 128 K elements instead of 64; everything else (stage bytes, swizzle, pipeline) is the
// bf16 kernel's.
template <int BN, int STAGES, int EPI, bool F8>
__device__ __forceinline__ void gemm_tn_body(const CUtensorMap& tmA, const CUtensorMap& tmB, int M, int N, int K,
                                             int ksplit, int n_tiles, int group_m, int trigger_early,
                                             const uint8_t* a_tiled, const uint8_t* b_tiled, const GemmEpiArgs& ep) {
  using C = GemmCfg<BN, STAGES>;
  constexpr int kBKe = F8 ? 2 * kBK : kBK;  // K elements per 128-byte stage row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / ksplit, split = blockIdx.x % ksplit;
  // Grouped rasterisation: group_m consecutive M tiles sweep all N tiles, so the A and B tiles a wave
  // touches stay in L2.
  const int m_tiles = (M + kBM - 1) / kBM;
  const int per_group = group_m * n_tiles;
  const int first_m = (tile / per_group) * group_m;
  const int gsize = min(m_tiles - first_m, group_m);
  const int m_tile = first_m + (tile % per_group) % gsize;
  const int n_tile = (tile % per_group) / gsize;
  const int kblocks = (K + kBKe - 1) / kBKe;
  const int kb0 = static_cast<int>(static_cast<int64_t>(split) * kblocks / ksplit);
  const int kb1 = static_cast<int>(static_cast<int64_t>(split + 1) * kblocks / ksplit);
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    if (!a_tiled) tma_prefetch_desc(&tmA);
    if (!b_tiled) tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (trigger_early) griddep_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      // Decode (transposed epilogues): A is the weight matrix, streamed exactly once.
      const bool a_streamed = EPI == kEpiStoreF32T || EPI == kEpiStoreBF16T || EPI == kEpiSwiGLUT;
      const uint64_t pol_a = a_streamed ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      // The weight operand (A for the transposed decode epilogues, B otherwise) does not depend on the
      // previous kernel: its first stages are requested before waiting for that kernel to finish.
      // Operands stored pre-tiled (the layer's weights) arrive as contiguous 16 KB blocks, each already
      // in the 128B-swizzled shared-memory layout of a 128-row x 64 tile, by 1D bulk copies; the others
      // through their tensor maps.
      const int kbt = kblocks;
      auto load_a = [&](int s, int kb) {
        if (a_tiled)
          bulk_load_hint(sA + s * C::kABytes, a_tiled + (static_cast<int64_t>(m_tile) * kbt + kb) * 16384, 16384,
                         &full[s], pol_a);
        else
          tma_load_2d(sA + s * C::kABytes, &tmA, &full[s], kb * kBKe, m_tile * kBM, pol_a);
      };
      auto load_b = [&](int s, int kb) {
        if (b_tiled) {
#pragma unroll
          for (int q = 0; q < BN / 128; ++q)
            bulk_load_hint(sB + s * C::kBBytes + q * 16384,
                           b_tiled + (static_cast<int64_t>(n_tile * (BN / 128) + q) * kbt + kb) * 16384, 16384,
                           &full[s], pol_b);
        } else {
          tma_load_2d(sB + s * C::kBBytes, &tmB, &full[s], kb * kBKe, n_tile * BN, pol_b);
        }
      };
      const int pre = nk < STAGES ? nk : STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::kStageBytes);
        if (a_streamed) load_a(i, kb0 + i);
        else load_b(i, kb0 + i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) {
        if (a_streamed) load_b(i, kb0 + i);
        else load_a(i, kb0 + i);
      }
      for (int i = pre; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, kErrWaitSmemEmpty)) break;
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        load_a(s, kb0 + i);
        load_b(s, kb0 + i);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_dense(F8 ? 0 : 1, kBM, BN);  // e4m3 x e4m3, or bf16 x bf16
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1, kErrWaitTmaFull)) break;
        tc_fence_after();
        const uint64_t da = sdesc_k_sw128(smem_u32(sA + s * C::kABytes));
        const uint64_t db = sdesc_k_sw128(smem_u32(sB + s * C::kBBytes));
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // 32 bytes of K per MMA (16 bf16 or 32 fp8) = +2 in the descriptor
          if constexpr (F8)
            umma_f8(tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
          else
            umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
    __syncwarp();
  }

  tn_epilogue<BN, EPI>(tmem, smem, ep, m_tile, n_tile, M, N, ksplit, split, warp, lane, accum);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// The epilogue of one 128 x BN tile (or of the tile's share after the split-K reduction); warps 2..5 own the
// accumulator's TMEM lane quarters; every warp takes part in the split-K cluster barriers.  `smem` (the idle
// stage ring) parks the partial tile of a split.
template <int BN, int EPI>
__device__ __forceinline__ void tn_epilogue(uint32_t tmem, uint8_t* smem, const GemmEpiArgs& ep, int m_tile, int n_tile,
                                            int M, int N, int ksplit, int split, int warp, int lane, uint64_t* accum) {
  const int q = warp & 3;          // TMEM lane quarter this warp may access
  const int r = q * 32 + lane;     // row inside the tile
  const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16);
  const bool epi_warp = warp >= 2 && warp < 6;
  GemmEpiArgs eo = ep;
  if (epi_warp) {
    griddep_wait();  // the epilogue writes buffers the previous kernel may still read
    if (ep.slot_epoch)
      eo.out = static_cast<char*>(ep.out) + static_cast<int64_t>((*ep.slot_epoch + 1) & 1) * ep.slot_bytes;
    mbar_wait(accum, 0, kErrWaitAccum);
    tc_fence_after();
  }
  if (ksplit == 1) {
    if (epi_warp) {
      const int m = m_tile * kBM + r;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(t_row + c0, v);
        apply_scales(eo, m, n_tile * BN + c0, M, N, v);
        epilogue16<EPI>(eo, m, n_tile * BN + c0, M, N, v);
      }
    }
  } else {
    // Split-K over the cluster: every slice parks its fp32 partial tile in its own (now idle) stage ring,
    // then slice s sums 16-column chunks s, s + ksplit, ... over all slices through distributed shared
    // memory and runs the epilogue for them, so the reduction and the epilogue are spread over the cluster.
    float4* part = reinterpret_cast<float4*>(smem);
    if (epi_warp) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(t_row + c0, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          part[(c0 / 4 + i) * kBM + r] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
    __syncwarp();
    cluster_sync();
    if (epi_warp) {
      const int m = m_tile * kBM + r;
      const uint32_t part_addr = smem_u32(smem);
#pragma unroll 1
      for (int c0 = split * 16; c0 < BN; c0 += 16 * ksplit) {
        // slice by slice, in slice order (holding every slice's columns at once took ~130 more registers
        // per thread, 190 in all, which left the two-CTAs-per-SM launches one CTA per SM: two waves)
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
#pragma unroll 1
        for (int rank = 0; rank < ksplit; ++rank) {
          const uint32_t base = mapa_shared(part_addr, rank);
          float4 p4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) p4[i] = ld_dsmem_f4(base + static_cast<uint32_t>(((c0 / 4 + i) * kBM + r) * 16));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[4 * i] += p4[i].x;
            v[4 * i + 1] += p4[i].y;
            v[4 * i + 2] += p4[i].z;
            v[4 * i + 3] += p4[i].w;
          }
        }
        apply_scales(eo, m, n_tile * BN + c0, M, N, v);
        epilogue16<EPI>(eo, m, n_tile * BN + c0, M, N, v);
      }
    }
    __syncwarp();
    cluster_sync();  // every slice keeps its shared memory until all have read it
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, int ksplit, int n_tiles, int group_m, int trigger_early, const uint8_t* a_tiled,
                   const uint8_t* b_tiled, GemmEpiArgs ep) {
  gemm_tn_body<BN, STAGES, EPI, false>(tmA, tmB, M, N, K, ksplit, n_tiles, group_m, trigger_early, a_tiled, b_tiled,
                                       ep);
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_f8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                      int N, int K, int ksplit, int n_tiles, int group_m, int trigger_early, const uint8_t* a_tiled,
                      const uint8_t* b_tiled, GemmEpiArgs ep) {
  gemm_tn_body<BN, STAGES, EPI, true>(tmA, tmB, M, N, K, ksplit, n_tiles, group_m, trigger_early, a_tiled, b_tiled,
                                      ep);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major bf16 matrix [rows, cols] with row stride ld, tiles of 64 (K) x box_rows, 128B swizzle.
static cudaError_t make_tmap(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                             int box_rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((ld * 2) & 15) || rows <= 0 || cols <= 0 || ld < cols)
    return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// How many clusters of `ks` CTAs of this kernel can be resident at once (the unit a split-K launch is
// scheduled in: a cluster must fit inside one GPC, so CTA-level occupancy overestimates it).
template <class Kern>
static int cluster_capacity(Kern kern, int ks, int smem, int threads = kGemmThreads) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ks * 64));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    int blocks = 0, dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, threads, smem);
    n = std::max(1, blocks * sms / ks);
  }
  return n;
}

// Split-K factor that minimises (waves of clusters) x (k-blocks per slice), from the real cluster
// occupancy; ties go to the smaller split.
template <class Kern>
static int choose_ksplit(Kern kern, int smem, int tiles, int kblocks, int (&cap)[9]) {
  int best = 1;
  double best_cost = 1e30;
  for (int ks = 1; ks <= 8 && ks <= kblocks; ++ks) {
    if (!cap[ks]) cap[ks] = cluster_capacity(kern, ks, smem);
    const double waves = static_cast<double>((tiles + cap[ks] - 1) / cap[ks]);
    const double cost = waves * ((kblocks + ks - 1) / ks) + (ks > 1 ? 2.0 : 0.0);  // + reduction overhead
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = ks;
    }
  }
  return best;
}

// Weight-streaming GEMMs: the largest split in [1, kmax] whose clusters all fit on the device at once (one
// wave), else 1.
template <class Kern>
static int one_wave_ksplit(Kern kern, int smem, int tiles, int kmax, int (&cap)[9], int threads = kGemmThreads) {
  for (int ks = std::min(kmax, 8); ks > 1; --ks) {
    if (!cap[ks]) cap[ks] = cluster_capacity(kern, ks, smem, threads);
    if (tiles <= cap[ks]) return ks;
  }
  return 1;
}

template <int BN, int STAGES, int EPI, bool F8 = false>
static cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, int ksplit,
                               const GemmEpiArgs& ep, bool pdl, bool trigger, cudaStream_t stream) {
  using C = GemmCfg<BN, STAGES>;
  auto kern = [] {
    if constexpr (F8) return gemm_tn_f8_kernel<BN, STAGES, EPI>;
    else return gemm_tn_kernel<BN, STAGES, EPI>;
  }();
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int m_tiles = (M + kBM - 1) / kBM;
  const int n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int kblocks = (K + (F8 ? 2 * kBK : kBK) - 1) / (F8 ? 2 * kBK : kBK);
  static int cap[9] = {0};  // clusters of each size this instantiation fits on the device, filled on first use
  if (ksplit == 0) ksplit = choose_ksplit(kern, C::kSmemBytes, tiles, kblocks, cap);
  if (ksplit < 0) ksplit = one_wave_ksplit(kern, C::kSmemBytes, tiles, std::min(-ksplit, kblocks), cap);
  ksplit = std::max(1, std::min(ksplit, std::min(8, kblocks)));
  const int group_m = std::min(16, m_tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles * ksplit));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(ksplit);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, M, N, K, ksplit, n_tiles, group_m, trigger ? 1 : 0,
                            static_cast<const uint8_t*>(ep.a_tiled), static_cast<const uint8_t*>(ep.b_tiled), ep);
}

template <int BN, int STAGES>
static cudaError_t dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                                int ksplit, const GemmEpiArgs& ep, bool pdl, bool trigger, cudaStream_t s) {
  switch (epi) {
    case kEpiStoreF32: return launch_gemm<BN, STAGES, kEpiStoreF32>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    case kEpiStoreBF16: return launch_gemm<BN, STAGES, kEpiStoreBF16>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    case kEpiStoreF32T: return launch_gemm<BN, STAGES, kEpiStoreF32T>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    case kEpiStoreBF16T: return launch_gemm<BN, STAGES, kEpiStoreBF16T>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    case kEpiSwiGLUT: return launch_gemm<BN, STAGES, kEpiSwiGLUT>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_bf16_tn(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, int epi,
                         const GemmEpiArgs& ep, int ksplit, cudaStream_t stream, bool pdl, bool trigger) {
  if (M <= 0 || N <= 0 || K <= 0 || (K & 7)) return cudaErrorInvalidValue;
  if (epi == kEpiSwiGLUT && (M & 1)) return cudaErrorInvalidValue;
  if (ep.residual && (epi != kEpiStoreBF16T || ep.res_ld < M)) return cudaErrorInvalidValue;
  int BN;
  if (N <= 16) BN = 16;
  else if (N <= 32) BN = 32;
  else if (N <= 64) BN = 64;
  else if (N <= 128) BN = 128;
  else BN = 256;
  if (ep.b_tiled && BN < 128) BN = 128;  // a tiled B operand comes in whole 128-row blocks
  // Weight-streaming (decode) GEMMs start from N tiles of at most 64 tokens (the tiles of a wide batch read
  // the same weight blocks at about the same time: one HBM read, the rest L2 hits); batches wider than 64
  // tokens may take 128- or 256-token tiles below.
  if (ep.a_tiled && BN > 64) BN = 64;
  if ((ep.a_tiled && A != ep.a_tiled) || (ep.b_tiled && B != ep.b_tiled)) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  std::memset(&ta, 0, sizeof(ta));
  std::memset(&tb, 0, sizeof(tb));
  cudaError_t e = cudaSuccess;
  if (!ep.a_tiled && (e = make_tmap(&ta, A, M, K, lda, kBM)) != cudaSuccess) return e;
  if (!ep.b_tiled && (e = make_tmap(&tb, B, N, K, ldb, BN)) != cudaSuccess) return e;
  // GEMMs whose A operand is a pre-tiled weight matrix (the decode projections) stream that matrix from
  // HBM with ~190 KB in flight per SM and split-K only as far as the whole launch stays one wave, so no CTA
  // waits for another to finish before it starts streaming: one CTA per SM with an 8-stage ring, or, for
  // launches of more tiles than SMs (wide tensor-parallel batches), two CTAs per SM with 4-stage rings.
  // (Two 4-stage CTAs per SM with a deeper split measured slower than one 8-stage CTA for in_proj.)
  // Other skinny tiles use a 3-stage ring (< 75 KB) so three CTAs share an SM; wide tiles take the SM.
  if (ep.a_tiled) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (N > 64 && ksplit <= 0) {
      // Wide batches (tensor-parallel decode: 64 sequences per GPU, so 128 .. 512 token columns): every CTA
      // streams its K range of one weight tile and of BN token rows, so per-CTA bytes ~ K / ksplit * (128 +
      // BN).  Wider token tiles mean fewer tiles, hence a deeper split inside one wave, hence fewer bytes per
      // CTA; but a split's fp32 partial tile (128 x BN x 4 bytes, (ksplit - 1) / ksplit of it crossing to
      // other CTAs) is reduced through distributed shared memory, which measured about 8 times slower per
      // byte than streaming operands.  Pick the BN in {64, 128, 256} that minimises the sum per SM (64 keeps
      // its two-CTAs-per-SM path for more tiles than SMs, where the two CTAs share the SM: at 128 tokens and
      // one GPU, 194 such tiles ran a layer step in 159 us, 97 tiles of 128 tokens in 135 us).
      const int m_tiles = (M + kBM - 1) / kBM, kblocks = (K + kBK - 1) / kBK;
      int best_bn = 64;
      double best = 1e30;
      for (int bn : {64, 128, 256}) {
        const int t = m_tiles * ((N + bn - 1) / bn);
        int ks, per_sm = 1;  // CTAs sharing an SM's bandwidth
        if (bn == 64 && t > sms) {
          ks = std::max(1, std::min(8, 2 * sms / t));
          per_sm = 2;
        } else if (bn == 64 || t <= sms) {
          ks = std::max(1, std::min(8, sms / t));
        } else {
          continue;
        }
        const double cost = per_sm * (static_cast<double>((kblocks + ks - 1) / ks) * (kBM + bn) +
                                      8.0 * 4.0 * bn * (ks - 1) / ks);  // operand rows of 128 B + the reduction
        if (cost < best - 1e-9) {
          best = cost;
          best_bn = bn;
        }
      }
      if (best_bn > 64) {
        const int t = m_tiles * ((N + best_bn - 1) / best_bn);
        const int ks = -std::max(1, std::min(8, sms / t));  // < 0: largest split that stays one wave
        if ((e = make_tmap(&tb, B, N, K, ldb, best_bn)) != cudaSuccess) return e;
        if (best_bn == 128) return dispatch_epi<128, 6>(epi, ta, tb, M, N, K, ks, ep, pdl, trigger, stream);
        return dispatch_epi<256, 4>(epi, ta, tb, M, N, K, ks, ep, pdl, trigger, stream);
      }
    }
    const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
    const int k1 = sms / tiles;
    const bool two_per_sm = ksplit <= 0 && k1 == 0;
    if (ksplit <= 0) ksplit = -std::max(1, std::min(8, two_per_sm ? 2 * sms / tiles : k1));  // < 0: one wave
    if (two_per_sm) {
      switch (BN) {  // rings of 4 stages, up to 4 x 24 KB
        case 16: return dispatch_epi<16, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
        case 32: return dispatch_epi<32, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
        default: return dispatch_epi<64, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
      }
    }
    switch (BN) {  // rings of 8 stages, up to 8 x 24 KB
      case 16: return dispatch_epi<16, 8>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
      case 32: return dispatch_epi<32, 8>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
      default: return dispatch_epi<64, 8>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    }
  }
  switch (BN) {
    case 16: return dispatch_epi<16, 3>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    case 32: return dispatch_epi<32, 3>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    case 64: return dispatch_epi<64, 3>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    case 128: return dispatch_epi<128, 6>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    default: return dispatch_epi<256, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
  }
}

// ---------------------------------------------------------------------------------------------
// fp8 (e4m3) decode projections
// ---------------------------------------------------------------------------------------------

// Row-major e4m3 matrix [rows, cols] (one byte per element, row stride ld bytes), tiles of 128 (K) x
// box_rows, 128B swizzle: the same shared-memory image per 128-byte row as the bf16 maps.
static cudaError_t make_tmap_u8(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                                int box_rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld & 15) || rows <= 0 || cols <= 0 || ld < cols)
    return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(2 * kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int BN, int STAGES>
static cudaError_t dispatch_epi_f8(int epi, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                                   int ksplit, const GemmEpiArgs& ep, bool pdl, bool trigger, cudaStream_t s) {
  switch (epi) {
    case kEpiStoreBF16T: return launch_gemm<BN, STAGES, kEpiStoreBF16T, true>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    case kEpiStoreF32T:
      return launch_gemm<BN, STAGES, kEpiStoreF32T, true>(ta, tb, M, N, K, ksplit, ep, pdl, trigger, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_f8_tn(const void* A_tiled, const void* B, int64_t ldb, int M, int N, int K, int epi,
                       const GemmEpiArgs& ep, cudaStream_t stream, bool pdl, bool trigger) {
  if (M <= 0 || N <= 0 || K <= 0 || (K % (2 * kBK)) || !A_tiled || ep.a_tiled != A_tiled || !ep.row_scale ||
      !ep.col_scale || ep.b_tiled)
    return cudaErrorInvalidValue;
  const int BN = N <= 16 ? 16 : (N <= 32 ? 32 : 64);
  CUtensorMap ta, tb;
  std::memset(&ta, 0, sizeof(ta));
  std::memset(&tb, 0, sizeof(tb));
  cudaError_t e = make_tmap_u8(&tb, B, N, K, ldb, BN);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int k1 = sms / tiles;
  const bool two_per_sm = k1 == 0;
  const int ksplit = -std::max(1, std::min(8, two_per_sm ? 2 * sms / tiles : k1));  // < 0: one wave
  if (two_per_sm) {
    switch (BN) {
      case 16: return dispatch_epi_f8<16, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
      case 32: return dispatch_epi_f8<32, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
      default: return dispatch_epi_f8<64, 4>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    }
  }
  switch (BN) {
    case 16: return dispatch_epi_f8<16, 8>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    case 32: return dispatch_epi_f8<32, 8>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
    default: return dispatch_epi_f8<64, 8>(epi, ta, tb, M, N, K, ksplit, ep, pdl, trigger, stream);
  }
}

// ---------------------------------------------------------------------------------------------
// Weight-only fp8 decode projections: e4m3 weights x bf16 activations
// ---------------------------------------------------------------------------------------------
// The weights stream as e4m3 (half the bytes of bf16) in the fp8 streaming layout (16 KB blocks of 128
// rows x 128 K, 128B swizzle); the activations stay bf16.  The tensor cores take bf16 x bf16 (kind::f16
// wants both operands of one type), so each weight stage is widened to bf16 in shared memory first -- by
// the epilogue warps, idle until the accumulator is ready -- into one of two 32 KB buffers (two 128 x 64
// SW128 tiles), exactly (every e4m3 value is a bf16 value); the per-row power-of-two scale is applied in the
// epilogue.  Pipeline per 128-K block i: warp 0 loads stage i % S (e4m3 A + bf16 B); warps 2..5 wait for it
// and for conversion buffer i % 2 to be free, widen A into it and arrive; warp 1 issues the 8 MMAs and
// commits both the stage and the buffer back.
template <int BN, int STAGES, int NCONV = 2>
struct W8Cfg {
  static constexpr int kConv = NCONV;                 // bf16 widening buffers
  static constexpr int kABytes = 16384;             // e4m3 [128 rows][128 K]
  static constexpr int kBTile = BN * kBK * 2;       // bf16 [BN rows][64 K], SW128
  static constexpr int kStageBytes = kABytes + 2 * kBTile;
  static constexpr int kConvOff = STAGES * kStageBytes;
  static constexpr int kBarOffset = kConvOff + NCONV * 32768;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static_assert(kSmemBytes <= 227 * 1024, "weight-only fp8 GEMM shared memory");
  static_assert(BN * kBM * 4 <= STAGES * kStageBytes, "split-K partial tile must fit in the stage ring");
  static_assert(kStageBytes % 1024 == 0 && kBTile % 1024 == 0, "SW128 tiles need 1024-byte alignment");
};

// 16 e4m3 values (one 16-byte chunk) -> the 16 bf16 values e4m3 * 2^-120 (two 16-byte chunks), exactly, by
// placing the bits: e4m3 s.eeee.mmm -> bf16 s.0000eeee.mmm0000.  A normal e4m3 (eeee > 0) becomes the normal
// bf16 2^(eeee - 127) (1 + m/8) = value * 2^-120, an e4m3 subnormal (eeee = 0) the bf16 subnormal
// 2^-126 (m/8) = value * 2^-120, and zero stays zero; the quantiser never writes NaN.  Integer ALU work only
// (byte permute, shift, mask), where the conversion instructions through f16 and f32 took four per pair of
// values.  The epilogue multiplies the accumulator by 2^120 (GemmEpiArgs.acc_scale).
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2_scaled(uint32_t w, uint32_t sel) {
  uint32_t u;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(u) : "r"(w), "r"(sel));  // byte b_lo -> bits 8..15, b_hi -> 24..31
  return (u & 0x80008000u) | ((u >> 4) & 0x07F007F0u);            // sign stays; magnitude moves to bits 4..10
}
__device__ __forceinline__ void e4m3x16_to_bf16(const uint4& q, uint4& lo, uint4& hi) {
  lo = make_uint4(e4m3x2_to_bf16x2_scaled(q.x, 0x1504u), e4m3x2_to_bf16x2_scaled(q.x, 0x3524u),
                  e4m3x2_to_bf16x2_scaled(q.y, 0x1504u), e4m3x2_to_bf16x2_scaled(q.y, 0x3524u));
  hi = make_uint4(e4m3x2_to_bf16x2_scaled(q.z, 0x1504u), e4m3x2_to_bf16x2_scaled(q.z, 0x3524u),
                  e4m3x2_to_bf16x2_scaled(q.w, 0x1504u), e4m3x2_to_bf16x2_scaled(q.w, 0x3524u));
}

constexpr int kW8Threads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 widen the weights (2..5 then the epilogue)

template <int BN, int STAGES, int NCONV, int EPI>
__global__ void __launch_bounds__(kW8Threads, 1)
    gemm_tn_w8_kernel(const __grid_constant__ CUtensorMap tmB, int M, int N, int K, int ksplit, int n_tiles,
                      int group_m, int trigger_early, const uint8_t* a8, GemmEpiArgs ep) {
  using C = W8Cfg<BN, STAGES, NCONV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* conv = smem + C::kConvOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* cfull = empty + STAGES;
  uint64_t* cempty = cfull + C::kConv;
  uint64_t* accum = cempty + C::kConv;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  auto stage_a = [&](int st) { return smem + st * C::kStageBytes; };
  auto stage_b = [&](int st) { return smem + st * C::kStageBytes + C::kABytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / ksplit, split = blockIdx.x % ksplit;
  const int m_tiles = (M + kBM - 1) / kBM;
  const int per_group = group_m * n_tiles;
  const int first_m = (tile / per_group) * group_m;
  const int gsize = min(m_tiles - first_m, group_m);
  const int m_tile = first_m + (tile % per_group) % gsize;
  const int n_tile = (tile % per_group) / gsize;
  const int kblocks = K / (2 * kBK);
  const int kb0 = static_cast<int>(static_cast<int64_t>(split) * kblocks / ksplit);
  const int kb1 = static_cast<int>(static_cast<int64_t>(split + 1) * kblocks / ksplit);
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int c = 0; c < C::kConv; ++c) {
      mbar_init(&cfull[c], (kW8Threads - 64) / 32);  // one arrival per converter warp
      mbar_init(&cempty[c], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (trigger_early) griddep_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
      auto load_a = [&](int st, int kb) {
        bulk_load_hint(stage_a(st), a8 + (static_cast<int64_t>(m_tile) * kblocks + kb) * 16384, 16384, &full[st], pol_a);
      };
      auto load_b = [&](int st, int kb) {
        tma_load_2d(stage_b(st), &tmB, &full[st], kb * 2 * kBK, n_tile * BN, pol_b);
        tma_load_2d(stage_b(st) + C::kBTile, &tmB, &full[st], kb * 2 * kBK + kBK, n_tile * BN, pol_b);
      };
      // the weights do not depend on the previous kernel: the first stages are requested before waiting
      const int pre = nk < STAGES ? nk : STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::kStageBytes);
        load_a(i, kb0 + i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_b(i, kb0 + i);
      for (int i = pre; i < nk; ++i) {
        const int st = i % STAGES;
        if (!mbar_wait(&empty[st], ((i / STAGES) & 1) ^ 1, kErrWaitSmemEmpty)) break;
        mbar_arrive_expect_tx(&full[st], C::kStageBytes);
        load_a(st, kb0 + i);
        load_b(st, kb0 + i);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_dense(1, kBM, BN);
      for (int i = 0; i < nk; ++i) {
        const int st = i % STAGES, c = i % C::kConv;
        if (!mbar_wait(&cfull[c], (i / C::kConv) & 1, kErrWaitTmaFull)) break;
        if (!mbar_wait(&full[st], (i / STAGES) & 1, kErrWaitTmaFull)) break;
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint64_t da = sdesc_k_sw128(smem_u32(conv + c * 32768 + t * 16384));
          const uint64_t db = sdesc_k_sw128(smem_u32(stage_b(st) + t * C::kBTile));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || t > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[st]);
        umma_commit(&cempty[c]);
      }
      umma_commit(accum);
    }
    __syncwarp();
  } else {
    // Widen each e4m3 stage into a bf16 buffer.  Thread j handles 16-byte chunks j, j + 256, j + 512, j + 768:
    // chunk idx is row idx / 8, stored position idx % 8 = logical 16-wide K chunk kc ^ (row % 8), so the
    // row's swizzle phase -- and with it every address offset -- is the same for all four.  The two bf16
    // halves of a chunk go to tile kc / 4 at 8-wide positions 2 kc % 8 and + 1; lanes with kc < 4 store
    // their low half first and the others their high half, so the 8 lanes of each store phase hit 8
    // distinct 16-byte bank groups.
    const int ctid = threadIdx.x - 64;
    const int pos = ctid & 7, row0 = ctid >> 3, sw = row0 & 7;  // row0 + 32 j keeps row % 8 == sw
    const int kc = pos ^ sw, c8 = (2 * kc) & 7;
    const uint32_t off_first = (kc >> 2) * 16384 + ((((kc < 4) ? c8 : c8 + 1) ^ sw) << 4);
    const uint32_t off_second = (kc >> 2) * 16384 + ((((kc < 4) ? c8 + 1 : c8) ^ sw) << 4);
    for (int i = 0; i < nk; ++i) {
      const int st = i % STAGES, c = i % C::kConv;
      if (!mbar_wait(&full[st], (i / STAGES) & 1, kErrWaitTmaFull)) break;
      if (!mbar_wait(&cempty[c], ((i / C::kConv) & 1) ^ 1, kErrWaitSmemEmpty)) break;
      const uint8_t* a = stage_a(st) + row0 * 128 + pos * 16;
      uint8_t* d = conv + c * 32768 + row0 * 128;
      uint4 q[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = *reinterpret_cast<const uint4*>(a + j * 32 * 128);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 lo, hi;
        e4m3x16_to_bf16(q[j], lo, hi);
        *reinterpret_cast<uint4*>(d + j * 32 * 128 + off_first) = kc < 4 ? lo : hi;
        *reinterpret_cast<uint4*>(d + j * 32 * 128 + off_second) = kc < 4 ? hi : lo;
      }
      fence_proxy_async_shared();  // the widened tile is read by the tensor cores (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&cfull[c]);
    }
  }
  tn_epilogue<BN, EPI>(tmem, smem, ep, m_tile, n_tile, M, N, ksplit, split, warp, lane, accum);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

template <int BN, int STAGES, int NCONV, int EPI>
static cudaError_t launch_w8(const CUtensorMap& tb, const void* a8, int M, int N, int K, const GemmEpiArgs& ep,
                             bool pdl, bool trigger, cudaStream_t stream, int sms) {
  using C = W8Cfg<BN, STAGES, NCONV>;
  auto kern = gemm_tn_w8_kernel<BN, STAGES, NCONV, EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int m_tiles = (M + kBM - 1) / kBM, n_tiles = (N + BN - 1) / BN, tiles = m_tiles * n_tiles;
  const int kblocks = K / (2 * kBK);
  static int cap[9] = {0};
  int ksplit = one_wave_ksplit(kern, C::kSmemBytes, tiles, std::min(std::max(1, sms / tiles), kblocks), cap,
                               kW8Threads);
  const int group_m = std::min(16, m_tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles * ksplit));
  cfg.blockDim = dim3(kW8Threads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(ksplit);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kern, tb, M, N, K, ksplit, n_tiles, group_m, trigger ? 1 : 0,
                            static_cast<const uint8_t*>(a8), ep);
}

template <int BN, int STAGES, int NCONV>
static cudaError_t dispatch_w8(int epi, const CUtensorMap& tb, const void* a8, int M, int N, int K,
                               const GemmEpiArgs& ep, bool pdl, bool trigger, cudaStream_t s, int sms) {
  switch (epi) {
    case kEpiStoreBF16T: return launch_w8<BN, STAGES, NCONV, kEpiStoreBF16T>(tb, a8, M, N, K, ep, pdl, trigger, s, sms);
    case kEpiStoreF32T:
      return launch_w8<BN, STAGES, NCONV, kEpiStoreF32T>(tb, a8, M, N, K, ep, pdl, trigger, s, sms);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_w8_tn(const void* A8_tiled, const void* B, int64_t ldb, int M, int N, int K, int epi,
                       const GemmEpiArgs& ep, cudaStream_t stream, bool pdl, bool trigger) {
  if (M <= 0 || N <= 0 || K <= 0 || (K % (2 * kBK)) || !A8_tiled || !B || !ep.row_scale || ep.col_scale ||
      ep.b_tiled || (ep.residual && epi != kEpiStoreBF16T))
    return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int BN = N <= 16 ? 16 : (N <= 32 ? 32 : 64);
  if (BN == 64 && ((M + kBM - 1) / kBM) * ((N + 63) / 64) > sms) BN = 128;  // wide batches: one wave
  CUtensorMap tb;
  std::memset(&tb, 0, sizeof(tb));
  cudaError_t e = make_tmap(&tb, B, N, K, ldb, BN);
  if (e != cudaSuccess) return e;
  GemmEpiArgs ew = ep;
  ew.acc_scale = 0x1p120f;  // the widened weights are e4m3 * 2^-120
  switch (BN) {
    case 16: return dispatch_w8<16, 5, 2>(epi, tb, A8_tiled, M, N, K, ew, pdl, trigger, stream, sms);
    case 32: return dispatch_w8<32, 5, 2>(epi, tb, A8_tiled, M, N, K, ew, pdl, trigger, stream, sms);
    case 64: return dispatch_w8<64, 5, 2>(epi, tb, A8_tiled, M, N, K, ew, pdl, trigger, stream, sms);
    default: return dispatch_w8<128, 3, 2>(epi, tb, A8_tiled, M, N, K, ew, pdl, trigger, stream, sms);
  }
}

// The smallest power of two 2^e with amax / 2^e <= 448 (e4m3's largest finite value), from the bits of
// amax / 448: that value itself when it is a power of two, else the next power up; 1 for an all-zero row.
__device__ __forceinline__ float e4m3_scale(float amax) {
  if (!(amax > 0.f)) return 1.f;
  const uint32_t b = __float_as_uint(__fdiv_rn(amax, 448.f));
  const uint32_t ex = (b >> 23) & 0xffu;
  if (ex == 0u) return __uint_as_float(1u << 23);  // below the normal range: 2^-126
  return (b & 0x7fffffu) ? __uint_as_float((ex + 1u) << 23) : __uint_as_float(b);
}

// 8 floats (already divided by the scale, |v| <= 448) -> 8 e4m3 bytes (round to nearest even) and the
// dequantised values v8 * scale as 8 bf16.
__device__ __forceinline__ void e4m3_pack8(const float (&v)[8], float scale, uint2& q, uint4& deq) {
  uint32_t qw[2];
  uint32_t* dw = reinterpret_cast<uint32_t*>(&deq);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8x2_storage_t p = __nv_cvt_float2_to_fp8x2(make_float2(v[2 * i], v[2 * i + 1]), __NV_SATFINITE, __NV_E4M3);
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(p, __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const __nv_bfloat162 bb = __floats2bfloat162_rn(f.x * scale, f.y * scale);
    dw[i] = *reinterpret_cast<const uint32_t*>(&bb);
    if (i & 1) qw[i >> 1] |= static_cast<uint32_t>(p) << 16;
    else qw[i >> 1] = static_cast<uint32_t>(p);
  }
  q = make_uint2(qw[0], qw[1]);
}

__device__ __forceinline__ float amax8_bf16(const uint4& v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

__device__ __forceinline__ void unpack8_bf16(const uint4& v, float inv, float (&o)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x * inv;
    o[2 * i + 1] = f.y * inv;
  }
}

// One warp per (padded) weight row: lane l handles 16-byte chunk l % 8 of bf16 blocks kb = l / 8, + 4, ...
__global__ void quantize_tiled_weights_kernel(uint8_t* __restrict__ w16, int rows, int cols, int prow_total,
                                              uint8_t* __restrict__ w8, float* __restrict__ scale,
                                              const float* __restrict__ row_amax) {
  const int row = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= prow_total) return;
  const int mt = row / kBM, r = row % kBM, c = lane & 7;
  const int kbt16 = cols / kBK, kbt8 = cols / (2 * kBK);
  auto src = [&](int kb) {
    return w16 + (static_cast<int64_t>(mt) * kbt16 + kb) * 16384 + r * 128 + ((c ^ (r & 7)) << 4);
  };
  float amax = 0.f;
  for (int kb = lane >> 3; kb < kbt16; kb += 4) amax = fmaxf(amax, amax8_bf16(*reinterpret_cast<const uint4*>(src(kb))));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if (row_amax) amax = row < rows ? row_amax[row] : 0.f;  // the whole row's maximum (a column shard's rows)
  const float s = e4m3_scale(amax), inv = 1.f / s;
  if (lane == 0 && row < rows) scale[row] = s;
  for (int kb = lane >> 3; kb < kbt16; kb += 4) {
    uint4* p16 = reinterpret_cast<uint4*>(src(kb));
    float v[8];
    unpack8_bf16(*p16, inv, v);
    uint2 q;
    uint4 deq;
    e4m3_pack8(v, s, q, deq);
    *p16 = deq;
    const int k0 = kb * kBK + c * 8, kb8 = k0 / (2 * kBK), b = k0 % (2 * kBK);
    *reinterpret_cast<uint2*>(w8 + (static_cast<int64_t>(mt) * kbt8 + kb8) * 16384 + r * 128 +
                              (((b >> 4) ^ (r & 7)) << 4) + (b & 15)) = q;
  }
}

cudaError_t quantize_tiled_weights_fp8(void* w_tiled, int rows, int cols, void* w8, float* scale,
                                       cudaStream_t stream, const float* row_amax) {
  if (rows <= 0 || cols <= 0 || (cols % (2 * kBK)) || !w_tiled || !w8 || !scale) return cudaErrorInvalidValue;
  const int64_t prows = static_cast<int64_t>(tiled_weight_bytes(rows, cols) / 16384) / (cols / kBK) * kBM;
  count_launch();
  quantize_tiled_weights_kernel<<<static_cast<unsigned>((prows * 32 + 255) / 256), 256, 0, stream>>>(
      static_cast<uint8_t*>(w_tiled), rows, cols, static_cast<int>(prows), static_cast<uint8_t*>(w8), scale, row_amax);
  return cudaGetLastError();
}

// One warp per row of a row-major bf16 matrix: out[row] = max |src[row][:]|.
__global__ void row_amax_kernel(const uint16_t* __restrict__ src, int64_t ld, int rows, int cols, float* __restrict__ out) {
  const int row = static_cast<int>((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* r = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(row) * ld);
  float m = 0.f;
  for (int i = lane; i < cols / 8; i += 32) m = fmaxf(m, amax8_bf16(r[i]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) out[row] = m;
}

cudaError_t row_amax_bf16(const void* src, int64_t ld, int rows, int cols, float* out, cudaStream_t stream) {
  if (!src || !out || rows <= 0 || cols <= 0 || (cols & 7) || (ld & 7) || (reinterpret_cast<uintptr_t>(src) & 15))
    return cudaErrorInvalidValue;
  count_launch();
  row_amax_kernel<<<static_cast<unsigned>((static_cast<int64_t>(rows) * 32 + 255) / 256), 256, 0, stream>>>(
      static_cast<const uint16_t*>(src), ld, rows, cols, out);
  return cudaGetLastError();
}

// One CTA per activation row.  Programmatic dependent launch: the next kernel may start at once (it waits
// for this one before reading xq / xs); this one waits for the previous kernel before reading x.
__global__ void __launch_bounds__(256) quantize_rows_kernel(const uint16_t* __restrict__ x, int64_t ld, int cols,
                                                            uint8_t* __restrict__ xq, float* __restrict__ xs) {
  __shared__ float red[8];
  griddep_launch_dependents();
  griddep_wait();
  const int row = blockIdx.x, tid = threadIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ld);
  const int nc = cols / 8;
  float amax = 0.f;
  for (int i = tid; i < nc; i += 256) amax = fmaxf(amax, amax8_bf16(xr[i]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float s = e4m3_scale(amax), inv = 1.f / s;
  if (tid == 0) xs[row] = s;
  uint2* q8 = reinterpret_cast<uint2*>(xq + static_cast<int64_t>(row) * cols);
  for (int i = tid; i < nc; i += 256) {
    float v[8];
    unpack8_bf16(xr[i], inv, v);
    uint2 q;
    uint4 deq;
    e4m3_pack8(v, s, q, deq);
    q8[i] = q;
  }
}

cudaError_t quantize_rows_fp8(const void* x, int64_t ld, int rows, int cols, void* xq, float* xs,
                              cudaStream_t stream) {
  if (rows <= 0 || cols <= 0 || (cols % 16) || (ld % 8) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(xq) & 15) || !xs)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, quantize_rows_kernel, static_cast<const uint16_t*>(x), ld, cols,
                            static_cast<uint8_t*>(xq), xs);
}

// ---------------------------------------------------------------------------------------------
// Persistent 128 x 256 GEMM for the prefill projections
// ---------------------------------------------------------------------------------------------
// One CTA per SM walks the tiles blockIdx.x, + gridDim.x, ... in grouped raster order.  TMEM holds two
// 128 x 256 fp32 accumulators (all 512 columns): warp 1 issues the MMAs of the next tile into one while
// the epilogue warps drain the other, and warp 0 keeps the 4-stage ring full across tile boundaries.
// Eight epilogue warps (two per TMEM lane quarter, one per 128-column half) stage each 64-byte-wide
// column chunk of their half in shared memory (64B-swizzled) and write it with one TMA tensor store, so
// the output leaves as whole lines instead of 16-byte pieces of 128 different rows.
//
// kEpiPrefillInProj fuses the causal conv (K = 4) + SiLU of the conv channels into the epilogue.  Its
// M tiles advance by 125 rows and start 3 rows early, so every output row finds its 3 predecessors in
// the same tile (tile rows 0..2 are recomputed halo and never stored; 2.4% extra MMA work instead of a
// separate conv pass over HBM).  A row's predecessors sit in the 3 lanes below it (warp shuffles);
// lanes 0..2 of lane quarters 1..3 take them from the previous quarter's warp through shared memory.
// Predecessors before the start of a sequence come from conv_state (9B/kernels/layer_reader.cpp:103-124:
// the conv window continues the cached history); the raw last 3 inputs of each sequence go to conv_tail,
// from which conv_state_roll_tail() rolls the state after the kernel.  The conv taps of the tile's 256
// channels are staged in shared memory once per tile.
constexpr int kPBN = 256;
constexpr int kPStages = 4;
constexpr int kConvHalo = 3;
constexpr int kPEpiWarps = 8;
constexpr int kPThreads = 64 + 32 * kPEpiWarps;
using PCfg = GemmCfg<kPBN, kPStages>;
// Shared memory after the stage ring: barriers | output staging [2 halves][128 rows][64 B] |
// conv taps [256] float4 | conv exchange [2 halves][4 quarters][3 rows][16] floats.
constexpr int kPOutStage = PCfg::kBarOffset + 1024;
constexpr int kPConvW = kPOutStage + 2 * kBM * 64;
constexpr int kPXch = kPConvW + kPBN * 16;
constexpr int kPSmemBytes = kPXch + 2 * 4 * 48 * 4 + 1024;
static_assert(kPSmemBytes <= 227 * 1024, "persistent GEMM shared memory");
static_assert(kPOutStage % 1024 == 0, "64B-swizzled staging needs 512-byte alignment");

// Named barriers: id 1 + half over the 4 epilogue warps of one column half, id 3 (vote) and id 4 over all
// 8 epilogue warps; 0 is __syncthreads.
__device__ __forceinline__ void epi_half_sync(int half) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
}
__device__ __forceinline__ void epi_all_sync() { asm volatile("bar.sync 4, 256;" ::: "memory"); }
__device__ __forceinline__ bool epi_bar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 3, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void store_f32x16(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// Row `srow` of a 64-byte-wide staging tile with the TMA 64B swizzle (16-byte chunk c of row r at chunk
// c ^ ((r / 2) % 4)); four 16-byte chunks.
__device__ __forceinline__ void stage_row64(uint8_t* stage, int srow, const uint4 (&c)[4]) {
  uint8_t* row = stage + srow * 64;
  const int sw = (srow >> 1) & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(row + ((i ^ sw) << 4)) = c[i];
}

// Conv of one 16-column chunk (tile columns c0 .. c0 + 15, all conv channels) in place on v, for tile row
// r = 32 q + lane, output row `row` (valid when `store`).  Ends with the half's first barrier.
__device__ __forceinline__ void conv_chunk(const GemmEpiArgs& ep, float (&v)[16], int q, int half, int lane,
                                           int row, bool store, int n0, const float4* cw, float* xw,
                                           const float* xp) {
  if (lane >= 32 - kConvHalo) store_f32x16(xw + (lane - (32 - kConvHalo)) * 16, v);
  epi_half_sync(half);
  // h1/h2/h3 = inputs at t - 1, t - 2, t - 3.  Predecessor j of lane l < j is lane 32 - j + l of the
  // previous warp, i.e. exchange row 3 - j + l.
  float h1[16], h2[16], h3[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    h1[j] = __shfl_up_sync(0xffffffffu, v[j], 1);
    h2[j] = __shfl_up_sync(0xffffffffu, v[j], 2);
    h3[j] = __shfl_up_sync(0xffffffffu, v[j], 3);
  }
  if (q > 0 && lane < kConvHalo) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (lane < 1) h1[j] = xp[(2 + lane) * 16 + j];
      if (lane < 2) h2[j] = xp[(1 + lane) * 16 + j];
      h3[j] = xp[lane * 16 + j];
    }
  }
  if (!store) return;
  const int cr = ep.conv_rows, T = ep.seq_len;
  const int b = row / T, t = row - b * T;
  if (t < kConvHalo) {
    // Taps before the sequence start: conv_state row 3 + t - j holds the input at time t - j.
    const float* cs = ep.conv_state + static_cast<int64_t>(b) * 3 * cr + n0;
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      if (t < 1) {
        const float4 x = *reinterpret_cast<const float4*>(cs + static_cast<int64_t>(2 + t) * cr + j);
        h1[j] = x.x; h1[j + 1] = x.y; h1[j + 2] = x.z; h1[j + 3] = x.w;
      }
      if (t < 2) {
        const float4 x = *reinterpret_cast<const float4*>(cs + static_cast<int64_t>(1 + t) * cr + j);
        h2[j] = x.x; h2[j + 1] = x.y; h2[j + 2] = x.z; h2[j + 3] = x.w;
      }
      const float4 x = *reinterpret_cast<const float4*>(cs + static_cast<int64_t>(t) * cr + j);
      h3[j] = x.x; h3[j + 1] = x.y; h3[j + 2] = x.z; h3[j + 3] = x.w;
    }
  }
  if (t >= T - kConvHalo) store_f32x16(ep.conv_tail + (static_cast<int64_t>(b) * 3 + (t - T + 3)) * cr + n0, v);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float4 w = cw[j];
    v[j] = silu_fast(w.x * h3[j] + w.y * h2[j] + w.z * h1[j] + w.w * v[j]);
  }
}

template <int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmOut,
                           int M, int N, int K, int m_stride, int m_tiles, int n_tiles, int group_m,
                           const uint8_t* b_tiled, GemmEpiArgs ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kPStages * PCfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PCfg::kBarOffset);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int halo = kBM - m_stride;
  const int tiles = m_tiles * n_tiles;
  const int kblocks = (K + kBK - 1) / kBK;
  const int per_group = group_m * n_tiles;
  auto coords = [&](int t, int& mt, int& nt) {
    const int first_m = (t / per_group) * group_m;
    const int gsize = min(m_tiles - first_m, group_m);
    mt = first_m + (t % per_group) % gsize;
    nt = (t % per_group) / gsize;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kPEpiWarps);  // one arrival per epilogue warp
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kPBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      const uint64_t pol = policy_evict_last();
      auto load_a = [&](int s, int mt, int kb) {
        tma_load_2d(sA + s * PCfg::kABytes, &tmA, &full[s], kb * kBK, mt * m_stride - halo, pol);
      };
      auto load_b = [&](int s, int nt, int kb) {
#pragma unroll
        for (int h = 0; h < kPBN / 128; ++h)
          bulk_load_hint(sB + s * PCfg::kBBytes + h * 16384,
                         b_tiled + (static_cast<int64_t>(nt * (kPBN / 128) + h) * kblocks + kb) * 16384, 16384,
                         &full[s], pol);
      };
      // The weights do not depend on the previous kernel: the first stages of the first tile's B are
      // requested before waiting for it.
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < tiles) {
        int mt, nt;
        coords(blockIdx.x, mt, nt);
        pre = min(kblocks, kPStages);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], PCfg::kStageBytes);
          load_b(i, nt, i);
        }
      }
      griddep_wait();
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        int mt, nt;
        coords(t, mt, nt);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = static_cast<int>(it % kPStages);
          if (static_cast<int>(it) < pre) {
            load_a(s, mt, kb);
            continue;
          }
          if (!mbar_wait(&empty[s], ((it / kPStages) & 1) ^ 1, kErrWaitSmemEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], PCfg::kStageBytes);
          load_a(s, mt, kb);
          load_b(s, nt, kb);
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits.
        for (uint32_t j = it; j > 0 && j + kPStages > it; --j)
          mbar_wait(&full[(j - 1) % kPStages], ((j - 1) / kPStages) & 1, kErrWaitTmaFull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_dense(1, kBM, kPBN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++local) {
        const int a = local & 1;
        if (!mbar_wait(&acc_empty[a], ((local >> 1) & 1) ^ 1, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(a * kPBN);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = static_cast<int>(it % kPStages);
          if (!mbar_wait(&full[s], (it / kPStages) & 1, kErrWaitTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_k_sw128(smem_u32(sA + s * PCfg::kABytes));
          const uint64_t db = sdesc_k_sw128(smem_u32(sB + s * PCfg::kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[a]);
      }
    }
    __syncwarp();
  } else {
    griddep_wait();  // the epilogue writes buffers the previous kernel may still read
    constexpr bool kSwiGLU = EPI == kEpiSwiGLU;
    constexpr int kOutBytes = (EPI == kEpiStoreBF16 || kSwiGLU) ? 2 : 4;
    // accumulator columns per 64-byte staged output row: 16 (fp32), 32 (bf16), 64 (SwiGLU: gate/up pairs)
    constexpr int kChunk = kSwiGLU ? 64 : 64 / kOutBytes;
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;       // column half [128 half, +128) of each tile
    const int r = q * 32 + lane;
    const int etid = (warp - 2) * 32 + lane;
    const bool issuer = etid == half * 128;  // one thread per half issues the TMA stores
    const uint64_t out_policy = policy_evict_first();
    uint8_t* stage = smem + kPOutStage + half * kBM * 64;
    const float4* cw = reinterpret_cast<const float4*>(smem + kPConvW);
    float* xs = reinterpret_cast<float*>(smem + kPXch) + half * 4 * 48;
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int a = local & 1;
      const bool ok = mbar_wait(&acc_full[a], (local >> 1) & 1, kErrWaitAccum);
      if (epi_bar_any(!ok)) break;  // every epilogue warp leaves together
      tc_fence_after();
      int mt, nt;
      coords(t, mt, nt);
      const int row = mt * m_stride - halo + r;
      const bool store = r >= halo && row < M;
      if constexpr (EPI == kEpiPrefillInProj) {
        if (nt * kPBN < ep.conv_rows) {  // conv taps of the tile's channels
          const int c = nt * kPBN + etid;
          if (c < ep.conv_rows)
            reinterpret_cast<float4*>(smem + kPConvW)[etid] = __ldg(reinterpret_cast<const float4*>(ep.conv_w) + c);
          epi_all_sync();
        }
      }
      const uint32_t t_row = tmem + static_cast<uint32_t>(a * kPBN) + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int c0 = half * (kPBN / 2); c0 < (half + 1) * (kPBN / 2); c0 += kChunk) {
        float v[kChunk];
#pragma unroll
        for (int c16 = 0; c16 < kChunk / 16; ++c16)
          tmem_ld16(t_row + c0 + 16 * c16, *reinterpret_cast<float(*)[16]>(v + 16 * c16));
        const int n0 = nt * kPBN + c0;
        if (issuer) bulk_wait_read();  // the previous store has read the staging rows
        bool done = false;
        if constexpr (EPI == kEpiPrefillInProj) {
          if (n0 < ep.conv_rows) {
            conv_chunk(ep, *reinterpret_cast<float(*)[16]>(v), q, half, lane, row, store, n0, cw + c0, xs + q * 48,
                       xs + (q > 0 ? q - 1 : 0) * 48);
            done = true;
          }
        }
        if (!done) epi_half_sync(half);
        if (r >= halo) {
          uint4 c[4];
          if constexpr (kOutBytes == 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              c[i] = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]), __float_as_uint(v[4 * i + 2]),
                                __float_as_uint(v[4 * i + 3]));
          } else {
            float o[32];
            if constexpr (kSwiGLU) {
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = silu_fast(v[2 * i]) * v[2 * i + 1];
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = v[i];
              if (ep.residual && store) {  // bf16(acc + residual) of this row's 32 columns
                const uint4* rr = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(ep.residual) +
                                                                 static_cast<int64_t>(row) * ep.res_ld + n0);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const uint4 rv = rr[i];
                  const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float2 f = __bfloat1622float2(rh[j]);
                    o[8 * i + 2 * j] += f.x;
                    o[8 * i + 2 * j + 1] += f.y;
                  }
                }
              }
            }
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              __nv_bfloat162 h2 = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
              w[i] = *reinterpret_cast<uint32_t*>(&h2);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) c[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
          stage_row64(stage, r - halo, c);
        }
        fence_proxy_async_shared();
        epi_half_sync(half);
        if (issuer) {
          // the output streams past L2 (evict-first) so that the x row blocks and weight tiles of the
          // current raster group stay resident
          tma_store_2d_hint(&tmOut, stage, kSwiGLU ? n0 / 2 : n0, mt * m_stride, out_policy);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    if (issuer) bulk_wait_all();  // the stores have left shared memory and completed
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 2 * kPBN);
}

cudaError_t make_tmap_plain(void* map, const void* ptr, int elem_bytes, int64_t rows, int64_t cols, int64_t ld,
                            int box_cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((elem_bytes != 2 && elem_bytes != 4) || (reinterpret_cast<uintptr_t>(ptr) & 15) || ((ld * elem_bytes) & 15) ||
      rows <= 0 || cols <= 0 || ld < cols || (box_cols * elem_bytes) & 15 || box_cols <= 0 || box_cols > 256 ||
      box_rows <= 0 || box_rows > 256)
    return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t est[2] = {1, 1};
  CUresult r = fn(static_cast<CUtensorMap*>(map),
                  elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, est, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Output tensor map of the persistent GEMM: [rows, cols] with row stride ld elements, boxes of 64 bytes
// (box_cols elements) x box_rows rows, 64-byte swizzle.
static cudaError_t make_out_tmap(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols, int64_t ld, bool bf16,
                                 int box_cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const int es = bf16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((ld * es) & 15) || rows <= 0 || cols <= 0 || ld < cols ||
      box_cols * es != 64 || box_rows <= 0 || box_rows > 256)
    return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * es)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t est[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims,
                  strides, box, est, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int EPI>
static cudaError_t launch_persistent(const CUtensorMap& ta, const CUtensorMap& to, const void* b_tiled, int M,
                                     int N, int K, int m_stride, const GemmEpiArgs& ep, bool pdl,
                                     cudaStream_t stream) {
  auto kern = gemm_persistent_kernel<EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int m_tiles = (M + m_stride - 1) / m_stride;
  const int n_tiles = (N + kPBN - 1) / kPBN;
  const int tiles = m_tiles * n_tiles;
  const int group_m = std::min(16, m_tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min(tiles, sms)));
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  count_launch();
  return cudaLaunchKernelEx(&cfg, kern, ta, to, M, N, K, m_stride, m_tiles, n_tiles, group_m,
                            static_cast<const uint8_t*>(b_tiled), ep);
}

cudaError_t gemm_bf16_persistent(const void* A, int64_t lda, const void* B_tiled, int M, int N, int K, int epi,
                                 const GemmEpiArgs& ep, cudaStream_t stream, bool pdl) {
  if (M <= 0 || N <= 0 || K <= 0 || (K & 7) || !B_tiled || !ep.out) return cudaErrorInvalidValue;
  CUtensorMap ta, to;
  std::memset(&ta, 0, sizeof(ta));
  std::memset(&to, 0, sizeof(to));
  cudaError_t e = make_tmap(&ta, A, M, K, lda, kBM);
  if (e != cudaSuccess) return e;
  switch (epi) {
    case kEpiStoreF32:
      if ((e = make_out_tmap(&to, ep.out, M, N, ep.ld, false, 16, kBM)) != cudaSuccess) return e;
      return launch_persistent<kEpiStoreF32>(ta, to, B_tiled, M, N, K, kBM, ep, pdl, stream);
    case kEpiStoreBF16:
      if (ep.residual && (ep.res_ld < N || (ep.res_ld & 7) || (reinterpret_cast<uintptr_t>(ep.residual) & 15) || (N & 31)))
        return cudaErrorInvalidValue;
      if ((e = make_out_tmap(&to, ep.out, M, N, ep.ld, true, 32, kBM)) != cudaSuccess) return e;
      return launch_persistent<kEpiStoreBF16>(ta, to, B_tiled, M, N, K, kBM, ep, pdl, stream);
    case kEpiSwiGLU:
      if ((N & 1) || ep.residual) return cudaErrorInvalidValue;
      if ((e = make_out_tmap(&to, ep.out, M, N / 2, ep.ld, true, 32, kBM)) != cudaSuccess) return e;
      return launch_persistent<kEpiSwiGLU>(ta, to, B_tiled, M, N, K, kBM, ep, pdl, stream);
    case kEpiPrefillInProj:
      if (ep.seq_len <= 0 || ep.conv_rows <= 0 || (ep.conv_rows & 15) || ep.conv_rows > N || (ep.ld & 3) ||
          (M % ep.seq_len) || !ep.conv_w || !ep.conv_state || !ep.conv_tail ||
          (reinterpret_cast<uintptr_t>(ep.conv_state) & 15) || (reinterpret_cast<uintptr_t>(ep.conv_tail) & 15) ||
          (reinterpret_cast<uintptr_t>(ep.conv_w) & 15))
        return cudaErrorInvalidValue;
      if ((e = make_out_tmap(&to, ep.out, M, N, ep.ld, false, 16, kBM - kConvHalo)) != cudaSuccess) return e;
      return launch_persistent<kEpiPrefillInProj>(ta, to, B_tiled, M, N, K, kBM - kConvHalo, ep, pdl, stream);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------------------------
// Pre-tiled weights
// ---------------------------------------------------------------------------------------------
size_t tiled_weight_bytes(int rows, int cols) {
  const int64_t mt = ((rows + kBM - 1) / kBM + 1) & ~1;  // even number of 128-row blocks (pairs for BN = 256)
  return static_cast<size_t>(mt) * ((cols + kBK - 1) / kBK) * 16384;
}

// dst block (mt, kb) = rows [128 mt, +128) x cols [64 kb, +64) of src, in the K-major 128B-swizzled layout
// (row r at r * 128 bytes, 16-byte chunk c at chunk c ^ (r % 8)); rows past `rows` are zero.
__global__ void tile_weights_kernel(const uint16_t* __restrict__ src, int64_t ld, int rows, int cols,
                                    uint4* __restrict__ dst, int64_t nchunks) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nchunks) return;
  const int kbt = (cols + kBK - 1) / kBK;
  const int64_t blk = i >> 10;  // 1024 chunks of 16 B per 16 KB block
  const int w = static_cast<int>(i & 1023), r = w >> 3, cs = w & 7;
  const int mt = static_cast<int>(blk / kbt), kb = static_cast<int>(blk % kbt);
  const int row = mt * kBM + r, col = kb * kBK + ((cs ^ (r & 7)) << 3);
  uint4 v = make_uint4(0, 0, 0, 0);
  if (row < rows && col < cols) v = *reinterpret_cast<const uint4*>(src + static_cast<int64_t>(row) * ld + col);
  dst[i] = v;
}

cudaError_t tile_weights_bf16(const void* src, int64_t ld, int rows, int cols, void* dst, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0 || (cols & 7) || (ld & 7) || (reinterpret_cast<uintptr_t>(src) & 15)) return cudaErrorInvalidValue;
  const int64_t n = static_cast<int64_t>(tiled_weight_bytes(rows, cols) / 16);
  count_launch();
  tile_weights_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      static_cast<const uint16_t*>(src), ld, rows, cols, static_cast<uint4*>(dst), n);
  return cudaGetLastError();
}

}  // namespace gdn
