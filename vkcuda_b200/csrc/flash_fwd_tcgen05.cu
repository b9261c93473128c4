// flash_fwd_tcgen05.cu - flash-attention forward on sm_100a tensor cores,
// fp16 or bf16 Q/K/V/O, fp32 scores, softmax statistics and accumulator.
//
// Computes, for each of BH independent [N][d] slices,
//   O = softmax_2(scale_log2 * Q K^T) V
// with base-2 exponentials, as the reference kernel flashAttn does
// (examples/flash_attn.vc:56-126: running max m, running sum l,
// alpha = exp2(m_old - m_new), p = exp2(s - m), O = acc / l), optionally
// causal (key j > query i masked, flash_attn.vc:100).
//
// Design, per CTA (one 128-row query tile of one slice; 2 CTAs per SM so one
// CTA's MMAs overlap the other's softmax):
//   TMEM (256 columns): S = Q K^T (128 x 128 fp32) in columns [0,128); the
//     probabilities P are written back as 16-bit pairs over S columns
//     [0,64); O (128 x d fp32) lives in columns [128, 128+d).
//   warp 4      TMA producer: Q once, then per key tile K and V (128 rows x
//               d, 128-byte swizzled 64-column boxes), one buffer each.
//   warp 5      allocates TMEM; lane 0 issues S = Q K^T (A and B from shared
//               memory, both K-major) and O += P V (A = P from TMEM, B = V
//               from shared memory, d-contiguous = MN-major).
//   warps 0..3  softmax, thread = query row: row max from S, conditional
//               rescale of O (only when a row max grows by more than 2^8,
//               which keeps p <= 256 and is exact after the final 1/l),
//               P = exp2(s * scale_log2 - m) packed to 16 bits into TMEM,
//               row sum l in fp32; at the end O / l is staged in shared
//               memory and stored with TMA.
// Causal tiles above the diagonal are skipped; keys >= N in the last tile
// and keys above the diagonal in the diagonal tile are masked.
// Roofline: 4*BH*N^2*d FLOP (half of that causal) against the dense tensor
// peak.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace vcb {
namespace {

constexpr int BQ = 128;    // query rows per CTA
constexpr int BKV = 128;   // keys per tile
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kSCol = 0;    // S / P columns
constexpr uint32_t kOCol = 128;  // O columns
constexpr uint32_t kBoxBytes = 128 * 128;  // 128 rows x 64 16-bit elements
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct __align__(8) FlashBarriers {
  uint64_t q_full;
  uint64_t k_full, k_empty;
  uint64_t v_full, v_empty;
  uint64_t s_full, p_full, o_full;
  uint32_t tmem_base;
};

template <int HD>
struct FlashSmem {
  static constexpr uint32_t kTileBytes = (HD / 64) * kBoxBytes;  // Q, K or V tile
  static constexpr uint32_t kQ = 0, kK = kTileBytes, kV = 2 * kTileBytes;
  static constexpr uint32_t kBars = 3 * kTileBytes;
  // Requested dynamic shared memory: the tiles, the barriers and alignment
  // slack, raised to ~100 KiB so at most two CTAs share an SM (their two
  // 256-column TMEM allocations fill the SM's 512 columns exactly).
  static constexpr size_t kUsed = 1024 + kBars + sizeof(FlashBarriers);
  static constexpr size_t kRequest = kUsed > 100 * 1024 ? kUsed : 100 * 1024;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  }
}

template <int HD, bool BF16>
__global__ void __launch_bounds__(kThreads, 2)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                 const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV,
                 const __grid_constant__ CUtensorMap tmO, int N, float scale_log2,
                 int causal) {
  using L = FlashSmem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sQ = smem + L::kQ;
  uint8_t *sK = smem + L::kK;
  uint8_t *sV = smem + L::kV;
  FlashBarriers *bars = reinterpret_cast<FlashBarriers *>(smem + L::kBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int num_qt = (N + BQ - 1) / BQ;
  const int qt = num_qt - 1 - blockIdx.y;  // heaviest causal tiles first
  const int kv_tiles_all = (N + BKV - 1) / BKV;
  const int nkv = causal ? min(qt + 1, kv_tiles_all) : kv_tiles_all;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->k_full, 1);
    mbar_init(&bars->k_empty, 1);
    mbar_init(&bars->v_full, 1);
    mbar_init(&bars->v_empty, 1);
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->p_full, kSoftmaxThreads);
    mbar_init(&bars->o_full, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 4) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&bars->q_full, L::kTileBytes);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_3d(sQ + c * kBoxBytes, &tmQ, c * 64, qt * BQ, bh, &bars->q_full);
      int k_loads = 0, v_loads = 0;
      for (int j = 0; j < nkv; ++j) {
        if (j > 0 && !mbar_wait(&bars->k_empty, (j - 1) & 1)) break;
        mbar_arrive_expect_tx(&bars->k_full, L::kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_3d(sK + c * kBoxBytes, &tmK, c * 64, j * BKV, bh, &bars->k_full);
        ++k_loads;
        if (j > 0 && !mbar_wait(&bars->v_empty, (j - 1) & 1)) break;
        mbar_arrive_expect_tx(&bars->v_full, L::kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_3d(sV + c * kBoxBytes, &tmV, c * 64, j * BKV, bh, &bars->v_full);
        ++v_loads;
      }
      // Drain the last loads before the CTA may exit (immediate unless a
      // wait gave up).
      mbar_wait(&bars->q_full, 0, 1000000000ull);
      if (k_loads) mbar_wait(&bars->k_full, (k_loads - 1) & 1, 1000000000ull);
      if (v_loads) mbar_wait(&bars->v_full, (v_loads - 1) & 1, 1000000000ull);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc_s = idesc_f16_f32(BQ, BKV, BF16, false, false);
      const uint32_t idesc_o = idesc_f16_f32(BQ, HD, BF16, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(&bars->q_full, 0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (!mbar_wait(&bars->k_full, j & 1)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t off = (ks / 4) * kBoxBytes + (ks % 4) * 32;
          mma_f16_ss(tmem + kSCol, smem_desc_sw128(q_addr + off, 16, 1024),
                     smem_desc_sw128(k_addr + off, 16, 1024), idesc_s, ks > 0 ? 1u : 0u);
        }
        mma_commit(&bars->k_empty);
        mma_commit(&bars->s_full);
        if (!mbar_wait(&bars->p_full, j & 1)) break;
        tc_fence_after();
        if (!mbar_wait(&bars->v_full, j & 1)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < BKV / 16; ++ks) {
          mma_f16_ts(tmem + kOCol, tmem + kSCol + ks * 8,
                     smem_desc_sw128(v_addr + ks * 16 * 128, kBoxBytes, 1024), idesc_o,
                     (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&bars->v_empty);
        mma_commit(&bars->o_full);
      }
    }
  } else {
    // -------------------------------------------------- softmax, warps 0..3
    const int row = warp * 32 + lane;  // == TMEM lane of this thread
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const int qi = qt * BQ + row;
    float m_run = -INFINITY;  // running max of scale_log2 * s
    float l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&bars->s_full, j & 1)) { ok = false; break; }
      tc_fence_after();
      const int key0 = j * BKV;
      const bool tail = (key0 + BKV > N);
      const bool diag = causal && (j == nkv - 1);
      const bool need_mask = tail || diag;
      // Pass 1: row max.
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t s[32];
        tmem_ld32(lane_base + kSCol + c * 32, s);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int key = key0 + c * 32 + t;
          const bool masked = need_mask && (key >= N || (causal && key > qi));
          const float v = masked ? -INFINITY : __uint_as_float(s[t]);
          mx = fmaxf(mx, v);
        }
      }
      const float m_cand = fmaxf(m_run, mx * scale_log2);
      const bool grow = m_cand > m_run + kRescaleThreshold;  // true on first tile
      if (__any_sync(0xffffffffu, grow)) {
        if (j > 0) {
          // O holds PV of earlier tiles: wait for the last one, then rescale
          // this warp's rows by exp2(m_run - m_cand).
          if (!mbar_wait(&bars->o_full, (j - 1) & 1)) { ok = false; }
          tc_fence_after();
          const float alpha = (m_run == -INFINITY) ? 0.0f : ex2_approx(m_run - m_cand);
          l_run *= alpha;
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_base + kOCol + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tmem_st32(lane_base + kOCol + c * 32, o);
          }
          tmem_st_wait();
        }
        m_run = m_cand;
      }
      const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
      // Pass 2: P = exp2(scale_log2 * s - m) -> 16-bit pairs over S columns.
      float lsum = 0.0f;
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t s[32];
        tmem_ld32(lane_base + kSCol + c * 32, s);
        tmem_ld_wait();
        uint32_t p[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int key = key0 + c * 32 + 2 * t;
          float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * t]), scale_log2, -m_use));
          float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * t + 1]), scale_log2, -m_use));
          if (need_mask) {
            if (key >= N || (causal && key > qi)) p0 = 0.0f;
            if (key + 1 >= N || (causal && key + 1 > qi)) p1 = 0.0f;
          }
          lsum += p0 + p1;
          p[t] = pack2<BF16>(p0, p1);
        }
        tmem_st16(lane_base + kSCol + c * 16, p);
      }
      l_run += lsum;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_full);
      if (!ok) break;
    }
    // Epilogue: O / l -> 16-bit, staged over the Q tile, TMA store.
    if (ok && mbar_wait(&bars->o_full, (nkv - 1) & 1)) {
      tc_fence_after();
      const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + kOCol + c * 32, o);
        tmem_ld_wait();
        // 32 fp32 -> 16 packed words = 64 bytes = chunks 4*(c%2) .. +3 of
        // the 128-byte row of box c/2.
        uint8_t *rowp = sQ + (c / 2) * kBoxBytes + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack2<BF16>(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
          w.y = pack2<BF16>(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
          w.z = pack2<BF16>(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
          w.w = pack2<BF16>(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
          const int chunk = (c % 2) * 4 + q;
          *reinterpret_cast<uint4 *>(rowp + ((chunk ^ (row & 7)) * 16)) = w;
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, kSoftmaxThreads);
      if (threadIdx.x == 0) {
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_store_3d(&tmO, sQ + c * kBoxBytes, c * 64, qt * BQ, bh);
        bulk_commit_group();
        bulk_wait_group<0>();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                  void *, const cuuint64_t *, const cuuint64_t *,
                                  const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool make_map_bhnd(CUtensorMap *map, bool bf16, const void *base, int BH, int N, int d) {
  auto encode = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!encode) return false;
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)N, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)N * d * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      3, const_cast<void *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int HD, bool BF16>
cudaError_t launch_typed(const FlashArgs &f, const CUtensorMap &q, const CUtensorMap &k,
                         const CUtensorMap &v, const CUtensorMap &o, cudaStream_t stream) {
  static int configured = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(configured & (1 << dev))) {
      cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<HD, BF16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)FlashSmem<HD>::kRequest);
      if (e != cudaSuccess) return e;
      configured |= (1 << dev);
    }
  }
  dim3 grid(f.BH, (f.N + BQ - 1) / BQ);
  flash_fwd_kernel<HD, BF16><<<grid, kThreads, FlashSmem<HD>::kRequest, stream>>>(
      q, k, v, o, f.N, f.scale_log2, f.causal ? 1 : 0);
  return cudaGetLastError();
}

struct FlashMapCache {
  const void *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
  int BH = 0, N = 0, d = 0, dtype = -1, device = -1;
  CUtensorMap mq, mk, mv, mo;
  bool valid = false;
};

}  // namespace

cudaError_t launch_flash_fwd_tcgen05(const FlashArgs &f, cudaStream_t stream) {
  if (f.dtype != 1 && f.dtype != 2) return cudaErrorInvalidValue;
  if (f.d != 64 && f.d != 128) return cudaErrorInvalidValue;
  if (f.BH <= 0 || f.N <= 0 || f.BH > 65535 * 32768) return cudaErrorInvalidValue;
  if ((f.N + BQ - 1) / BQ > 65535) return cudaErrorInvalidValue;
  for (const void *p : {f.Q, f.K, f.V, static_cast<const void *>(f.O)})
    if (reinterpret_cast<uintptr_t>(p) & 15u) return cudaErrorInvalidValue;
  const bool bf16 = (f.dtype == 2);
  static thread_local FlashMapCache cache;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(cache.valid && cache.q == f.Q && cache.k == f.K && cache.v == f.V && cache.o == f.O &&
        cache.BH == f.BH && cache.N == f.N && cache.d == f.d && cache.dtype == f.dtype &&
        cache.device == dev)) {
    bool ok = make_map_bhnd(&cache.mq, bf16, f.Q, f.BH, f.N, f.d) &&
              make_map_bhnd(&cache.mk, bf16, f.K, f.BH, f.N, f.d) &&
              make_map_bhnd(&cache.mv, bf16, f.V, f.BH, f.N, f.d) &&
              make_map_bhnd(&cache.mo, bf16, f.O, f.BH, f.N, f.d);
    if (!ok) {
      cache.valid = false;
      return cudaErrorInvalidValue;
    }
    cache.q = f.Q; cache.k = f.K; cache.v = f.V; cache.o = f.O;
    cache.BH = f.BH; cache.N = f.N; cache.d = f.d; cache.dtype = f.dtype;
    cache.device = dev;
    cache.valid = true;
  }
  if (f.d == 64)
    return bf16 ? launch_typed<64, true>(f, cache.mq, cache.mk, cache.mv, cache.mo, stream)
                : launch_typed<64, false>(f, cache.mq, cache.mk, cache.mv, cache.mo, stream);
  return bf16 ? launch_typed<128, true>(f, cache.mq, cache.mk, cache.mv, cache.mo, stream)
              : launch_typed<128, false>(f, cache.mq, cache.mk, cache.mv, cache.mo, stream);
}

}  // namespace vcb

VCB_DEFINE_ERROR_ACCESSOR(flash_tcgen05_error)
