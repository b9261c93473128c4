// gemm_f32_tcgen05.cu - fp32 D[M][N] = A[M][K] * B (+ Cin) on sm_100a tensor
// cores with fp32-level accuracy.
//
// Replaces the reference's fp32 SIMT GEMM, matmulTiled
// (examples/matmul_bench.vc:22-54: one thread per output, 16x16 tiles of A
// and B through shared memory, fp32 multiply-add over K), whose bar is 1e-4
// relative error against an fp64 loop (matmul_bench.vc:109-125).
//
// Method (a three-term split product): every fp32 operand x is split into
// hi = x with its low 13 mantissa bits cleared (exactly a tf32 value) and
// lo = x - hi (exact in fp32, |lo| < 2^-10 |x|), and the tensor cores
// accumulate hi_a*hi_b + (lo_a*hi_b + hi_a*lo_b) in fp32:
//   * hi_a*hi_b with tcgen05.mma kind::tf32 straight from the raw fp32
//     tiles: kind::tf32 uses only sign, exponent and the top 10 mantissa
//     bits of each operand (measured: the raw tile in place of an explicit
//     hi leaves the error unchanged, where an MMA that rounded its inputs
//     would leave errors near 2^-11), so hi is never written;
//   * both correction terms with one kind::f16 MMA (bf16, K = 16) per 8-deep
//     K step over packed tiles that hold, per group of 8 K indices, [lo | hi]
//     of A against [hi ; lo] of B, rounded to bf16 (2^-9 relative): 2 MMAs
//     per 8-deep step instead of the 3 of an all-tf32 split, and the 16-bit
//     operands halve the tensor cores' shared-memory reads for them.
// Each correction term is below 2^-10 |a*b| and carries <= 2^-8 of itself,
// the dropped lo_a*lo_b is below 2^-20 |a*b|: <= ~2^-17 |a*b| per product,
// round-to-nearest (unbiased), against 2^-24 for an fp32 FMA; far inside the
// reference's 1e-4. Non-finite inputs give NaN outputs (an infinity meets a
// zero low part), where an fp32 FMA loop would give inf for an infinity.
//
// Design: CTA pairs (cluster of two, cta_group::2), 256 x 256 output tiles,
// one persistent cluster per SM pair, 704 threads per CTA:
//   warp 0       TMA producer (each CTA): per 32-deep K stage, this CTA's 128
//                rows of A (128 x 32 fp32 = 16 KiB) and its 128-column half
//                of the B panel (16 KiB), swizzled, 3-stage ring.
//   warps 6..21  split (each CTA): once a stage lands, write the packed bf16
//                hi/lo tiles beside it (128-byte swizzled, 128-bit shared
//                accesses laid out so every quarter warp hits 32 banks),
//                fence the writes to the tensor proxy, arrive on CTA 0's
//                split barrier.
//   warp 1       CTA 0 lane 0 issues, per 8-deep K step, a tf32 pair MMA and
//                a bf16 pair MMA (M = 256, N = 256) from both CTAs' shared
//                memory into TMEM (2 x 256-column accumulators, one per
//                512-deep K chunk, alternating); its commits free the stage
//                in both CTAs and hand each chunk to the epilogues.
//   warps 2..5   epilogue (each CTA): tcgen05.ld of its 128 accumulator rows,
//                32 x 32 swizzled boxes TMA-stored for the first K chunk
//                (with the optional Cin addend) and TMA reduce-added for the
//                rest.
// B stored [K][N] (the demos' layout) is an MN-major operand; for tf32 that
// takes the 128-byte swizzle with 32-byte atoms, in TMA and descriptor.
// Grids that would fill at most half the SM pairs (the demos' sizes) with
// K <= 1024 split K in two: both halves reduce-add onto a C zeroed on the
// stream first, two round-to-nearest adds onto zero per element, so the
// result does not depend on their order (1024^3: 43.2 -> 30.9 us).
// Shared memory per stage: A raw, B raw, A packed, B packed = 64 KiB; 3
// stages + 32 KiB of epilogue staging = 224 KiB. Ragged M, N, K: TMA
// zero-fills loads outside the matrix and clips stores. Roofline: per
// 2*M*N*K fp32 FLOP delivered, the tensor pipe runs 2*M*N*K tf32 and
// 2*2*M*N*K bf16 FLOP; dense tf32 runs at half the bf16 rate, so the
// tensor-pipe time equals that of 4*M*N*K tf32 FLOP ("tf32-equivalent").
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace vcb {
namespace {

constexpr int BM = 128;               // rows of A per CTA (256 per pair)
constexpr int BN = 256;               // output columns per pair tile
constexpr int BK = 32;                // 32 fp32 = one 128-byte swizzle row
constexpr int kStages = 3;
constexpr uint32_t kTileBytes = 128 * BK * 4;         // 16 KiB
constexpr uint32_t kRawBytes = 2 * kTileBytes;        // A, B as loaded
constexpr uint32_t kStageBytes = 2 * kRawBytes;       // + A lo, B lo
constexpr int kAccCols = BN;
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr int kEpiCols = 32;
constexpr uint32_t kEpiBytes = BM * kEpiCols * 4;
constexpr int kEpiThreads = 128;
constexpr int kSplitWarps = 16;
// Warps: 0 TMA, 1 MMA, 2..5 epilogue, then the split warps.
constexpr int kFirstSplitWarp = 6;
constexpr int kThreads = (kFirstSplitWarp + kSplitWarps) * 32;
constexpr int kSplitThreads = kSplitWarps * 32;
constexpr int kUnitsPerThread = kTileBytes / 32 / kSplitThreads;  // per operand, per stage
constexpr int kGroupRows = 8;
constexpr size_t kGroupAboveBBytes = 64ull << 20;
// The tensor cores' fp32 accumulation truncates: a running sum loses about
// 2^-24.5 of itself per MMA (measured: 6.5e-6 relative after K = 256 of
// same-sign data, growing with K). So each tile accumulates K in chunks of
// kChunkK in TMEM, and the epilogue adds the chunks into D with round-to-
// nearest reduce-adds (TMA bulk reduce), bounding the truncation to one
// chunk's worth. Measured at 4096^3 (all-tf32 split): chunks of 256 / 512 /
// 1024 ran at 178 / 188 / 194 TFLOP/s (each chunk's staging and reduce
// traffic shares shared memory with the mainloop); 512 keeps the same-sign
// error near 1e-5.
constexpr int kChunkK = 512;

struct __align__(8) F32Barriers {
  uint64_t full[kStages];    // each CTA: its own TMA bytes landed
  uint64_t split[kStages];   // CTA 0: both CTAs' split warps done
  uint64_t empty[kStages];   // each CTA: the MMAs reading the stage completed
  uint64_t acc_full[2];      // each CTA
  uint64_t acc_empty[2];     // CTA 0 (both epilogues arrive)
  uint32_t tmem_base;
};

constexpr size_t kSmemBytes =
    1024 + kStages * kStageBytes + 2 * kEpiBytes + sizeof(F32Barriers);
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kTileBytes % (32 * kSplitThreads) == 0, "split work divides evenly");

// hi = x with the low 13 mantissa bits cleared (the tf32 value the MMA
// reads), lo = x - hi (exact for finite x; NaN for non-finite x, whose
// outputs are NaN either way).
__device__ __forceinline__ void split_tf32(uint32_t x, float &hi, float &lo) {
  hi = __uint_as_float(x & 0xffffe000u);
  lo = __uint_as_float(x) - hi;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float first, float second) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(first, second);
  return *reinterpret_cast<const uint32_t *>(&v);
}

// 8 consecutive fp32 values (p0, p1) -> their hi and lo parts as 8 bf16
// each (round to nearest), in the same order.
__device__ __forceinline__ void split8_bf16(const uint4 &p0, const uint4 &p1, uint4 &hi,
                                            uint4 &lo) {
  const uint32_t x[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
  float h[8], l[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) split_tf32(x[e], h[e], l[e]);
  hi = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                  pack_bf16x2(h[6], h[7]));
  lo = make_uint4(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]), pack_bf16x2(l[4], l[5]),
                  pack_bf16x2(l[6], l[7]));
}

// Stage this warp's 32 x 32 box (128-byte swizzle, as the D map) and store
// it, or add it onto D (round to nearest) when `add` is set.
__device__ __forceinline__ void epilogue_store_box(const CUtensorMap *tmD, uint8_t *warp_stage,
                                                   uint32_t (&v)[32], int lane, uint32_t &count,
                                                   int x, int y, bool add) {
  const int buf = count & 1;
  if (lane == 0) bulk_wait_group_read<1>();
  __syncwarp();
  uint8_t *dst = warp_stage + buf * 4096 + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4 *>(dst + ((j ^ (lane & 7)) * 16)) =
        make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (add) tma_reduce_add_2d(tmD, warp_stage + buf * 4096, x, y);
    else tma_store_2d(tmD, warp_stage + buf * 4096, x, y);
    bulk_commit_group();
  }
  ++count;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_f32_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmD,
                     const float *__restrict__ Cin, int64_t ldc, int M, int N, int K,
                     uint32_t idesc_full, uint32_t idesc_half, uint32_t idesc16_full,
                     uint32_t idesc16_half, int b_kn, int num_full, int num_units,
                     int group_rows, int chunk_kblocks, int split_k) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stage_base = smem;
  uint8_t *epi_base = smem + kStages * kStageBytes;
  F32Barriers *bars = reinterpret_cast<F32Barriers *>(epi_base + 2 * kEpiBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_m = (M + 2 * BM - 1) / (2 * BM);
  const int kblocks = (K + BK - 1) / BK;
  // Unit -> tile as in the fp16 pair kernel: full 256 x 256 tiles, then the
  // tail wave's tiles as 256 x 128 halves; groups of `group_rows` pair rows
  // walked column by column. With split_k = 2 (grids that would fill at most
  // half the clusters), unit u is the K part u % 2 of tile u / 2 instead,
  // and [kb_begin, kb_end) its K blocks.
  auto unit_tile = [&](int u, int &tm, int &n0, int &width, int &kb_begin, int &kb_end) {
    int tile = u, half = 0, part = 0;
    width = BN;
    if (split_k > 1) {
      tile = u / split_k;
      part = u % split_k;
    } else if (u >= num_full) {
      tile = num_full + (u - num_full) / 2;
      half = (u - num_full) & 1;
      width = BN / 2;
    }
    const int per = (kblocks + split_k - 1) / split_k;
    kb_begin = part * per;
    kb_end = min(kblocks, kb_begin + per);
    const int group = tile / (group_rows * tiles_n);
    const int first_m = group * group_rows;
    const int rows = min(tiles_m - first_m, group_rows);
    const int in_group = tile - group * group_rows * tiles_n;
    tm = first_m + in_group % rows;
    n0 = (in_group / rows) * BN + half * (BN / 2);
  };
  auto lead = [&](uint64_t *b) { return mapa_shared(smem_u32(b), 0); };
  auto peer = [&](uint64_t *b) { return mapa_shared(smem_u32(b), 1); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->split[s], 2 * kSplitWarps);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 2 * kEpiThreads);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (each CTA, its own barriers)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int u = cluster; ok && u < num_units; u += num_clusters) {
        int tm, n0, width, kb_begin, kb_end;
        unit_tile(u, tm, n0, width, kb_begin, kb_end);
        const int a_row = tm * 2 * BM + rank * BM;
        const int b_col = n0 + rank * (width / 2);
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1u)) { ok = false; break; }
          uint8_t *sA = stage_base + stage * kStageBytes;
          uint8_t *sB = sA + kTileBytes;
          mbar_arrive_expect_tx(&bars->full[stage], kRawBytes);
          tma_load_2d(sA, &tmA, kb * BK, a_row, &bars->full[stage]);
          if (b_kn) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_2d(sB + j * (32 * BK * 4), &tmB, b_col + j * 32, kb * BK,
                          &bars->full[stage]);
          } else {
            tma_load_2d(sB, &tmB, kb * BK, b_col, &bars->full[stage]);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every issued copy lands before the CTA may exit.
      const uint32_t last = issued < (uint32_t)kStages ? issued : (uint32_t)kStages;
      for (uint32_t i = 0; i < last; ++i) {
        const uint32_t idx = issued - 1 - i;
        mbar_wait(&bars->full[idx % kStages], (idx / kStages) & 1u, 1000000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (CTA 0)
      // Descriptors (raw and packed A / B of stage 0) built once and advanced
      // by 32-bit adds to their address field (addresses below 256 KiB: no
      // carry): fewer instructions per MMA on the issuing thread.
      const uint32_t a_raw0 = smem_u32(stage_base);
      const uint32_t b_raw0 = a_raw0 + kTileBytes;
      const uint64_t d_ar = smem_desc_sw128(a_raw0, 16, 1024);
      const uint64_t d_br = b_kn ? smem_desc_sw128_atom32(b_raw0, BK * 128, 512)
                                 : smem_desc_sw128(b_raw0, 16, 1024);
      const uint64_t d_ap = smem_desc_sw128(a_raw0 + kRawBytes, 16, 1024);
      const uint64_t d_bp = b_kn ? smem_desc_sw128(b_raw0 + kRawBytes, 64 * 128, 1024)
                                 : smem_desc_sw128(b_raw0 + kRawBytes, 16, 1024);
      const uint32_t ar_lo = (uint32_t)d_ar, ar_hi = (uint32_t)(d_ar >> 32);
      const uint32_t br_lo = (uint32_t)d_br, br_hi = (uint32_t)(d_br >> 32);
      const uint32_t ap_lo = (uint32_t)d_ap, ap_hi = (uint32_t)(d_ap >> 32);
      const uint32_t bp_lo = (uint32_t)d_bp, bp_hi = (uint32_t)(d_bp >> 32);
      // Per 8-deep step g (descriptor address units of 16 bytes).
      const uint32_t br_step = b_kn ? 1024 >> 4 : 32 >> 4;
      const uint32_t bp_step = b_kn ? 2048 >> 4 : 32 >> 4;
      const uint32_t empty_lead = lead(&bars->empty[0]), empty_peer = peer(&bars->empty[0]);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      // One accumulator per (unit, K chunk), alternating between the two.
      for (int u = cluster; ok && u < num_units; u += num_clusters) {
       int tm, n0, width, kb_begin, kb_end_unit;
       unit_tile(u, tm, n0, width, kb_begin, kb_end_unit);
       for (int kb0 = kb_begin; ok && kb0 < kb_end_unit; kb0 += chunk_kblocks, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const uint32_t idesc = (u < num_full) ? idesc_full : idesc_half;
        const uint32_t idesc16 = (u < num_full) ? idesc16_full : idesc16_half;
        if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kAccCols;
        const int kb_end = min(kb_end_unit, kb0 + chunk_kblocks);
        for (int kb = kb0; kb < kb_end; ++kb) {
          // Cluster-scope acquire: the other CTA's split writes (fenced to
          // the tensor proxy before its release arrive) precede these MMAs.
          if (!mbar_wait_cluster(&bars->split[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t soff = (stage * kStageBytes) >> 4;
#pragma unroll
          for (int g = 0; g < BK / 8; ++g) {
            // hi*hi: tf32 from the raw tiles. K-major: 8 fp32 = 32 bytes per
            // step inside the swizzle row. MN-major B (32-byte-atom
            // swizzle): 8 K-rows = 1024 bytes per step, 4-row groups 512
            // bytes apart, 32-column blocks BK x 128 bytes apart.
            mma_tf32_ss_pair_lohi(d_tmem, ar_lo + soff + g * (32 >> 4), ar_hi,
                                  br_lo + soff + g * br_step, br_hi, idesc,
                                  (kb != kb0 || g != 0) ? 1u : 0u);
            // lo*hi + hi*lo: one bf16 MMA of K = 16 over the packed tiles.
            // K-major: 16 bf16 = 32 bytes per step. MN-major B: 16 K-rows =
            // 2048 bytes per step, 8-row groups 1024 apart, 64-column blocks
            // 64 x 128 bytes apart.
            mma_f16_ss_pair_lohi(d_tmem, ap_lo + soff + g * (32 >> 4), ap_hi,
                                 bp_lo + soff + g * bp_step, bp_hi, idesc16, 1u);
          }
          mma_commit_pair(empty_lead + stage * 8);
          mma_commit_pair(empty_peer + stage * 8);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(lead(&bars->acc_full[acc]));
        mma_commit_pair(peer(&bars->acc_full[acc]));
       }
      }
    }
  } else if (warp >= kFirstSplitWarp) {
    // ---------------- split warps (each CTA)
    const int t = threadIdx.x - kFirstSplitWarp * 32;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = cluster; ok && u < num_units; u += num_clusters) {
      int tm, n0, width, kb_begin, kb_end;
      unit_tile(u, tm, n0, width, kb_begin, kb_end);
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->full[stage], phase))) { ok = false; break; }
        const uint32_t a_raw = smem_u32(stage_base + stage * kStageBytes);
        const uint32_t b_raw = a_raw + kTileBytes;
        const uint32_t a_pk = a_raw + kRawBytes;
        const uint32_t b_pk = b_raw + kRawBytes;
        // Work unit: 8 consecutive fp32 of one row (32 bytes in, 2 x 16
        // bytes of bf16 out); 512 per operand per stage, 2 per thread. The
        // unit order makes each quarter warp touch 8 distinct 16-byte bank
        // groups on every access.
#pragma unroll
        for (int i = 0; i < kUnitsPerThread; ++i) {
          // A (K-major rows of 128 bytes): row r, 8-deep K group g = raw
          // 16-byte chunks 2g, 2g+1 (128-byte swizzle: chunk c of row r at
          // c ^ (r & 7)). Packed row: [lo(8) | hi(8)] per group.
          const int u = i * kSplitThreads + t;
          const int r = u >> 2, g = u & 3, sw = r & 7;
          const uint32_t c0 = r * 128 + ((2 * g) ^ sw) * 16, c1 = r * 128 + ((2 * g + 1) ^ sw) * 16;
          uint4 hi, lo;
          split8_bf16(lds128(a_raw + c0), lds128(a_raw + c1), hi, lo);
          sts128(a_pk + c0, lo);
          sts128(a_pk + c1, hi);
        }
#pragma unroll
        for (int i = 0; i < kUnitsPerThread; ++i) {
          const int u = i * kSplitThreads + t;
          uint4 hi, lo;
          if (b_kn) {
            // B stored [K][N]: raw 32-column blocks j of 32 K-rows x 128
            // bytes (32-byte chunk q of row k at q ^ (k & 3)). Packed: 64-
            // column blocks jb of 64 K'-rows x 128 bytes (16-byte chunk c of
            // row k' at c ^ (k' & 7)); for K group g, rows 16g..16g+7 hold
            // hi, rows 16g+8..16g+15 lo.
            const int q = u & 3, jodd = (u >> 2) & 1, k = (u >> 3) & 31, jb = u >> 8;
            const uint32_t src = b_raw + (2 * jb + jodd) * 4096 + k * 128 + ((q ^ (k & 3)) * 32);
            const uint32_t o0 = jodd * 16;  // odd blocks read their halves in swapped order
            const uint4 pa = lds128(src + o0), pb = lds128(src + (16 - o0));
            split8_bf16(jodd ? pb : pa, jodd ? pa : pb, hi, lo);
            const int kr = k & 7;
            const uint32_t dst = b_pk + jb * 8192 + (16 * (k >> 3) + kr) * 128 +
                                 (((jodd * 4 + q) ^ kr) * 16);
            sts128(dst, hi);
            sts128(dst + 8 * 128, lo);
          } else {
            // B stored [N][K]: as A, packed row [hi(8) | lo(8)] per group.
            const int r = u >> 2, g = u & 3, sw = r & 7;
            const uint32_t c0 = r * 128 + ((2 * g) ^ sw) * 16;
            const uint32_t c1 = r * 128 + ((2 * g + 1) ^ sw) * 16;
            split8_bf16(lds128(b_raw + c0), lds128(b_raw + c1), hi, lo);
            sts128(b_pk + c0, hi);
            sts128(b_pk + c1, lo);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(&bars->split[stage]);
          else mbar_arrive_cluster(lead(&bars->split[stage]));
        }
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue (each CTA): warps 2..5, thread = row
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    uint8_t *warp_stage = epi_base + quad * 8192;
    const uint32_t acc_empty_lead0 = lead(&bars->acc_empty[0]);
    const uint32_t acc_empty_lead1 = lead(&bars->acc_empty[1]);
    int local = 0;
    uint32_t box_count = 0;
    bool ok = true;
    for (int u = cluster; ok && u < num_units; u += num_clusters) {
      int tm, n0, width, kb_begin, kb_end;
      unit_tile(u, tm, n0, width, kb_begin, kb_end);
      const int m0 = tm * 2 * BM + rank * BM;
      const int gr = m0 + row;
      const int nboxes = width / kEpiCols;
      for (int kb0 = kb_begin; kb0 < kb_end; kb0 += chunk_kblocks, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&bars->acc_full[acc], acc_phase)) { ok = false; break; }
        tc_fence_after();
        const bool first = kb0 == kb_begin;
        // The first chunk of an unsplit tile is stored; every other chunk is
        // added onto C (a split tile's parts both add onto the C the host
        // zeroed). A later chunk adds onto what this warp wrote for the
        // earlier ones: those writes must have completed first.
        const bool store = first && split_k == 1;
        if (!first) {
          if (lane == 0) bulk_wait_group<0>();
          __syncwarp();
        }
        for (int c = 0; c < nboxes; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + acc * kAccCols + c * kEpiCols, v);
          tmem_ld_wait();
          if (c == nboxes - 1) {
            tc_fence_before();
            if (rank == 0) mbar_arrive(&bars->acc_empty[acc]);
            else mbar_arrive_cluster(acc ? acc_empty_lead1 : acc_empty_lead0);
          }
          const int cn0 = n0 + c * kEpiCols;
          if (cn0 >= N) continue;
          if (kb0 == 0 && Cin != nullptr && gr < M) {
            const float *crow = Cin + (int64_t)gr * ldc;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (cn0 + j < N) v[j] = __float_as_uint(__uint_as_float(v[j]) + crow[cn0 + j]);
          }
          epilogue_store_box(&tmD, warp_stage, v, lane, box_count, cn0, m0 + quad * 32, !store);
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

struct F32MapCache {
  GemmArgs key{};
  int device = -1;
  CUtensorMap a, b, d;
  bool valid = false;
};

bool same_key(const GemmArgs &x, const GemmArgs &y) {
  return x.A == y.A && x.B == y.B && x.D == y.D && x.M == y.M && x.N == y.N &&
         x.K == y.K && x.lda == y.lda && x.ldb == y.ldb && x.ldd == y.ldd &&
         x.b_kn == y.b_kn;
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int clusters_resident(int dev, int sms) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return sms / 2;
  if (cached[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms & ~1, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_f32_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;
    }
    cached[dev] = n < sms / 2 ? n : sms / 2;
  }
  return cached[dev];
}

}  // namespace

cudaError_t launch_gemm_f32_tcgen05(const GemmArgs &g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaErrorInvalidValue;
  if (!al16(g.A) || !al16(g.B) || !al16(g.D)) return cudaErrorNotSupported;
  if (g.lda % 4 || g.ldb % 4 || g.ldd % 4) return cudaErrorNotSupported;
  if (g.lda < g.K || g.ldd < g.N) return cudaErrorInvalidValue;
  if (g.b_kn ? g.ldb < g.N : g.ldb < g.K) return cudaErrorInvalidValue;
  if (g.Cin && g.ldc < g.N) return cudaErrorInvalidValue;

  static thread_local F32MapCache cache;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(cache.valid && cache.device == dev && same_key(cache.key, g))) {
    const CUtensorMapDataType f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    bool ok = make_map_2d(&cache.a, f32, 4, g.A, g.K, g.M, g.lda, BK, BM);
    if (g.b_kn)
      ok = ok && make_map_2d(&cache.b, f32, 4, g.B, g.N, g.K, g.ldb, 32, BK,
                             CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    else
      ok = ok && make_map_2d(&cache.b, f32, 4, g.B, g.K, g.N, g.ldb, BK, BN / 2);
    ok = ok && make_map_2d(&cache.d, f32, 4, g.D, g.N, g.M, g.ldd, kEpiCols, 32);
    if (!ok) {
      cache.valid = false;
      return cudaErrorNotSupported;
    }
    cache.key = g;
    cache.device = dev;
    cache.valid = true;
  }

  static uint64_t configured_device_mask = 0;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(configured_device_mask & (1ull << dev))) {
      cudaError_t e = cudaFuncSetAttribute(gemm_f32_pair_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemBytes);
      if (e != cudaSuccess) return e;
      if (dev < 64) configured_device_mask |= (1ull << dev);
    }
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms < 2) return cudaErrorNotSupported;
  const int pair_tiles = ((g.M + 2 * BM - 1) / (2 * BM)) * ((g.N + BN - 1) / BN);
  const int resident = clusters_resident(dev, sms);
  const int kblocks = (g.K + BK - 1) / BK;
  constexpr int kChunkBlocks = kChunkK / BK;
  // Split K in two when the tiles would fill at most half the clusters and
  // each half is at most one K chunk: both halves add onto a zeroed C, so
  // every element gets exactly two round-to-nearest adds onto zero and the
  // result does not depend on their order.
  // The split zeroes D before the kernel reads Cin, so it is taken only when
  // Cin does not share memory with D (an in-place D == Cin keeps split_k = 1,
  // where each element of Cin is read before the same element of D is stored).
  bool cin_overlaps_d = false;
  if (g.Cin) {
    const uintptr_t d0 = reinterpret_cast<uintptr_t>(g.D);
    const uintptr_t d1 = d0 + ((size_t)(g.M - 1) * (size_t)g.ldd + (size_t)g.N) * sizeof(float);
    const uintptr_t c0 = reinterpret_cast<uintptr_t>(g.Cin);
    const uintptr_t c1 = c0 + ((size_t)(g.M - 1) * (size_t)g.ldc + (size_t)g.N) * sizeof(float);
    cin_overlaps_d = c0 < d1 && d0 < c1;
  }
  const int split_k = (!cin_overlaps_d && 2 * pair_tiles <= resident && kblocks >= 2 &&
                       kblocks <= 2 * kChunkBlocks)
                          ? 2
                          : 1;
  int clusters, num_full, num_units;
  if (split_k == 2) {
    num_full = num_units = 2 * pair_tiles;
    clusters = num_units;
    cudaError_t e = cudaMemset2DAsync(g.D, (size_t)g.ldd * sizeof(float), 0,
                                      (size_t)g.N * sizeof(float), g.M, stream);
    if (e != cudaSuccess) return e;
  } else {
    clusters = pair_tiles < resident ? pair_tiles : resident;
    const int tail = pair_tiles % clusters;
    const bool split = tail > 0 && 2 * tail <= clusters;
    num_full = split ? pair_tiles - tail : pair_tiles;
    num_units = split ? num_full + 2 * tail : pair_tiles;
  }
  const uint32_t idesc_full = idesc_tf32_f32(2 * BM, BN, false, g.b_kn);
  const uint32_t idesc_half = idesc_tf32_f32(2 * BM, BN / 2, false, g.b_kn);
  const uint32_t idesc16_full = idesc_f16_f32(2 * BM, BN, true, false, g.b_kn);
  const uint32_t idesc16_half = idesc_f16_f32(2 * BM, BN / 2, true, false, g.b_kn);
  gemm_f32_pair_kernel<<<2 * clusters, kThreads, kSmemBytes, stream>>>(
      cache.a, cache.b, cache.d, g.Cin, g.ldc, g.M, g.N, g.K, idesc_full, idesc_half,
      idesc16_full, idesc16_half, g.b_kn ? 1 : 0, num_full, num_units,
      (size_t)g.K * (size_t)g.N * 4 > kGroupAboveBBytes ? kGroupRows : 1, kChunkBlocks, split_k);
  return cudaGetLastError();
}

}  // namespace vcb

VCB_DEFINE_ERROR_ACCESSOR(gemm_f32_error)
