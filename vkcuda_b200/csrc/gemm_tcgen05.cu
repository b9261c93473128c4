// gemm_tcgen05.cu - D[M][N] (fp32) = A[M][K] * B (+ Cin) on sm_100a tensor
// cores; fp16 or bf16 inputs, fp32 accumulation.
//
// Replaces the cooperative-matrix GEMMs of the reference demos:
// test/wmma_gemm.vc:19-33 (one 8x8x16 tile, D = A*B + C) and
// examples/matmul_coopmat_bench.vc:60-110 (16x16 tiles of 2x2 8x8x16 MMAs,
// accumulator streamed through global C every K step).
//
// Two kernels: gemm_tcgen05_pair_kernel (CTA pairs, cta_group::2, used when
// M > 128; described at its definition) and the single-CTA kernel below.
//
// Single-CTA design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile 128x64 and B tile 64x256 (or 256x64)
//               per stage, 128-byte swizzled, 4-stage ring (48 KiB/stage).
//   Work units are 128 x 256 output tiles; when the last partial wave would
//   fill at most half the SMs, its tiles are split into two 128 x 128 units
//   each so that the tail costs half a tile time (4096^3: 512 tiles over 148
//   SMs = 444 full units + 136 half units).
//   warp 1      allocates 512 TMEM columns; lane 0 issues tcgen05.mma
//               (M=128, N=256, K=16, fp32 accumulator in TMEM), commits each
//               stage back to the producer and each finished tile to the
//               epilogue. Two accumulators (2 x 256 columns) alternate, so
//               the MMAs of tile i+1 overlap the epilogue of tile i.
//   warps 2..5  epilogue: tcgen05.ld 32 columns per thread-row, optional
//               Cin addend; each warp stages its own 32 x 32 fp32 box in
//               shared memory (2 x 4 KiB per warp, 128-byte swizzle) and
//               TMA-stores it, with no barrier between the warps.
// Ragged M, N and K are handled by TMA: loads zero-fill outside the matrix
// and stores clip, so any shape whose row strides meet TMA's 16-byte rule
// runs here. Roofline: 2*M*N*K FLOP against the dense fp16/bf16 tensor peak.
//
// Measured (clock64 and global-timer traces of the pair kernel on B200): an
// N = 256 pair MMA takes 128 cycles of the tensor pipe, and the single
// issuing thread is what limits the mainloop: with descriptors rebuilt per
// MMA it spent ~150 cycles per MMA, and the tail's half units (half the MMA
// work) took as long as full units. Descriptors are now built once and
// advanced by 32-bit adds (~61 cycles per MMA issue), and each barrier stage
// holds two 64-deep K blocks, so one wait and one commit per CTA serve 8
// MMAs (a wait ~86 cycles, a commit ~54, measured), and the whole warp runs
// the issuing loop with elected MMAs: 4096^3 1242 -> 1368 TFLOP/s per
// launch. Stage count (4 / 5 / 6 blocks in flight) did not change the unit
// time; three blocks per stage in two stages was slower.
// The epilogue (~5K cycles per tile) is hidden by the second accumulator.
// The pair kernel is launched with programmatic stream
// serialization, so back-to-back GEMMs overlap the next launch and its set-up
// with the current one's last wave (400 back-to-back 4096^3 launches: 112.4
// -> 110.3 us each). With A in TMEM the MMA alone costs 138-140 cycles, but
// copying each K = 16 slice of A there (tcgen05.cp into 32 columns of the
// drained accumulator, then the TS form) made this kernel 25-35 % slower
// (4096^3: 776 vs 1197 TFLOP/s), so A stays in shared memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace vcb {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int kStages = 4;
constexpr int kAccCols = BN;
constexpr uint32_t kTmemCols = 2 * kAccCols;  // 512: two accumulators
constexpr int kEpiCols = 32;
constexpr uint32_t kABytes = BM * BK * 2;
constexpr uint32_t kBBytes = BN * BK * 2;
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kEpiBytes = BM * kEpiCols * 4;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;

struct __align__(8) GemmBarriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

// Epilogue store of one 32 x 32 fp32 box: this warp's 32 accumulator rows
// (one per lane) x 32 columns. Each warp owns two 4 KiB staging buffers and
// its own bulk-store groups, so the four epilogue warps never wait for each
// other. The box is written with the 128-byte swizzle the D tensor map uses.
__device__ __forceinline__ void epilogue_store_box(const CUtensorMap *tmD, uint8_t *warp_stage,
                                                   uint32_t (&v)[32], int lane, uint32_t &count,
                                                   int x, int y) {
  const int buf = count & 1;
  if (lane == 0) bulk_wait_group_read<1>();  // the store that last used `buf` has read it
  __syncwarp();
  uint8_t *box = warp_stage + buf * 4096;
  uint8_t *dst = box + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4 *>(dst + ((j ^ (lane & 7)) * 16)) =
        make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmD, box, x, y);
    bulk_commit_group();
  }
  ++count;
}

constexpr size_t kSmemBytes =
    1024 /* alignment slack */ + kStages * kStageBytes + 2 * kEpiBytes + sizeof(GemmBarriers);

__global__ void __launch_bounds__(kThreads, 1)
gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmD,
                    const float *__restrict__ Cin, int64_t ldc, int M, int N, int K,
                    uint32_t idesc_full, uint32_t idesc_half, int b_kn, int num_full,
                    int num_units) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stage_base = smem;
  uint8_t *epi_base = smem + kStages * kStageBytes;
  GemmBarriers *bars = reinterpret_cast<GemmBarriers *>(epi_base + 2 * kEpiBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_n = (N + BN - 1) / BN;
  const int kblocks = (K + BK - 1) / BK;
  // Work unit u: u < num_full is the full 128 x 256 tile u; later units are
  // the tail tiles split in two 128 x 128 halves (unit -> tile, half).
  auto unit_tile = [&](int u, int &tm, int &n0, int &width) {
    int tile = u, half = 0;
    width = BN;
    if (u >= num_full) {
      tile = num_full + (u - num_full) / 2;
      half = (u - num_full) & 1;
      width = BN / 2;
    }
    tm = tile / tiles_n;
    n0 = (tile % tiles_n) * BN + half * (BN / 2);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], kEpiThreads);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
        int tm, n0, width;
        unit_tile(u, tm, n0, width);
        // The whole 256-wide B panel from n0 is loaded for half units too
        // (the MMA uses its first 128 columns): one transaction size.
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1u)) { ok = false; break; }
          uint8_t *sA = stage_base + stage * kStageBytes;
          uint8_t *sB = sA + kABytes;
          mbar_arrive_expect_tx(&bars->full[stage], kStageBytes);
          tma_load_2d(sA, &tmA, kb * BK, tm * BM, &bars->full[stage]);
          if (b_kn) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + j * (64 * BK * 2), &tmB, n0 + j * 64, kb * BK,
                          &bars->full[stage]);
          } else {
            tma_load_2d(sB, &tmB, kb * BK, n0, &bars->full[stage]);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every issued load must land before the CTA may exit (only
      // matters when a wait above gave up; otherwise these pass at once).
      const uint32_t last = issued < (uint32_t)kStages ? issued : (uint32_t)kStages;
      for (uint32_t i = 0; i < last; ++i) {
        const uint32_t idx = issued - 1 - i;
        mbar_wait(&bars->full[idx % kStages], (idx / kStages) & 1u, 1000000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      // Descriptors built once, advanced by 32-bit adds to their address
      // field (every address here is below 256 KiB: no carry out of it).
      const uint32_t base_addr = smem_u32(stage_base);
      const uint64_t da0 = smem_desc_sw128(base_addr, 16, 1024);
      const uint64_t db0 = b_kn ? smem_desc_sw128(base_addr + kABytes, 64 * BK * 2, 1024)
                                : smem_desc_sw128(base_addr + kABytes, 16, 1024);
      const uint32_t da_lo = (uint32_t)da0, da_hi = (uint32_t)(da0 >> 32);
      const uint32_t db_lo = (uint32_t)db0, db_hi = (uint32_t)(db0 >> 32);
      const uint32_t b_kstep = b_kn ? (16 * 128) >> 4 : 32 >> 4;  // per K = 16
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const uint32_t idesc = (u < num_full) ? idesc_full : idesc_half;
        if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kAccCols;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t soff = (stage * kStageBytes) >> 4;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss_lohi(d_tmem, da_lo + soff + k * (32 >> 4), da_hi, db_lo + soff + k * b_kstep,
                            db_hi, idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit(&bars->empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit(&bars->acc_full[acc]);
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5, thread = accumulator row
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    uint8_t *warp_stage = epi_base + quad * 8192;
    int local = 0;
    uint32_t chunk_count = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int tm, n0, width;
      unit_tile(u, tm, n0, width);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&bars->acc_full[acc], acc_phase)) break;
      tc_fence_after();
      const int m0 = tm * BM;
      const int gr = m0 + row;
      const int nchunks = width / kEpiCols;
      for (int c = 0; c < nchunks; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + acc * kAccCols + c * kEpiCols, v);
        tmem_ld_wait();
        if (c == nchunks - 1) {
          tc_fence_before();
          mbar_arrive(&bars->acc_empty[acc]);
        }
        const int cn0 = n0 + c * kEpiCols;
        if (cn0 >= N) continue;  // tile-uniform: whole box right of the matrix
        if (Cin != nullptr && gr < M) {
          const float *crow = Cin + (int64_t)gr * ldc;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (cn0 + j < N) v[j] = __float_as_uint(__uint_as_float(v[j]) + crow[cn0 + j]);
        }
        epilogue_store_box(&tmD, warp_stage, v, lane, chunk_count, cn0, m0 + quad * 32);
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------ CTA-pair kernel
// Same contract, for problems with at least two 128-row blocks: clusters of
// two CTAs drive one cta_group::2 MMA of M = 256 (128 rows per CTA), N = 256.
// Each CTA loads its own 128 rows of A and its own 128-column half of the B
// panel (16 + 16 KiB per 64-deep K block), so a CTA reads 32 KiB from L2 per
// block instead of 48 KiB for the same 128 x 256 outputs. CTA 0 issues the
// MMAs; both CTAs' TMA copies count on CTA 0's full barriers; CTA 0's commits
// release the empty barriers and accumulator-full barriers of both CTAs; both
// epilogues release CTA 0's accumulator-empty barriers. Each CTA's TMEM holds
// its 128 accumulator rows (2 x 256 columns, double-buffered). Work units are
// 256 x 256 pair tiles; a tail wave that fills at most half the clusters is
// split into 256 x 128 halves.
constexpr int kPairStages = 3;  // of kPairSub K blocks each
// Tile-order groups of 8 pair rows when the B operand exceeds this many bytes
// (it then no longer stays in L2 with row-major order: 8192^3 +6 %, while
// 4096^3, whose B fits, measured 1.5 % faster row-major).
constexpr int kGroupRows = 8;
constexpr size_t kGroupAboveBBytes = 64ull << 20;
constexpr uint32_t kPairABytes = 128 * BK * 2;  // this CTA's A rows
constexpr uint32_t kPairBBytes = 128 * BK * 2;  // this CTA's half of the B panel
constexpr uint32_t kPairSubBytes = kPairABytes + kPairBBytes;  // one 64-deep K block
// Each barrier stage holds kPairSub consecutive 64-deep K blocks: per stage
// the issuing thread waits once and commits once per CTA for 8 MMAs instead
// of 4 (it was the bottleneck: ~580 cycles of issue per 64-deep block against
// 512 of MMA, measured).
constexpr int kPairSub = 2;
constexpr uint32_t kPairStageBytes = kPairSub * kPairSubBytes;

struct __align__(8) PairBarriers {
  uint64_t full[kPairStages];   // used in CTA 0
  uint64_t empty[kPairStages];  // both CTAs
  uint64_t acc_full[2];         // both CTAs
  uint64_t acc_empty[2];        // used in CTA 0 (both epilogues arrive)
  uint32_t tmem_base;
};

constexpr size_t kPairSmemBytes =
    1024 + kPairStages * kPairStageBytes + 2 * kEpiBytes + sizeof(PairBarriers);

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmBh,
                         const __grid_constant__ CUtensorMap tmD,
                         const float *__restrict__ Cin, int64_t ldc, int M, int N, int K,
                         uint32_t idesc_full, uint32_t idesc_half, int b_kn, int num_full,
                         int num_units, int group_rows) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stage_base = smem;
  uint8_t *epi_base = smem + kPairStages * kPairStageBytes;
  PairBarriers *bars = reinterpret_cast<PairBarriers *>(epi_base + 2 * kEpiBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_m = (M + 2 * BM - 1) / (2 * BM);
  const int kstages = ((K + BK - 1) / BK + kPairSub - 1) / kPairSub;  // barrier stages per unit
  // Tile order: groups of `group_rows` pair rows, column by column within a
  // group, so the tiles in flight (one per cluster) share a few A and B
  // panels that stay in L2 even when all of B does not (8192^3, groups of 8:
  // ~70 MB in flight). group_rows = 1 is plain row-major order.
  auto unit_tile = [&](int u, int &tm, int &n0, int &width) {
    int tile = u, half = 0;
    width = BN;
    if (u >= num_full) {
      tile = num_full + (u - num_full) / 2;
      half = (u - num_full) & 1;
      width = BN / 2;
    }
    const int group = tile / (group_rows * tiles_n);
    const int first_m = group * group_rows;
    const int rows = min(tiles_m - first_m, group_rows);
    const int in_group = tile - group * group_rows * tiles_n;
    tm = first_m + in_group % rows;
    n0 = (in_group / rows) * BN + half * (BN / 2);
  };
  // Barrier addresses in the cluster window.
  auto lead = [&](uint64_t *b) { return mapa_shared(smem_u32(b), 0); };
  auto peer = [&](uint64_t *b) { return mapa_shared(smem_u32(b), 1); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 2 * kEpiThreads);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmBh);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Launched with programmatic stream serialization: the next launch may be
  // scheduled from here on (its blocks take an SM as this grid's leave it and
  // set up there), and this grid touches global memory only once the previous
  // one has completed.
  grid_launch_dependents();
  grid_dependency_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int u = cluster; ok && u < num_units; u += num_clusters) {
        int tm, n0, width;
        unit_tile(u, tm, n0, width);
        const int a_row = tm * 2 * BM + rank * BM;
        const int b_col = n0 + rank * (width / 2);
        // A half unit (N = 128 per pair) needs 64 columns of B per CTA: it
        // loads only those, so its stages carry 24 KiB per CTA instead of 32
        // (loading the full 128 made the tail's half units as slow as full
        // tiles: the stage copies, not the MMAs, set their pace).
        const bool half = width < BN;
        const uint32_t sub_bytes = kPairABytes + (half ? kPairBBytes / 2 : kPairBBytes);
        // A K block past K (odd block count) loads as zeros (TMA fill) and
        // adds nothing.
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1u)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[stage], 2 * kPairSub * sub_bytes);
          const uint32_t fb = lead(&bars->full[stage]);
#pragma unroll
          for (int sub = 0; sub < kPairSub; ++sub) {
            const int kb = ks * kPairSub + sub;
            uint8_t *sA = stage_base + stage * kPairStageBytes + sub * kPairSubBytes;
            uint8_t *sB = sA + kPairABytes;
            tma_load_2d_pair(sA, &tmA, kb * BK, a_row, fb);
            if (b_kn) {
              tma_load_2d_pair(sB, &tmB, b_col, kb * BK, fb);
              if (!half) tma_load_2d_pair(sB + 64 * BK * 2, &tmB, b_col + 64, kb * BK, fb);
            } else {
              tma_load_2d_pair(sB, half ? &tmBh : &tmB, kb * BK, b_col, fb);
            }
          }
          ++issued;
          if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain (CTA 0 sees both CTAs' bytes on its full barriers).
      if (rank == 0) {
        const uint32_t last = issued < (uint32_t)kPairStages ? issued : (uint32_t)kPairStages;
        for (uint32_t i = 0; i < last; ++i) {
          const uint32_t idx = issued - 1 - i;
          mbar_wait(&bars->full[idx % kPairStages], (idx / kPairStages) & 1u, 1000000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (CTA 0): the whole warp runs the loop,
      // one elected lane issues each MMA and commit; waits are made
      // warp-uniform (a timeout seen by any lane ends the loop for all).
      // Descriptors and the two CTAs' barrier addresses built once and
      // advanced by 32-bit adds: each instruction this thread issues per MMA
      // delays the MMAs (with descriptors rebuilt per MMA the issue pace,
      // not the tensor pipe, set the mainloop's rate: tail half-units, half
      // the MMA work, took as long as full units).
      const uint32_t base_addr = smem_u32(stage_base);
      const uint64_t da0 = smem_desc_sw128(base_addr, 16, 1024);
      const uint64_t db0 = b_kn ? smem_desc_sw128(base_addr + kPairABytes, 64 * BK * 2, 1024)
                                : smem_desc_sw128(base_addr + kPairABytes, 16, 1024);
      const uint32_t da_lo = (uint32_t)da0, da_hi = (uint32_t)(da0 >> 32);
      const uint32_t db_lo = (uint32_t)db0, db_hi = (uint32_t)(db0 >> 32);
      const uint32_t b_kstep = b_kn ? (16 * 128) >> 4 : 32 >> 4;  // per K = 16
      const uint32_t empty_lead = lead(&bars->empty[0]), empty_peer = peer(&bars->empty[0]);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int u = cluster; ok && u < num_units; u += num_clusters, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const uint32_t idesc = (u < num_full) ? idesc_full : idesc_half;
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kAccCols;
        for (int ks = 0; ks < kstages; ++ks) {
          if (!__all_sync(0xffffffffu, mbar_wait(&bars->full[stage], phase))) { ok = false; break; }
          tc_fence_after();
          const uint32_t soff = (stage * kPairStageBytes) >> 4;
#pragma unroll
          for (int k = 0; k < kPairSub * (BK / 16); ++k) {
            const uint32_t off = soff + (k / (BK / 16)) * (kPairSubBytes >> 4);
            const int kk = k % (BK / 16);
            mma_f16_ss_pair_lohi_warp(d_tmem, da_lo + off + kk * (32 >> 4), da_hi,
                                 db_lo + off + kk * b_kstep, db_hi, idesc,
                                 (ks | k) != 0 ? 1u : 0u);
          }
          mma_commit_pair_warp(empty_lead + stage * 8);
          mma_commit_pair_warp(empty_peer + stage * 8);
          if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair_warp(lead(&bars->acc_full[acc]));
        mma_commit_pair_warp(peer(&bars->acc_full[acc]));
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): warps 2..5, thread = row
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    uint8_t *warp_stage = epi_base + quad * 8192;
    const uint32_t acc_empty_lead0 = lead(&bars->acc_empty[0]);
    const uint32_t acc_empty_lead1 = lead(&bars->acc_empty[1]);
    int local = 0;
    uint32_t chunk_count = 0;
    for (int u = cluster; u < num_units; u += num_clusters, ++local) {
      int tm, n0, width;
      unit_tile(u, tm, n0, width);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&bars->acc_full[acc], acc_phase)) break;
      tc_fence_after();
      const int m0 = tm * 2 * BM + rank * BM;
      const int gr = m0 + row;
      const int nchunks = width / kEpiCols;
      for (int c = 0; c < nchunks; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + acc * kAccCols + c * kEpiCols, v);
        tmem_ld_wait();
        if (c == nchunks - 1) {
          tc_fence_before();
          if (rank == 0) mbar_arrive(&bars->acc_empty[acc]);
          else mbar_arrive_cluster(acc ? acc_empty_lead1 : acc_empty_lead0);
        }
        const int cn0 = n0 + c * kEpiCols;
        if (cn0 >= N) continue;
        if (Cin != nullptr && gr < M) {
          const float *crow = Cin + (int64_t)gr * ldc;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (cn0 + j < N) v[j] = __float_as_uint(__uint_as_float(v[j]) + crow[cn0 + j]);
        }
        epilogue_store_box(&tmD, warp_stage, v, lane, chunk_count, cn0, m0 + quad * 32);
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  cluster_sync();  // both CTAs done with TMEM and with each other's barriers
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                  void *, const cuuint64_t *, const cuuint64_t *,
                                  const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

bool make_map_2d(CUtensorMap *map, CUtensorMapDataType type, int elem_bytes,
                 const void *base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto encode = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!encode) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, type, 2, const_cast<void *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

struct MapCache {
  GemmArgs key{};
  int device = -1;
  CUtensorMap a, b, b_pair, b_pair_half, d;
  bool valid = false;
};

bool same_key(const GemmArgs &x, const GemmArgs &y) {
  return x.A == y.A && x.B == y.B && x.D == y.D && x.M == y.M && x.N == y.N &&
         x.K == y.K && x.lda == y.lda && x.ldb == y.ldb && x.ldd == y.ldd &&
         x.bf16 == y.bf16 && x.b_kn == y.b_kn;
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Clusters of two that can be resident at once (SM pairs within GPCs); the
// persistent grid must not exceed it or late clusters would run a second wave.
int pair_clusters_resident(int dev, int sms) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return sms / 2;
  if (cached[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms & ~1, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kPairSmemBytes;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tcgen05_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;
    }
    cached[dev] = n < sms / 2 ? n : sms / 2;
  }
  return cached[dev];
}

}  // namespace

cudaError_t launch_gemm_tcgen05(const GemmArgs &g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaErrorInvalidValue;
  // TMA rules: 16-byte aligned bases, row strides multiples of 16 bytes.
  if (!al16(g.A) || !al16(g.B) || !al16(g.D)) return cudaErrorNotSupported;
  if (g.lda % 8 || g.ldb % 8 || g.ldd % 4) return cudaErrorNotSupported;
  if (g.lda < g.K || g.ldd < g.N) return cudaErrorInvalidValue;
  if (g.b_kn ? g.ldb < g.N : g.ldb < g.K) return cudaErrorInvalidValue;
  if (g.Cin && g.ldc < g.N) return cudaErrorInvalidValue;

  static thread_local MapCache cache;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(cache.valid && cache.device == dev && same_key(cache.key, g))) {
    const CUtensorMapDataType t16 =
        g.bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    bool ok = make_map_2d(&cache.a, t16, 2, g.A, g.K, g.M, g.lda, BK, BM);
    if (g.b_kn) {
      ok = ok && make_map_2d(&cache.b, t16, 2, g.B, g.N, g.K, g.ldb, 64, BK);
      cache.b_pair = cache.b;
      cache.b_pair_half = cache.b;
    } else {
      ok = ok && make_map_2d(&cache.b, t16, 2, g.B, g.K, g.N, g.ldb, BK, BN);
      ok = ok && make_map_2d(&cache.b_pair, t16, 2, g.B, g.K, g.N, g.ldb, BK, BN / 2);
      ok = ok && make_map_2d(&cache.b_pair_half, t16, 2, g.B, g.K, g.N, g.ldb, BK, BN / 4);
    }
    ok = ok && make_map_2d(&cache.d, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.D, g.N, g.M,
                           g.ldd, kEpiCols, 32);
    if (!ok) {
      cache.valid = false;
      return cudaErrorNotSupported;
    }
    cache.key = g;
    cache.device = dev;
    cache.valid = true;
  }

  static uint64_t configured_device_mask = 0;  // devices whose smem attributes are set
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(configured_device_mask & (1ull << dev))) {
      cudaError_t e = cudaFuncSetAttribute(gemm_tcgen05_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemBytes);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_tcgen05_pair_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kPairSmemBytes);
      if (e != cudaSuccess) return e;
      if (dev < 64) configured_device_mask |= (1ull << dev);
    }
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (g.M > BM && sms >= 2) {
    // CTA-pair kernel: 256 x 256 pair tiles over sms / 2 clusters.
    const int pair_tiles = ((g.M + 2 * BM - 1) / (2 * BM)) * ((g.N + BN - 1) / BN);
    const int resident = pair_clusters_resident(dev, sms);
    const int clusters = pair_tiles < resident ? pair_tiles : resident;
    const int tail = pair_tiles % clusters;
    const bool split = tail > 0 && 2 * tail <= clusters;
    const int num_full = split ? pair_tiles - tail : pair_tiles;
    const int num_units = split ? num_full + 2 * tail : pair_tiles;
    const uint32_t idesc_full = idesc_f16_f32(2 * BM, BN, g.bf16, false, g.b_kn);
    const uint32_t idesc_half = idesc_f16_f32(2 * BM, BN / 2, g.bf16, false, g.b_kn);
    // Programmatic stream serialization: back-to-back launches overlap the
    // next one's launch and set-up with this one's last wave (the kernel
    // waits for the previous grid before touching global memory).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kPairSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_tcgen05_pair_kernel, cache.a, cache.b_pair,
                              cache.b_pair_half, cache.d,
                              g.Cin, g.ldc, g.M, g.N, g.K, idesc_full, idesc_half,
                              g.b_kn ? 1 : 0, num_full, num_units,
                              (size_t)g.K * (size_t)g.N * 2 > kGroupAboveBBytes ? kGroupRows : 1);
  }
  const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  const int grid = tiles < sms ? tiles : sms;
  // Tail split: when the last partial wave fills at most half the CTAs, its
  // tiles run as two half-width units each, halving the tail's duration.
  const int tail = tiles % grid;
  const bool split = tail > 0 && 2 * tail <= grid;
  const int num_full = split ? tiles - tail : tiles;
  const int num_units = split ? num_full + 2 * tail : tiles;
  const uint32_t idesc_full = idesc_f16_f32(BM, BN, g.bf16, false, g.b_kn);
  const uint32_t idesc_half = idesc_f16_f32(BM, BN / 2, g.bf16, false, g.b_kn);
  gemm_tcgen05_kernel<<<grid, kThreads, kSmemBytes, stream>>>(
      cache.a, cache.b, cache.d, g.Cin, g.ldc, g.M, g.N, g.K, idesc_full, idesc_half,
      g.b_kn ? 1 : 0, num_full, num_units);
  return cudaGetLastError();
}

}  // namespace vcb

VCB_DEFINE_ERROR_ACCESSOR(gemm_tcgen05_error)
