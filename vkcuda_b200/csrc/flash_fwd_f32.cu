// flash_fwd_f32.cu - fp32 flash-attention forward on CUDA cores, for the
// reference demo's own precision (examples/flash_attn.vc:56-126: fp32
// Q/K/V/O, scale = log2(e)/sqrt(d) applied to QK^T, base-2 online softmax,
// causal mask key j > query i) and for the fp32 benchmark config.
//
// The reference gives one thread a whole query row. Here a row is split over
// kLanes lanes of a warp (lane l takes keys l, l + kLanes, ... of each key
// tile), every lane keeps its own running max / sum / accumulator in fp32,
// and the partial states are merged with shuffles at the end:
//   m = max(m_a, m_b), l = l_a 2^(m_a-m) + l_b 2^(m_b-m), acc likewise.
// Any head dimension d <= 128. K/V tiles (64 keys; 32 at d > 64, halving the
// shared memory) stream through a ring of kStages shared-memory buffers
// filled by cp.async (16-byte copies when d % 4 == 0 and the rows are 16-byte
// aligned, else 4-byte), so the loads of the next tiles overlap the
// arithmetic on the current one. Rows are padded to d + 4 floats: lanes that
// read 16 bytes of different keys' rows at the same column then fall on
// distinct banks within every quarter warp, and each dot product runs as
// four independent FMA chains over float4 reads. Small grids (the
// 1 x 256 x 64 demo shape is 16.8 MFLOP, latency-bound) run 4 rows of 32
// lanes per block, for more blocks, with a 4-deep ring (all of a 256-key
// sequence in flight at once); grids that would not give every SM a 4-row
// block run, up to d = 64, 2 rows of 64 lanes (two warps per row: each lane
// walks half as many keys; 1 x 256 x 64: 8.5 -> 5.8 us per launch); grids
// that fill the GPU run 8 rows of 16 lanes, so that each staged K/V element
// serves twice the rows in a block of the same 128 threads, with a 2-deep
// ring so that several blocks share an SM. A lane rescales its running state
// once per key tile (to the tile's maximum), and the lanes of a row merge
// their states at the end through shared memory: each lane rescales its own
// accumulators to the row maximum and writes them, then sums a column per
// output element (a shuffle butterfly over the 64-wide accumulators took a
// fifth of the kernel's instructions). exp2f is the accurate CUDA function,
// so the result tracks an fp64 evaluation to ~1e-6 for unit-variance inputs.
#include <cuda_runtime.h>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "internal.h"

namespace vcb {
namespace {


__device__ __forceinline__ void cp_async4(float *smem_dst, const float *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void cp_async16(float *smem_dst, const float *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src)
               : "memory");
}

// Shared memory: Q rows, then kStages K buffers and kStages V buffers of
// kKeyTile keys; rows padded to D + 4 floats (16-byte aligned rows whose
// 16-byte columns spread over the banks, see above).
template <int D, int kRows, int kLanes, int kStages>
struct F32Smem {
  static constexpr int kKeyTile = D > 64 ? 32 : 64;
  static constexpr int kThreads = kRows * kLanes;
  static constexpr int kPitch = D + 4;
  static constexpr size_t kQ = 0;
  static constexpr size_t kK = kQ + size_t(kRows) * kPitch;
  static constexpr size_t kV = kK + kStages * size_t(kKeyTile) * kPitch;
  static constexpr size_t kFloats = kV + kStages * size_t(kKeyTile) * kPitch;
  static constexpr size_t kBytes = kFloats * sizeof(float);
};

// D is the compile-time capacity; the head dimension d <= D is a launch
// argument (columns d..D-1 of the staged tiles are zero, so they add nothing).
template <int D, int kRows, int kLanes, int kStages>
__global__ void __launch_bounds__(kRows * kLanes)
flash_f32_kernel(const float *__restrict__ Q, const float *__restrict__ K,
                 const float *__restrict__ V, float *__restrict__ O, int N, int d,
                 float scale_log2, int causal, int vec16) {
  using L = F32Smem<D, kRows, kLanes, kStages>;
  constexpr int kKeyTile = L::kKeyTile, kThreads = L::kThreads;
  extern __shared__ float fsm[];
  float *Qs = fsm + L::kQ;
  const int64_t base = static_cast<int64_t>(blockIdx.y) * N * d;
  const int q0 = blockIdx.x * kRows;
  const int r = threadIdx.x / kLanes, lane = threadIdx.x % kLanes;
  const int qi = q0 + r;

  for (int i = threadIdx.x; i < kRows * D; i += kThreads) {
    const int rr = i / D, dd = i % D;
    Qs[rr * L::kPitch + dd] =
        (q0 + rr < N && dd < d) ? Q[base + static_cast<int64_t>(q0 + rr) * d + dd] : 0.0f;
  }
  // Stage key tile t into buffer b: cp.async for elements in range, zeros
  // (plain stores) elsewhere; one commit group per tile.
  auto stage = [&](int t, int b) {
    float *Kb = fsm + L::kK + size_t(b) * kKeyTile * L::kPitch;
    float *Vb = fsm + L::kV + size_t(b) * kKeyTile * L::kPitch;
    const int k0 = t * kKeyTile;
    if (vec16) {
      // d % 4 == 0: a 4-float group is wholly inside or outside the row.
      for (int i = threadIdx.x; i < kKeyTile * (D / 4); i += kThreads) {
        const int rr = i / (D / 4), dd = (i % (D / 4)) * 4;
        float *kd = Kb + rr * L::kPitch + dd, *vd = Vb + rr * L::kPitch + dd;
        if (k0 + rr < N && dd < d) {
          const int64_t off = base + static_cast<int64_t>(k0 + rr) * d + dd;
          cp_async16(kd, K + off);
          cp_async16(vd, V + off);
        } else {
          *reinterpret_cast<float4 *>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4 *>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    } else {
      for (int i = threadIdx.x; i < kKeyTile * D; i += kThreads) {
        const int rr = i / D, dd = i % D;
        float *kd = Kb + rr * L::kPitch + dd, *vd = Vb + rr * L::kPitch + dd;
        if (k0 + rr < N && dd < d) {
          const int64_t off = base + static_cast<int64_t>(k0 + rr) * d + dd;
          cp_async4(kd, K + off);
          cp_async4(vd, V + off);
        } else {
          *kd = 0.0f;
          *vd = 0.0f;
        }
      }
    }
    cp_async_commit();
  };

  float m = -INFINITY, l = 0.0f, acc[D];
#pragma unroll
  for (int dd = 0; dd < D; ++dd) acc[dd] = 0.0f;
  // Up to d = 64 the query row also lives in registers (beside the 64
  // accumulators); wider rows are read from shared memory.
  constexpr bool kQInRegs = D <= 64;
  constexpr int kH = kKeyTile / kLanes;  // keys of a tile per lane
  // Merge area per row, +16 floats so that the two rows of a warp (16 lanes
  // each) fall on opposite halves of the banks.
  constexpr int kMergeRowStride = D * (kLanes + 1) + 16;
  static_assert(size_t(kRows) * kMergeRowStride <= L::kFloats, "merge area fits");
  float4 qreg[kQInRegs ? D / 4 : 1];

  const int kend = causal ? min(N, q0 + kRows) : N;
  const int ntiles = (kend + kKeyTile - 1) / kKeyTile;
  // Tiles 0 .. kStages-2 up front; every iteration adds one more (or an empty
  // group past the end), so "all but the newest kStages-1 groups complete"
  // means tile t has landed.
#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) {
    if (t < ntiles) stage(t, t);
    else cp_async_commit();
  }
  for (int t = 0; t < ntiles; ++t) {
    const int ahead = t + kStages - 1;
    if (ahead < ntiles) stage(ahead, ahead % kStages);
    else cp_async_commit();
    cp_async_wait<kStages - 1>();  // this thread's copies of tile t have landed
    __syncthreads();  // everyone's copies and zero fills of tile t (and Q) visible
    const float *Kb = fsm + L::kK + size_t(t % kStages) * kKeyTile * L::kPitch;
    const float *Vb = fsm + L::kV + size_t(t % kStages) * kKeyTile * L::kPitch;
    const float *qrow = Qs + r * L::kPitch;
    if (kQInRegs && t == 0) {
#pragma unroll
      for (int c = 0; c < (kQInRegs ? D / 4 : 1); ++c)
        qreg[c] = reinterpret_cast<const float4 *>(qrow)[c];
    }
    // Scores of this lane's keys of the tile first, then one rescale of the
    // running state to the tile's maximum, then the probabilities.
    float sc[kH];
    float mt = m;
#pragma unroll
    for (int h = 0; h < kH; ++h) {
      const int jj = lane + h * kLanes;
      const int j = t * kKeyTile + jj;
      const float4 *k4 = reinterpret_cast<const float4 *>(Kb + jj * L::kPitch);
      const float4 *q4 = reinterpret_cast<const float4 *>(qrow);
      float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;
#pragma unroll
      for (int c = 0; c < D / 4; ++c) {
        const float4 qv = kQInRegs ? qreg[kQInRegs ? c : 0] : q4[c];
        const float4 kv = k4[c];
        d0 = fmaf(qv.x, kv.x, d0);
        d1 = fmaf(qv.y, kv.y, d1);
        d2 = fmaf(qv.z, kv.z, d2);
        d3 = fmaf(qv.w, kv.w, d3);
      }
      const bool valid = j < N && !(causal && j > qi);
      sc[h] = valid ? ((d0 + d1) + (d2 + d3)) * scale_log2 : -INFINITY;
      mt = fmaxf(mt, sc[h]);
    }
    if (mt > m) {
      const float alpha = exp2f(m - mt);  // 0 when m = -inf
      l *= alpha;
#pragma unroll
      for (int dd = 0; dd < D; ++dd) acc[dd] *= alpha;
      m = mt;
    }
#pragma unroll
    for (int h = 0; h < kH; ++h) {
      if (sc[h] == -INFINITY) continue;  // masked or past the end
      const int jj = lane + h * kLanes;
      const float p = exp2f(sc[h] - m);
      l += p;
      const float4 *v4 = reinterpret_cast<const float4 *>(Vb + jj * L::kPitch);
#pragma unroll
      for (int c = 0; c < D / 4; ++c) {
        const float4 vv = v4[c];
        acc[4 * c] = fmaf(p, vv.x, acc[4 * c]);
        acc[4 * c + 1] = fmaf(p, vv.y, acc[4 * c + 1]);
        acc[4 * c + 2] = fmaf(p, vv.z, acc[4 * c + 2]);
        acc[4 * c + 3] = fmaf(p, vv.w, acc[4 * c + 3]);
      }
    }
    __syncthreads();  // buffer t % kStages is refilled by the stage() of iteration t + 1
  }
  // Merge the row's kLanes lane states (consecutive lanes: one warp, half a
  // warp, or two warps for kLanes = 64): the row maximum and the rescaled sum
  // by shuffles (and, across the two warps of a 64-lane row, through shared
  // memory), the rescaled accumulators through shared memory (all of the
  // dynamic area is free once the last tile's trailing barrier has passed),
  // [D][kLanes + 1] per row so that both the writes and the column sums below
  // touch 32 distinct banks; each lane then sums the output columns
  // dd = lane (mod kLanes).
  constexpr int kWarpLanes = kLanes < 32 ? kLanes : 32;
  constexpr int kRowWarps = kLanes / kWarpLanes;
  __shared__ float row_red[kRows][kRowWarps][2];
  float mrow = m;
#pragma unroll
  for (int off = kWarpLanes / 2; off > 0; off >>= 1)
    mrow = fmaxf(mrow, __shfl_xor_sync(0xffffffffu, mrow, off));
  if (kRowWarps > 1) {
    if ((lane & 31) == 0) row_red[r][lane >> 5][0] = mrow;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kRowWarps; ++w) mrow = fmaxf(mrow, row_red[r][w][0]);
  }
  const float own = (m == -INFINITY) ? 0.0f : exp2f(m - mrow);
  float lrow = l * own;
#pragma unroll
  for (int off = kWarpLanes / 2; off > 0; off >>= 1)
    lrow += __shfl_xor_sync(0xffffffffu, lrow, off);
  if (kRowWarps > 1) {
    if ((lane & 31) == 0) row_red[r][lane >> 5][1] = lrow;
  }
  float *part = fsm + size_t(r) * kMergeRowStride;
#pragma unroll
  for (int dd = 0; dd < D; ++dd) part[dd * (kLanes + 1) + lane] = acc[dd] * own;
  if (kRowWarps > 1) {
    __syncthreads();
    lrow = 0.0f;
#pragma unroll
    for (int w = 0; w < kRowWarps; ++w) lrow += row_red[r][w][1];
  } else {
    __syncwarp();
  }
  if (qi < N) {
    const float inv = 1.0f / lrow;
    for (int dd = lane; dd < d; dd += kLanes) {
      const float *col = part + dd * (kLanes + 1);
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int j = 0; j < kLanes; j += 2) {
        s0 += col[j];
        s1 += col[j + 1];
      }
      O[base + static_cast<int64_t>(qi) * d + dd] = (s0 + s1) * inv;
    }
  }
}

template <int D, int kRows, int kLanes, int kStages>
cudaError_t launch_dr(const FlashArgs &f, cudaStream_t stream) {
  using L = F32Smem<D, kRows, kLanes, kStages>;
  static uint64_t configured = 0;  // devices whose smem attribute is set
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(configured & (1ull << dev))) {
      cudaError_t e = cudaFuncSetAttribute(flash_f32_kernel<D, kRows, kLanes, kStages>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)L::kBytes);
      if (e != cudaSuccess) return e;
      if (dev < 64) configured |= (1ull << dev);
    }
  }
  dim3 grid((f.N + kRows - 1) / kRows, f.BH);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec16 = (f.d % 4 == 0 && al16(f.K) && al16(f.V)) ? 1 : 0;
  flash_f32_kernel<D, kRows, kLanes, kStages><<<grid, L::kThreads, L::kBytes, stream>>>(
      static_cast<const float *>(f.Q), static_cast<const float *>(f.K),
      static_cast<const float *>(f.V), static_cast<float *>(f.O), f.N, f.d, f.scale_log2,
      f.causal ? 1 : 0, vec16);
  return cudaGetLastError();
}

// 4 rows of 32 lanes while 8-row blocks would not give every SM two of them,
// else 8 rows of 16 lanes.
template <int D>
cudaError_t launch_d(const FlashArgs &f, cudaStream_t stream) {
  const int sms = sm_count_current();
  const long long blocks8 = (long long)f.BH * ((f.N + 7) / 8);
  if (blocks8 >= 2LL * sms) return launch_dr<D, 8, 16, 2>(f, stream);
  // Grids too small to fill the GPU with 4-row blocks: up to d = 64, two
  // rows of 64 lanes (two warps) per block halve the keys each lane walks.
  if (D <= 64 && (long long)f.BH * ((f.N + 3) / 4) < sms) {
    if constexpr (D <= 64) return launch_dr<D, 2, 64, 4>(f, stream);
  }
  return launch_dr<D, 4, 32, 4>(f, stream);
}

}  // namespace

cudaError_t launch_flash_fwd_f32(const FlashArgs &f, cudaStream_t stream) {
  if (f.BH <= 0 || f.N <= 0 || f.BH > 65535) return cudaErrorInvalidValue;
  // Smallest compiled capacity that holds d.
  if (f.d <= 0 || f.d > 128) return cudaErrorInvalidValue;
  if (f.d <= 16) return launch_d<16>(f, stream);
  if (f.d <= 32) return launch_d<32>(f, stream);
  if (f.d <= 64) return launch_d<64>(f, stream);
  return launch_d<128>(f, stream);
}

}  // namespace vcb
