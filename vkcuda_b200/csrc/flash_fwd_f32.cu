// flash_fwd_f32.cu - fp32 flash-attention forward on CUDA cores, for the
// reference demo's own precision (examples/flash_attn.vc:56-126: fp32
// Q/K/V/O, scale = log2(e)/sqrt(d) applied to QK^T, base-2 online softmax,
// causal mask key j > query i) and for the fp32 benchmark config.
//
// The reference gives one thread a whole query row. Here a row is split over
// 16 lanes (each takes every 16th key of a 32-key tile held in shared
// memory), every lane keeps its own running max / sum / accumulator in fp32,
// and the 16 partial states are merged with shuffles at the end:
//   m = max(m_a, m_b), l = l_a 2^(m_a-m) + l_b 2^(m_b-m), acc likewise.
// 8 rows per 128-thread block; any head dimension d <= 128. exp2f is the
// accurate CUDA function, so the result tracks an fp64 evaluation to ~1e-6
// for unit-variance inputs.
#include <cuda_runtime.h>
#include <cmath>
#include <cstdint>

#include "internal.h"

namespace vcb {
namespace {

constexpr int kRows = 8, kSplit = 16, kKeyTile = 32;

// D is the compile-time capacity; the head dimension d <= D is a launch
// argument (columns d..D-1 of the staged tiles are zero, so they add nothing).
template <int D>
__global__ void __launch_bounds__(kRows *kSplit)
flash_f32_kernel(const float *__restrict__ Q, const float *__restrict__ K,
                 const float *__restrict__ V, float *__restrict__ O, int N, int d,
                 float scale_log2, int causal) {
  __shared__ float Qs[kRows][D + 1];
  __shared__ float Ks[kKeyTile][D + 1];
  __shared__ float Vs[kKeyTile][D + 1];
  const int64_t base = static_cast<int64_t>(blockIdx.y) * N * d;
  const int q0 = blockIdx.x * kRows;
  const int r = threadIdx.x / kSplit, sp = threadIdx.x % kSplit;
  const int qi = q0 + r;

  for (int i = threadIdx.x; i < kRows * D; i += blockDim.x) {
    const int rr = i / D, dd = i % D;
    Qs[rr][dd] = (q0 + rr < N && dd < d) ? Q[base + static_cast<int64_t>(q0 + rr) * d + dd] : 0.0f;
  }
  float m = -INFINITY, l = 0.0f, acc[D];
#pragma unroll
  for (int dd = 0; dd < D; ++dd) acc[dd] = 0.0f;

  const int kend = causal ? min(N, q0 + kRows) : N;
  for (int k0 = 0; k0 < kend; k0 += kKeyTile) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKeyTile * D; i += blockDim.x) {
      const int rr = i / D, dd = i % D;
      const bool in = (k0 + rr < N) && dd < d;
      const int64_t off = base + static_cast<int64_t>(k0 + rr) * d + dd;
      Ks[rr][dd] = in ? K[off] : 0.0f;
      Vs[rr][dd] = in ? V[off] : 0.0f;
    }
    __syncthreads();
    for (int jj = sp; jj < kKeyTile; jj += kSplit) {
      const int j = k0 + jj;
      if (j >= N || (causal && j > qi)) continue;
      float dot = 0.0f;
#pragma unroll
      for (int dd = 0; dd < D; ++dd) dot = fmaf(Qs[r][dd], Ks[jj][dd], dot);
      const float s = dot * scale_log2;
      if (s > m) {
        const float alpha = exp2f(m - s);  // 0 when m = -inf
        l *= alpha;
#pragma unroll
        for (int dd = 0; dd < D; ++dd) acc[dd] *= alpha;
        m = s;
      }
      const float p = exp2f(s - m);
      l += p;
#pragma unroll
      for (int dd = 0; dd < D; ++dd) acc[dd] = fmaf(p, Vs[jj][dd], acc[dd]);
    }
  }
  // Merge the 16 lane states of the row (lanes of a row are consecutive).
#pragma unroll
  for (int off = kSplit / 2; off > 0; off >>= 1) {
    const float m_o = __shfl_xor_sync(0xffffffffu, m, off);
    const float l_o = __shfl_xor_sync(0xffffffffu, l, off);
    const float mn = fmaxf(m, m_o);
    const float a = (m == -INFINITY) ? 0.0f : exp2f(m - mn);
    const float b = (m_o == -INFINITY) ? 0.0f : exp2f(m_o - mn);
    l = l * a + l_o * b;
#pragma unroll
    for (int dd = 0; dd < D; ++dd) {
      const float acc_o = __shfl_xor_sync(0xffffffffu, acc[dd], off);
      acc[dd] = acc[dd] * a + acc_o * b;
    }
    m = mn;
  }
  if (qi < N) {
    const float inv = 1.0f / l;
#pragma unroll
    for (int dd = 0; dd < D; ++dd)
      if (dd % kSplit == sp && dd < d) O[base + static_cast<int64_t>(qi) * d + dd] = acc[dd] * inv;
  }
}

}  // namespace

cudaError_t launch_flash_fwd_f32(const FlashArgs &f, cudaStream_t stream) {
  if (f.BH <= 0 || f.N <= 0 || f.BH > 65535) return cudaErrorInvalidValue;
  dim3 grid((f.N + kRows - 1) / kRows, f.BH);
  const float *Q = static_cast<const float *>(f.Q), *K = static_cast<const float *>(f.K),
              *V = static_cast<const float *>(f.V);
  float *O = static_cast<float *>(f.O);
  const int c = f.causal ? 1 : 0;
  // Smallest compiled capacity that holds d.
  if (f.d <= 0 || f.d > 128) return cudaErrorInvalidValue;
  if (f.d <= 16)
    flash_f32_kernel<16><<<grid, kRows * kSplit, 0, stream>>>(Q, K, V, O, f.N, f.d, f.scale_log2, c);
  else if (f.d <= 32)
    flash_f32_kernel<32><<<grid, kRows * kSplit, 0, stream>>>(Q, K, V, O, f.N, f.d, f.scale_log2, c);
  else if (f.d <= 64)
    flash_f32_kernel<64><<<grid, kRows * kSplit, 0, stream>>>(Q, K, V, O, f.N, f.d, f.scale_log2, c);
  else
    flash_f32_kernel<128><<<grid, kRows * kSplit, 0, stream>>>(Q, K, V, O, f.N, f.d, f.scale_log2, c);
  return cudaGetLastError();
}

}  // namespace vcb
