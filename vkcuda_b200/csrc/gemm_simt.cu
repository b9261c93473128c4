// gemm_simt.cu - CUDA-core GEMMs for the cases the tensor-core path does not
// take:
//   * fp16/bf16 -> fp32 GEMM with arbitrary strides and alignment (row
//     strides that break TMA's 16-byte rule), same contract as the tcgen05
//     path: D = A * B (+ Cin), fp32 accumulation in K order;
//   * fp32 D = A * B (+ Cin) with strides the fp32 tensor-core path
//     (gemm_f32_tcgen05.cu) cannot take; that path serves the reference's
//     SIMT benchmark kernel matmulTiled (examples/matmul_bench.vc:22-54,
//     16x16 shared-memory tiles) otherwise.
// Both use 64x64 output tiles per 256-thread block with 4x4 outputs per
// thread and 16-deep K slabs staged in shared memory.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "internal.h"

namespace vcb {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

// out[m][n] = sum_k A[m][k] * B(k, n) (+ Cin[m][n]); B(k, n) = b_kn ?
// B[k*ldb + n] : B[n*ldb + k].
template <typename T>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const T *__restrict__ A, const T *__restrict__ B, float *__restrict__ D,
                 const float *__restrict__ Cin, int M, int N, int K, int64_t lda,
                 int64_t ldb, int64_t ldd, int64_t ldc, int b_kn) {
  __shared__ float As[TK][TM + 1];
  __shared__ float Bs[TK][TN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int r = i / TK, k = i % TK;
      const int gm = m0 + r, gk = k0 + k;
      As[k][r] = (gm < M && gk < K) ? to_f32(A[(int64_t)gm * lda + gk]) : 0.0f;
    }
    for (int i = threadIdx.x; i < TN * TK; i += 256) {
      int c, k;
      if (b_kn) { k = i / TN; c = i % TN; } else { c = i / TK; k = i % TK; }
      const int gn = n0 + c, gk = k0 + k;
      float v = 0.0f;
      if (gn < N && gk < K)
        v = to_f32(b_kn ? B[(int64_t)gk * ldb + gn] : B[(int64_t)gn * ldb + gk]);
      Bs[k][c] = v;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx + 16 * j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (Cin) v += Cin[(int64_t)gm * ldc + gn];
      D[(int64_t)gm * ldd + gn] = v;
    }
  }
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmArgs &g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K < 0) return cudaErrorInvalidValue;
  dim3 grid((g.N + TN - 1) / TN, (g.M + TM - 1) / TM);
  if (grid.y > 65535) return cudaErrorInvalidValue;
  if (g.bf16)
    gemm_simt_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(g.A), static_cast<const __nv_bfloat16 *>(g.B),
        g.D, g.Cin, g.M, g.N, g.K, g.lda, g.ldb, g.ldd, g.ldc, g.b_kn ? 1 : 0);
  else
    gemm_simt_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half *>(g.A), static_cast<const __half *>(g.B), g.D, g.Cin,
        g.M, g.N, g.K, g.lda, g.ldb, g.ldd, g.ldc, g.b_kn ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_gemm_f32_simt(const GemmArgs &g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K < 0) return cudaErrorInvalidValue;
  dim3 grid((g.N + TN - 1) / TN, (g.M + TM - 1) / TM);
  if (grid.y > 65535) return cudaErrorInvalidValue;
  gemm_simt_kernel<float><<<grid, 256, 0, stream>>>(
      static_cast<const float *>(g.A), static_cast<const float *>(g.B), g.D, g.Cin, g.M, g.N,
      g.K, g.lda, g.ldb, g.ldd, g.ldc, g.b_kn ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace vcb
