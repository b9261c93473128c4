// internal.h - host-side launchers of the sm_100a kernels, shared by the
// runtime (registry adapters) and the flat C ABI. All return cudaError_t;
// shape errors that the kernels cannot serve come back as
// cudaErrorInvalidValue before anything is launched.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace vcb {

// ---- streaming (stream_kernels.cu)
// SM count of the current device (cached per device).
int sm_count_current();
int stream_max_blocks();
cudaError_t launch_vadd_f32(const float *a, const float *b, float *c, int64_t n,
                            cudaStream_t stream);
// Cross-GPU sum of the ranks' fp64 results without a library collective:
// every rank owns one mailbox in its device memory; each rank's kernel
// stores its result into slot `epoch & 1` of every mailbox over NVLink
// (peer stores into memory mapped with CUDA IPC), then the epoch as a flag,
// then waits (bounded) for all ranks' flags in its own mailbox and adds the
// results in rank order, so every rank ends with the same value. Two slots
// suffice: a rank can be at most one epoch ahead of any other.
constexpr int kMaxPeers = 8;
struct PeerMailbox {
  double partial[2][kMaxPeers];
  unsigned long long flag[2][kMaxPeers];
};
struct PeerExchange {
  PeerMailbox *mbox[kMaxPeers];  // rank i's mailbox, as addressed from this GPU
  int rank, world;               // world == 0: no exchange
  unsigned long long epoch;      // >= 1, increasing per call
};

// Sum of x (or of c = x + b written out when b != nullptr) into *out (device
// double). `partials` holds >= max_blocks doubles and `ticket` one zeroed
// unsigned int; both are left ready for the next call. With `px`, *out is the
// sum over the ranks of `px` (see PeerExchange).
cudaError_t launch_sum_f32(const float *x, const float *b, float *c, int64_t n,
                           double *out, double *partials, unsigned int *ticket,
                           int max_blocks, cudaStream_t stream,
                           const PeerExchange *px = nullptr);
// The sum of launch_sum_f32 (same grid, same order, bit-identical result)
// with its block partials and ticket in a static device array of the library
// instead of caller- or runtime-allocated memory. Allocates nothing. At most
// noalloc_sum_capacity() blocks: a grid that needs more is refused with
// cudaErrorInvalidValue and *blocks_needed says how many it needed.
int noalloc_sum_capacity();
cudaError_t launch_sum_f32_noalloc(const float *x, int64_t n, double *out, cudaStream_t stream,
                                   int *blocks_needed);
// a[i] = base + i for i < n (the multi-device demo's pattern fill).
cudaError_t launch_fill_pattern(int *a, int base, int64_t n, cudaStream_t stream);
// Block reduce with the reference's pairing; lim_in >= 0 selects the
// bounds-checked form (lim_in / lim_out: elements in and out hold).
cudaError_t launch_block_reduce_demo(const float *in, float *out, int n, int block,
                                     int groups, cudaStream_t stream, int64_t lim_in = -1,
                                     int64_t lim_out = -1);
// Bounds-checked forms (VC_CHECK_BOUNDS=1): each access is checked against
// the elements its buffer holds; a miss records kErrOutOfBounds and is skipped.
cudaError_t launch_fill_pattern_checked(int *a, int base, int64_t n, int64_t lim,
                                        cudaStream_t stream);
cudaError_t launch_vadd_f32_checked(const float *a, const float *b, float *c, int64_t n,
                                    int64_t lim_a, int64_t lim_b, int64_t lim_c,
                                    cudaStream_t stream);

// ---- GEMM (gemm_tcgen05.cu, gemm_simt.cu)
struct GemmArgs {
  const void *A;      // [M][K] row-major, stride lda elements
  const void *B;      // b_kn ? [K][N] (stride ldb) : [N][K] (stride ldb)
  float *D;           // [M][N] fp32, stride ldd
  const float *Cin;   // optional [M][N] fp32 addend, stride ldc
  int M, N, K;
  int64_t lda, ldb, ldd, ldc;
  bool bf16;          // element type of A and B (fp16 otherwise)
  bool b_kn;          // B stored K-rows x N-columns
};
// tcgen05 path; cudaErrorNotSupported when the strides / alignment do not
// meet its TMA requirements (then the caller uses the SIMT path).
cudaError_t launch_gemm_tcgen05(const GemmArgs &g, cudaStream_t stream);
cudaError_t launch_gemm_simt(const GemmArgs &g, cudaStream_t stream);
// fp32 in, fp32 out (A and B of `g` point to float; `g.bf16` is ignored):
// the tensor-core path (three tf32 products per fp32 product, fp32-level
// accuracy; cudaErrorNotSupported when strides / alignment break TMA's
// 16-byte rule) and the CUDA-core path (any strides).
cudaError_t launch_gemm_f32_tcgen05(const GemmArgs &g, cudaStream_t stream);
cudaError_t launch_gemm_f32_simt(const GemmArgs &g, cudaStream_t stream);
// 2-D tensor map over a row-major matrix of `outer` rows x `inner` elements
// (row stride in elements), box box_inner x box_outer, zero fill outside.
bool make_map_2d(CUtensorMap *map, CUtensorMapDataType type, int elem_bytes,
                 const void *base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                 uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// ---- flash attention (flash_fwd_tcgen05.cu, flash_fwd_f32.cu)
struct FlashArgs {
  const void *Q, *K, *V;
  void *O;
  int BH, N, d;
  float scale_log2;  // scores * scale_log2 are exponentiated in base 2
  bool causal;
  int dtype;         // 0 f32, 1 f16, 2 bf16
};
cudaError_t launch_flash_fwd_tcgen05(const FlashArgs &f, cudaStream_t stream);
cudaError_t launch_flash_fwd_f32(const FlashArgs &f, cudaStream_t stream);

// ---- device error words, one accessor per translation unit
int stream_kernels_error(int clear);
int gemm_tcgen05_error(int clear);
int gemm_f32_error(int clear);
int flash_tcgen05_error(int clear);
int selftest_error(int clear);
cudaError_t launch_selftest_bounded_wait(unsigned timeout_us, cudaStream_t stream);

// ---- runtime-owned scratch (runtime.cpp): per (device, stream) partials
// buffer and ticket for the reductions. Never freed before vcShutdown.
cudaError_t reduce_scratch(cudaStream_t stream, double **partials,
                           unsigned int **ticket, int *capacity);

// Driver entry point for tensor-map encoding (fetched once via the runtime).
void *tensor_map_encoder();

}  // namespace vcb
