// stream_kernels.cu - the bandwidth-bound half of the hot path on sm_100a:
//   * vadd:       c = a + b                         (test/vadd.vc:12-17)
//   * sum:        one fp64 scalar = sum of x         (test/reduce.vc scaled up)
//   * vadd_sum:   c = a + b and sum(c) in one pass   (both, fused: 12 B/elem)
//   * block reduce with the reference's exact pairing (test/reduce.vc:11-38)
//
// Layout and roofline: flat fp32 arrays in HBM. From 2^25 elements vadd and
// the fused vadd+sum stream through shared memory with 1-D bulk copies
// (stream_bulk_kernel: 1.02 of the measured copy rate at 2^30, 8-10 % above
// the vector kernels). The vector kernels move 16-byte vectors with
// streaming cache hints, keep 4 vectors per operand in flight per thread,
// and run one wave of resident CTAs on every SM (3 per SM at their 40
// registers a thread) so every SM has enough bytes in flight to cover HBM
// latency. Algorithmic traffic:
// vadd 12 B/elem, sum 4 B/elem, vadd_sum 12 B/elem.
//
// Summation order: each thread adds runs of up to 16 elements in fp32 and
// folds each run into an fp64 accumulator; warps and blocks combine in fp64;
// block partials land in a scratch array and the last block to finish adds
// them in index order. The result is deterministic for a given grid.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "../../include/vc_b200.h"
#include "internal.h"
#include "ptx.cuh"

namespace vcb {
namespace {

constexpr int kStreamThreads = 512;
constexpr int kUnroll = 4;

__device__ __forceinline__ float4 ld_stream(const float4 *p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4 *p, float4 v) { __stcs(p, v); }

__device__ __forceinline__ float4 add4(float4 x, float4 y) {
  return make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
}
__device__ __forceinline__ float hsum4(float4 v) { return (v.x + v.y) + (v.z + v.w); }

// c[i] = a[i] + b[i] over n4 float4 vectors, grid-stride, 4 vectors per
// thread per trip.
__global__ void __launch_bounds__(kStreamThreads)
vadd_vec_kernel(const float4 *__restrict__ a, const float4 *__restrict__ b,
                float4 *__restrict__ c, int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      va[u] = ld_stream(a + i + u * stride);
      vb[u] = ld_stream(b + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) st_stream(c + i + u * stride, add4(va[u], vb[u]));
  }
  for (; i < n4; i += stride) st_stream(c + i, add4(ld_stream(a + i), ld_stream(b + i)));
}

// Scalar form for the tail (n % 4) and for unaligned pointers.
__global__ void vadd_scalar_kernel(const float *__restrict__ a,
                                   const float *__restrict__ b,
                                   float *__restrict__ c, int64_t begin,
                                   int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride)
    c[i] = a[i] + b[i];
}

// Block-wide fp64 sum; result valid in thread 0.
__device__ __forceinline__ double block_sum_f64(double v, double *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    t = lane < nw ? red[lane] : 0.0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t += __shfl_down_sync(0xffffffffu, t, off);
  }
  return t;
}

// Peer exchange of this GPU's total (one thread): store it into slot
// epoch & 1 of every rank's mailbox, then the epoch as this rank's flag there
// (a system-scope fence between, so a peer that sees the flag sees the
// value), then wait for every rank's flag in this GPU's own mailbox and add
// the values in rank order. A wait past kExchangeLimitNs records a timeout in
// the device error word and gives NaN.
constexpr unsigned long long kExchangeLimitNs = 2000000000ull;
__device__ double exchange_sum(double total, const PeerExchange &px) {
  const int slot = static_cast<int>(px.epoch & 1ull);
  for (int i = 0; i < px.world; ++i)
    *reinterpret_cast<volatile double *>(&px.mbox[i]->partial[slot][px.rank]) = total;
  __threadfence_system();
  for (int i = 0; i < px.world; ++i)
    *reinterpret_cast<volatile unsigned long long *>(&px.mbox[i]->flag[slot][px.rank]) =
        px.epoch;
  PeerMailbox *own = px.mbox[px.rank];
  const uint64_t t0 = global_timer_ns();
  for (int i = 0; i < px.world; ++i) {
    const volatile unsigned long long *f = &own->flag[slot][i];
    for (uint32_t spin = 1; *f != px.epoch; ++spin) {
      if ((spin & 255u) == 0u && global_timer_ns() - t0 > kExchangeLimitNs) {
        record_error(kErrWaitTimeout);
        return __longlong_as_double(0x7ff8000000000000ll);  // NaN
      }
    }
  }
  __threadfence_system();
  double sum = 0.0;
  for (int i = 0; i < px.world; ++i)
    sum += *reinterpret_cast<const volatile double *>(&own->partial[slot][i]);
  return sum;
}

// Last-block-done combine: block partials -> *out in index order (then, with
// px.world > 0, summed over the ranks); the ticket counter is reset so the
// scratch is ready for the next launch.
__device__ __forceinline__ void combine_partials(double block_total, double *partials,
                                                 unsigned int *ticket, double *out,
                                                 double *red, const PeerExchange &px) {
  __shared__ bool is_last;
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = block_total;
    __threadfence();
    const unsigned int done = atomicAdd(ticket, 1u);
    is_last = (done == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Fixed-order combine: thread t sums partials t, t+blockDim, ...; then the
  // block tree (fixed shape) adds those.
  double v = 0.0;
  for (unsigned int i = threadIdx.x; i < gridDim.x; i += blockDim.x)
    v += static_cast<volatile double *>(partials)[i];
  __syncthreads();
  const double total = block_sum_f64(v, red);
  if (threadIdx.x == 0) {
    *ticket = 0u;
    *out = px.world > 0 ? exchange_sum(total, px) : total;
  }
}

// sum(x) with optional fused vadd: when `b` is non-null, c = x + b is written
// and summed; otherwise x itself is summed (c unused).
template <bool kFused>
__global__ void __launch_bounds__(kStreamThreads)
sum_vec_kernel(const float4 *__restrict__ x, const float4 *__restrict__ b,
               float4 *__restrict__ c, int64_t n4, const float *__restrict__ xs,
               const float *__restrict__ bs, float *__restrict__ cs,
               int64_t n, double *partials, unsigned int *ticket,
               double *out, const PeerExchange px) {
  __shared__ double red[kStreamThreads / 32];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  double acc = 0.0;
  int64_t i = tid;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      v[u] = ld_stream(x + i + u * stride);
      if (kFused) v[u] = add4(v[u], ld_stream(b + i + u * stride));
    }
    float run = 0.0f;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (kFused) st_stream(c + i + u * stride, v[u]);
      run += hsum4(v[u]);
    }
    acc += static_cast<double>(run);
  }
  for (; i < n4; i += stride) {
    float4 v = ld_stream(x + i);
    if (kFused) {
      v = add4(v, ld_stream(b + i));
      st_stream(c + i, v);
    }
    acc += static_cast<double>(hsum4(v));
  }
  // Scalar tail (n not a multiple of 4): elements [4*n4, n).
  for (int64_t j = 4 * n4 + tid; j < n; j += stride) {
    float v = xs[j];
    if (kFused) {
      v = v + bs[j];
      cs[j] = v;
    }
    acc += static_cast<double>(v);
  }
  const double total = block_sum_f64(acc, red);
  __syncthreads();
  combine_partials(total, partials, ticket, out, red, px);
}

// Scalar-pointer form of sum for inputs that are not 16-byte aligned.
template <bool kFused>
__global__ void __launch_bounds__(kStreamThreads)
sum_scalar_kernel(const float *__restrict__ x, const float *__restrict__ b,
                  float *__restrict__ c, int64_t n, double *partials,
                  unsigned int *ticket, double *out, const PeerExchange px) {
  __shared__ double red[kStreamThreads / 32];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  double acc = 0.0;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n;
       j += stride) {
    float v = x[j];
    if (kFused) {
      v = v + b[j];
      c[j] = v;
    }
    acc += static_cast<double>(v);
  }
  const double total = block_sum_f64(acc, red);
  __syncthreads();
  combine_partials(total, partials, ticket, out, red, px);
}

// c = a + b (and, with kSum, sum(c)) through shared memory with 1-D bulk
// copies: one CTA per SM, a producer thread streams 8 KiB chunks of a and b
// into a 4-stage ring (cp.async.bulk, completion on an mbarrier), 8 consumer
// warps add them into a staging ring that one thread bulk-stores to c.
// Measured on B200 (2^30 floats): 6660 GB/s for c = a + b against 6274 for
// the float4 grid-stride kernel on the same box, 1.02 of the measured copy
// rate (6 stages or 16 KiB chunks measured 1-10 % slower, 2 or more CTAs per
// SM slower too). Chunks cover the first n - n % 2048 elements; the consumers add the
// rest with plain loads. Needs a, b, c 16-byte aligned. Summation: each
// consumer thread adds its 8 elements of a chunk in fp32 and folds that into
// an fp64 accumulator; fp64 block tree and last-block combine as
// sum_vec_kernel (deterministic for a given grid).
constexpr int kBulkChunk = 8192;                 // bytes per operand per stage
constexpr int kBulkStages = 4;
constexpr int kBulkConsumers = 256;              // 8 warps
constexpr int kBulkThreads = kBulkConsumers + 32;  // + the producer warp
constexpr size_t kBulkSmem = 3 * kBulkStages * kBulkChunk + 2 * kBulkStages * 8 + 128;

template <bool kSum>
__global__ void __launch_bounds__(kBulkThreads, 1)
stream_bulk_kernel(const float *__restrict__ a, const float *__restrict__ b,
                   float *__restrict__ c, int64_t n, double *partials, unsigned int *ticket,
                   double *out, const PeerExchange px) {
  extern __shared__ __align__(128) uint8_t bulk_smem[];
  __shared__ double red[kBulkThreads / 32];
  __shared__ int go;
  uint8_t *sa = bulk_smem, *sb = sa + kBulkStages * kBulkChunk, *sc = sb + kBulkStages * kBulkChunk;
  uint64_t *full = reinterpret_cast<uint64_t *>(sc + kBulkStages * kBulkChunk);
  uint64_t *empty = full + kBulkStages;
  constexpr int kFloats = kBulkChunk / 4;
  const int64_t nchunks = n / kFloats;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kBulkConsumers / 32);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double acc = 0.0;
  if (warp == kBulkConsumers / 32) {
    // ---- producer
    if (lane == 0) {
      int it = 0;
      for (int64_t ch = blockIdx.x; ch < nchunks; ch += gridDim.x, ++it) {
        const int s = it % kBulkStages;
        if (!mbar_wait(&empty[s], ((it / kBulkStages) & 1) ^ 1)) break;
        mbar_arrive_expect_tx(&full[s], 2 * kBulkChunk);
        bulk_load_1d(sa + s * kBulkChunk, a + ch * kFloats, kBulkChunk, &full[s]);
        bulk_load_1d(sb + s * kBulkChunk, b + ch * kFloats, kBulkChunk, &full[s]);
      }
    }
  } else {
    // ---- consumers (named barrier 1: the 256 consumer threads)
    const int t = threadIdx.x;
    int it = 0;
    for (int64_t ch = blockIdx.x; ch < nchunks; ch += gridDim.x, ++it) {
      const int s = it % kBulkStages;
      if (t == 0) {
        go = mbar_wait(&full[s], (it / kBulkStages) & 1) ? 1 : 0;
        // The store that last used staging slot s (kBulkStages chunks ago)
        // has read it.
        bulk_wait_group_read<kBulkStages - 1>();
      }
      named_bar_sync(1, kBulkConsumers);
      if (!go) break;
      const float4 *va = reinterpret_cast<const float4 *>(sa + s * kBulkChunk);
      const float4 *vb = reinterpret_cast<const float4 *>(sb + s * kBulkChunk);
      float4 *vc = reinterpret_cast<float4 *>(sc + s * kBulkChunk);
      float run = 0.0f;
#pragma unroll
      for (int q = 0; q < kBulkChunk / 16 / kBulkConsumers; ++q) {
        const int i = t + q * kBulkConsumers;
        const float4 v = add4(va[i], vb[i]);
        vc[i] = v;
        if (kSum) run += hsum4(v);
      }
      if (kSum) acc += static_cast<double>(run);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      named_bar_sync(1, kBulkConsumers);
      if (t == 0) {
        bulk_store_1d(c + ch * kFloats, sc + s * kBulkChunk, kBulkChunk);
        bulk_commit_group();
      }
    }
    // Elements past the last whole chunk.
    for (int64_t j = nchunks * kFloats + static_cast<int64_t>(blockIdx.x) * kBulkConsumers + t;
         j < n; j += static_cast<int64_t>(gridDim.x) * kBulkConsumers) {
      const float v = a[j] + b[j];
      c[j] = v;
      if (kSum) acc += static_cast<double>(v);
    }
    if (t == 0) bulk_wait_group<0>();
  }
  if (kSum) {
    const double total = block_sum_f64(acc, red);
    __syncthreads();
    combine_partials(total, partials, ticket, out, red, px);
  }
}

// Demo block reduce. The pairing follows the reference tree exactly: with
// s = block/2, block/4, ..., 1 (integer halving), slot t < s takes slot t + s.
// Levels with s > 16 go through shared memory; the last levels (every live
// slot then below 32) run as warp shuffles inside warp 0, which pair the same
// slots (lane t reads lane t + s, and slots >= s are never written at that
// level), so each partial is bit-identical to the reference for any block
// size, power of two or not.
//
// VC_CHECK_BOUNDS=1 forms of the demo kernels (debug aid): the same loops
// with every global access checked against the elements its buffer holds
// from the pointer on (the allocation registry's figure; INT64_MAX for memory
// the registry does not know). An index past its limit records
// kErrOutOfBounds in the error word and the access is skipped, so a wrong
// index ends the launch with a status the host reads instead of a fault.
struct AccessLimits {
  int64_t a, b, c;  // elements readable / writable from each pointer
};
__device__ __forceinline__ bool in_limit(int64_t i, int64_t limit) {
  if (i < limit) return true;
  record_error(kErrOutOfBounds);
  return false;
}

template <bool CHECK>
__global__ void block_reduce_demo_kernel(const float *__restrict__ in,
                                         float *__restrict__ out, int n,
                                         int block, AccessLimits lim) {
  extern __shared__ float slots[];
  const int t = threadIdx.x;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * block + t;
  slots[t] = (t < block && i < n && (!CHECK || in_limit(i, lim.a))) ? in[i] : 0.0f;
  __syncthreads();
  int s = block / 2;
  // Shared-memory levels until every slot that can still contribute
  // (index < 2s) lies inside warp 0, i.e. s <= 16.
  for (; s > 16; s /= 2) {
    if (t < s) slots[t] = slots[t] + slots[t + s];
    __syncthreads();
  }
  if (t < 32) {
    // Lanes >= block hold no slot; a lane t < s only reads lane t + s < 2s,
    // and 2s <= 32 here.
    float v = (t < block) ? slots[t] : 0.0f;
    for (; s > 0; s /= 2) {
      const float other = __shfl_down_sync(0xffffffffu, v, s);
      if (t < s) v = v + other;
    }
    if (t == 0 && (!CHECK || in_limit(blockIdx.x, lim.c))) out[blockIdx.x] = v;
  }
}

__global__ void fill_f64_kernel(double *p, double v) { *p = v; }

// a[i] = base + i for i < n (test/multigpu.vc:24-27, the multi-device demo's
// pattern fill), grid-stride.
template <bool CHECK>
__global__ void fill_pattern_kernel(int *__restrict__ a, int base, int64_t n, int64_t lim) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride)
    if (!CHECK || in_limit(i, lim)) a[i] = base + static_cast<int>(i);
}

// Bounds-checked vadd (scalar: a debug path, not a fast one).
__global__ void vadd_checked_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                    float *__restrict__ c, int64_t n, AccessLimits lim) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride)
    if (in_limit(i, lim.a) && in_limit(i, lim.b) && in_limit(i, lim.c)) c[i] = a[i] + b[i];
}

int resident_per_sm();

int stream_grid(int64_t work_items) {
  const int sm_count = sm_count_current();
  // One wave of resident 512-thread CTAs (the grid-stride loops then keep
  // every SM streaming to the end; a partial second wave measured 2-8 %
  // slower: 3 vs 4 CTAs per SM at 40 registers a thread); fewer CTAs when
  // the array is small.
  const int64_t full = static_cast<int64_t>(sm_count) * resident_per_sm();
  const int64_t need = (work_items + kStreamThreads - 1) / kStreamThreads;
  int64_t g = need < full ? need : full;
  return g < 1 ? 1 : static_cast<int>(g);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 512-thread CTAs of the streaming kernels that fit on one SM at once (the
// least over the vector kernels, which share one grid size), per device.
int resident_per_sm() {
  constexpr int kMaxDevices = 64;
  static int by_device[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 3;
  int *slot = (dev >= 0 && dev < kMaxDevices) ? &by_device[dev] : nullptr;
  int r = slot ? __atomic_load_n(slot, __ATOMIC_RELAXED) : 0;
  if (r <= 0) {
    r = 4;
    int k = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, vadd_vec_kernel, kStreamThreads, 0) ==
            cudaSuccess && k > 0)
      r = k < r ? k : r;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, sum_vec_kernel<true>, kStreamThreads,
                                                      0) == cudaSuccess && k > 0)
      r = k < r ? k : r;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, sum_vec_kernel<false>, kStreamThreads,
                                                      0) == cudaSuccess && k > 0)
      r = k < r ? k : r;
    cudaGetLastError();
    if (slot) __atomic_store_n(slot, r, __ATOMIC_RELAXED);
  }
  return r;
}

}  // namespace

int sm_count_current() {
  // One slot per device (the grid of every streaming launch depends on the
  // SM count of the device it runs on); filled on first use, racing threads
  // store the same value.
  constexpr int kMaxDevices = 64;
  static int by_device[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int *slot = (dev >= 0 && dev < kMaxDevices) ? &by_device[dev] : nullptr;
  int sms = slot ? __atomic_load_n(slot, __ATOMIC_RELAXED) : 0;
  if (sms <= 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0)
      return 148;
    if (slot) __atomic_store_n(slot, sms, __ATOMIC_RELAXED);
  }
  return sms;
}

int stream_max_blocks() { return sm_count_current() * 4; }

// The bulk-copy form serves aligned arrays from this many elements on (one
// CTA per SM; below it the grid-stride kernels, which measured faster at
// 2^24: vadd 30.2 against 34.9 us, the fused pair equal).
constexpr int64_t kBulkMinElems = int64_t(1) << 25;

// Grid of the bulk-copy kernels: one CTA per SM, no more than the chunks.
int bulk_grid(int64_t n, bool sum) {
  static std::mutex mu;
  static uint64_t configured[2] = {0, 0};  // devices whose smem attribute is set
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(configured[sum] & (1ull << dev))) {
      cudaError_t e = sum ? cudaFuncSetAttribute(stream_bulk_kernel<true>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kBulkSmem)
                          : cudaFuncSetAttribute(stream_bulk_kernel<false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kBulkSmem);
      if (e != cudaSuccess) return 0;
      if (dev < 64) configured[sum] |= (1ull << dev);
    }
  }
  const int64_t chunks = n / (kBulkChunk / 4);
  const int sms = sm_count_current();
  return (int)(chunks < sms ? (chunks > 0 ? chunks : 1) : sms);
}

cudaError_t launch_vadd_f32(const float *a, const float *b, float *c, int64_t n,
                            cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if (n >= kBulkMinElems && aligned16(a) && aligned16(b) && aligned16(c)) {
    const int grid = bulk_grid(n, false);
    if (grid > 0) {
      stream_bulk_kernel<false><<<grid, kBulkThreads, kBulkSmem, stream>>>(
          a, b, c, n, nullptr, nullptr, nullptr, PeerExchange{});
      return cudaGetLastError();
    }
  }
  if (aligned16(a) && aligned16(b) && aligned16(c)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      vadd_vec_kernel<<<stream_grid(n4 / kUnroll + 1), kStreamThreads, 0, stream>>>(
          reinterpret_cast<const float4 *>(a), reinterpret_cast<const float4 *>(b),
          reinterpret_cast<float4 *>(c), n4);
    }
    if (n % 4)
      vadd_scalar_kernel<<<1, 32, 0, stream>>>(a, b, c, n4 * 4, n);
  } else {
    vadd_scalar_kernel<<<stream_grid(n / kUnroll + 1), kStreamThreads, 0, stream>>>(
        a, b, c, 0, n);
  }
  return cudaGetLastError();
}

cudaError_t launch_sum_f32(const float *x, const float *b, float *c, int64_t n,
                           double *out, double *partials, unsigned int *ticket,
                           int max_blocks, cudaStream_t stream, const PeerExchange *pxp) {
  if (n < 0) return cudaErrorInvalidValue;
  PeerExchange px{};
  if (pxp != nullptr) {
    if (pxp->world < 1 || pxp->world > kMaxPeers || pxp->rank < 0 || pxp->rank >= pxp->world ||
        pxp->epoch == 0)
      return cudaErrorInvalidValue;
    for (int i = 0; i < pxp->world; ++i)
      if (pxp->mbox[i] == nullptr) return cudaErrorInvalidValue;
    px = *pxp;
  }
  const bool fused = (b != nullptr);
  const bool vec = aligned16(x) && (!fused || (aligned16(b) && aligned16(c)));
  const int64_t units = vec ? (n / 4) / kUnroll + 1 : n / kUnroll + 1;
  int grid = stream_grid(units);
  if (grid > max_blocks) grid = max_blocks;
  if (fused && vec && n >= kBulkMinElems) {
    int bgrid = bulk_grid(n, true);
    if (bgrid > max_blocks) bgrid = max_blocks;
    if (bgrid > 0) {
      stream_bulk_kernel<true><<<bgrid, kBulkThreads, kBulkSmem, stream>>>(
          x, b, c, n, partials, ticket, out, px);
      return cudaGetLastError();
    }
  }
  if (vec) {
    const int64_t n4 = n / 4;
    if (fused)
      sum_vec_kernel<true><<<grid, kStreamThreads, 0, stream>>>(
          reinterpret_cast<const float4 *>(x), reinterpret_cast<const float4 *>(b),
          reinterpret_cast<float4 *>(c), n4, x, b, c, n, partials, ticket, out, px);
    else
      sum_vec_kernel<false><<<grid, kStreamThreads, 0, stream>>>(
          reinterpret_cast<const float4 *>(x), nullptr, nullptr, n4, x, nullptr,
          nullptr, n, partials, ticket, out, px);
  } else {
    if (fused)
      sum_scalar_kernel<true><<<grid, kStreamThreads, 0, stream>>>(x, b, c, n, partials,
                                                                   ticket, out, px);
    else
      sum_scalar_kernel<false><<<grid, kStreamThreads, 0, stream>>>(
          x, nullptr, nullptr, n, partials, ticket, out, px);
  }
  return cudaGetLastError();
}

cudaError_t launch_fill_pattern(int *a, int base, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  fill_pattern_kernel<false><<<stream_grid(n / kUnroll + 1), kStreamThreads, 0, stream>>>(
      a, base, n, 0);
  return cudaGetLastError();
}

cudaError_t launch_fill_pattern_checked(int *a, int base, int64_t n, int64_t lim,
                                        cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  fill_pattern_kernel<true><<<stream_grid(n / kUnroll + 1), kStreamThreads, 0, stream>>>(
      a, base, n, lim);
  return cudaGetLastError();
}

cudaError_t launch_vadd_f32_checked(const float *a, const float *b, float *c, int64_t n,
                                    int64_t lim_a, int64_t lim_b, int64_t lim_c,
                                    cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  vadd_checked_kernel<<<stream_grid(n / kUnroll + 1), kStreamThreads, 0, stream>>>(
      a, b, c, n, AccessLimits{lim_a, lim_b, lim_c});
  return cudaGetLastError();
}

cudaError_t launch_block_reduce_demo(const float *in, float *out, int n, int block,
                                     int groups, cudaStream_t stream, int64_t lim_in,
                                     int64_t lim_out) {
  if (block <= 0 || block > 1024 || groups <= 0) return cudaErrorInvalidValue;
  // Threads: at least one warp so the shuffle levels have 32 lanes.
  const int threads = block < 32 ? 32 : ((block + 31) / 32) * 32;
  if (lim_in < 0)
    block_reduce_demo_kernel<false><<<groups, threads, threads * sizeof(float), stream>>>(
        in, out, n, block, AccessLimits{0, 0, 0});
  else
    block_reduce_demo_kernel<true><<<groups, threads, threads * sizeof(float), stream>>>(
        in, out, n, block, AccessLimits{lim_in, 0, lim_out});
  return cudaGetLastError();
}

// ------------------------------------------------------------------------
// Allocation-free sum: vc_sum_f32_noalloc.
//
// Some callers cannot allocate device memory at call time: a serving process
// that reserved its whole device budget at start-up and hands out no more, a
// latency-critical loop that must not enter the driver allocator (cudaMalloc
// can synchronise the device and takes a process-wide lock), or a host
// library calling in from a callback where a first-use allocation would be
// an unexpected side effect. vc_sum_f32 gets its block partials from a
// runtime-owned buffer that is cudaMalloc'd on first use per stream; this
// entry point instead keeps them in a fixed array compiled into the library.
//
// The array below exists once per GPU that loads the library and stays
// resident until the process exits. It holds kNoAllocMaxPartials block
// partials (8 KiB) plus the ticket counter, which bounds the grid to 1024
// blocks; the grid is the same one vc_sum_f32 uses (one wave of resident CTAs,
// 444 on a B200), so both entries add the same partials in the same order.
// A device that would need more blocks than that is refused with an error.
// Every call shares the array and it keeps the last call's contents: the
// ticket is cleared on the stream before each launch (the partial slots are
// written before they are read), and calls that overlap on the GPU (two
// streams at once) race on the array.
constexpr int kNoAllocMaxPartials = 1024;

struct NoAllocSumScratch {
  double partials[kNoAllocMaxPartials];
  unsigned int ticket;
};

static __device__ __align__(256) NoAllocSumScratch g_sum_noalloc_scratch;

// Device address of the array on the current device. In host code the
// symbol's name is a host-side stand-in, not a device address, so it is
// looked up once per device (that device current) and cached.
static cudaError_t noalloc_scratch_address(NoAllocSumScratch **out) {
  static std::mutex mu;
  static std::unordered_map<int, NoAllocSumScratch *> by_device;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  auto it = by_device.find(dev);
  if (it == by_device.end()) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sum_noalloc_scratch);
    if (e != cudaSuccess) return e;
    it = by_device.emplace(dev, static_cast<NoAllocSumScratch *>(p)).first;
  }
  *out = it->second;
  return cudaSuccess;
}

int noalloc_sum_capacity() { return kNoAllocMaxPartials; }

cudaError_t launch_sum_f32_noalloc(const float *x, int64_t n, double *out, cudaStream_t stream,
                                   int *blocks_needed) {
  if (n < 0) return cudaErrorInvalidValue;
  const bool vec = aligned16(x);
  const int64_t units = vec ? (n / 4) / kUnroll + 1 : n / kUnroll + 1;
  const int grid = stream_grid(units);
  if (blocks_needed) *blocks_needed = grid;
  if (grid > kNoAllocMaxPartials) return cudaErrorInvalidValue;
  NoAllocSumScratch *scratch = nullptr;
  cudaError_t e = noalloc_scratch_address(&scratch);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(&scratch->ticket, 0, sizeof(unsigned int), stream);
  if (e != cudaSuccess) return e;
  return launch_sum_f32(x, nullptr, nullptr, n, out, scratch->partials, &scratch->ticket,
                        kNoAllocMaxPartials, stream);
}

}  // namespace vcb

VCB_DEFINE_ERROR_ACCESSOR(stream_kernels_error)
