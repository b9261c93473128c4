/*===- vc_b200.h - flat C ABI of libVCRuntime (B200 build) -----------------===
 *
 * Plain-C entry points exported by vkcuda_b200/lib/libVCRuntime.so. They are
 * what a foreign-function caller (Python ctypes, a cgo or JNI stub) binds:
 * `extern "C"`, plain pointers and sizes, no C++ or torch types.
 *
 * Two groups:
 *  1. vc_* mirrors of the reference runtime API, one per vc:: function of
 *     include/vc/Runtime/VCRuntime.h in junka/vkcuda (line numbers cited on
 *     each). Return values are the VCError codes of that header as int.
 *  2. Native hot-path entries with explicit shapes: vadd, sum-reduce, the
 *     fused pair, the demo block reduce, GEMM and the flash-attention forward.
 *     They replace the bodies of the demo kernels named on each
 *     (examples/flash_attn.vc, test/wmma_gemm.vc,
 *     examples/matmul_coopmat_bench.vc, test/vadd.vc, test/reduce.vc).
 *
 * Pointers passed to kernels are device addresses (vc_malloc, cudaMalloc or a
 * torch tensor's data_ptr). `stream` is a CUDA stream handle (cudaStream_t);
 * NULL means the current device's legacy default stream. A VCStreamHandle
 * from vc_stream_create is the same kind of value.
 *===----------------------------------------------------------------------===*/
#ifndef VC_B200_H
#define VC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* VCError values (reference VCRuntime.h:64-74). */
enum {
  VC_SUCCESS = 0,
  VC_INVALID_VALUE = 1,
  VC_OUT_OF_MEMORY = 2,
  VC_INVALID_KERNEL = 3,
  VC_INVALID_DEVICE = 4,
  VC_INITIALIZATION_ERROR = 5,
  VC_MAP_FAILED = 6,
  VC_NOT_READY = 7,
  VC_UNKNOWN = 8
};

/* VCMemcpyKind values (reference VCRuntime.h:77-81). */
enum { VC_H2D = 0, VC_D2H = 1, VC_D2D = 2 };

/* Element types of the native entries. */
enum { VC_DTYPE_F32 = 0, VC_DTYPE_F16 = 1, VC_DTYPE_BF16 = 2 };

/* Byte-compatible with vc::VCDeviceProperties (reference VCRuntime.h:255-268). */
typedef struct vc_device_properties {
  char name[256];
  size_t totalGlobalMem;
  size_t sharedMemPerBlock;
  size_t sharedMemPerMultiprocessor;
  int warpSize;
  int maxThreadsPerBlock;
  int maxThreadsDim[3];
  int maxGridSize[3];
  int clockRate;
  int multiProcessorCount;
  int major;
  int minor;
} vc_device_properties;

/* Byte-compatible with vc::VCPointerAttributes (reference VCRuntime.h:321-326). */
typedef struct vc_pointer_attributes {
  int memoryType; /* 0 Unregistered, 1 Device, 2 Host, 3 Managed */
  void *devicePointer;
  void *hostPointer;
  size_t size;
} vc_pointer_attributes;

/* Byte-compatible with vc::VCKernelArg (reference VCRuntime.h:690-694). */
typedef struct vc_kernel_arg {
  int kind; /* 0 Pointer, 1 Scalar, 2 Image */
  const void *data;
  size_t size;
} vc_kernel_arg;

/* ---- 1. runtime API mirrors ------------------------------------------- */
int vc_init(void);                                   /* vcInit  VCRuntime.h:126 */
int vc_shutdown(void);                               /* vcShutdown  :129 */
int vc_get_device_count(int *count);                 /* vcGetDeviceCount  :239 */
int vc_get_device(int *device);                      /* vcGetDevice  :244 */
int vc_set_device(int device);                       /* vcSetDevice  :249 */
int vc_get_device_properties(vc_device_properties *out, int device); /* :272 */
int vc_occupancy_max_potential_block_size(int *minGridSize, int *blockSize,
                                          void *kernel, size_t dynSmem,
                                          int blockSizeLimit); /* :289-293 */
int vc_pointer_get_attributes(vc_pointer_attributes *out, const void *ptr); /* :331 */
int vc_malloc(void **devPtr, size_t bytes);          /* vcMalloc  :335 */
int vc_malloc_host(void **hostPtr, size_t bytes);    /* vcMallocHost  :339 */
int vc_malloc_managed(void **devPtr, size_t bytes);  /* vcMallocManaged  :354 */
int vc_free(void *ptr);                              /* vcFree  :362 */
int vc_malloc_async(void **devPtr, size_t bytes, void *stream); /* :369 */
int vc_free_async(void *ptr, void *stream);          /* vcFreeAsync  :381 */
int vc_memcpy(void *dst, const void *src, size_t count, int kind);      /* :426 */
int vc_memcpy_s(void *dst, const void *src, size_t count, int kind,
                void *stream);                                          /* :429 */
int vc_memcpy_async_s(void *dst, const void *src, size_t count, int kind,
                      void *stream);                                    /* :443 */
int vc_memcpy_async(void *dst, const void *src, size_t count, int kind); /* :447 */
int vc_memcpy_peer(void *dst, int dstDevice, const void *src, int srcDevice,
                   size_t bytes);                                       /* :457 */
int vc_memcpy_peer_async(void *dst, int dstDevice, const void *src,
                         int srcDevice, size_t bytes, void *stream);    /* :465 */
int vc_memset(void *ptr, int value, size_t count);   /* vcMemset  :474 */
int vc_memset_async_s(void *ptr, int value, size_t count, void *stream); /* :482 */
int vc_memcpy_2d_async(void *dst, size_t dpitch, const void *src,
                       size_t spitch, size_t width, size_t height, int kind,
                       void *stream);                                   /* :502 */
int vc_memset_2d_async(void *dst, size_t pitch, int value, size_t width,
                       size_t height, void *stream);                    /* :514 */
int vc_device_synchronize(void);                     /* :518 */
int vc_stream_create(void **out);                    /* vcStreamCreate  :521 */
int vc_stream_destroy(void *stream);                 /* :524 */
int vc_stream_synchronize(void *stream);             /* :527 */
int vc_stream_query(void *stream, int *done);        /* :532 */
int vc_launch_host_func(void *stream, void (*fn)(void *), void *userData); /* :542 */
int vc_event_create(void **out);                     /* vcEventCreate  :551 */
int vc_event_destroy(void *event);                   /* :554 */
int vc_event_record(void *event, void *stream);      /* :561 */
int vc_stream_wait_event(void *stream, void *event); /* :568 */
int vc_event_query(void *event, int *done);          /* :572 */
int vc_event_synchronize(void *event);               /* :575 */
int vc_event_elapsed_time(float *ms, void *start, void *end); /* :586 */
int vc_graph_create(void **out);                     /* vcGraphCreate  :596 */
int vc_graph_destroy(void *graph);                   /* :601 */
int vc_graph_begin_record(void *graph);              /* :608 */
int vc_graph_end_record(void *graph);                /* :612 */
int vc_graph_launch(void *graph, void *stream);      /* :616 */
int vc_graph_reset(void *graph);                     /* :621 */
int vc_load_kernel(const uint32_t *words, size_t wordCount,
                   const char *entryPoint, void **outKernel);           /* :625 */
int vc_load_kernel_from_file(const char *path, const char *entryPoint,
                             void **outKernel);                         /* :629 */
int vc_release_kernel(void *kernel);                 /* vcReleaseKernel  :685 */
int vc_launch_kernel(void *kernel, unsigned gridDim, unsigned blockDim,
                     const vc_kernel_arg *args, int argCount);          /* :699 */
int vc_launch_kernel_s(void *kernel, unsigned gridDim, unsigned blockDim,
                       const vc_kernel_arg *args, int argCount,
                       void *stream);                                   /* :712 */
int vc_launch_kernel_2d_s(void *kernel, unsigned gridX, unsigned gridY,
                          unsigned blockX, unsigned blockY,
                          const vc_kernel_arg *args, int argCount,
                          void *stream);                                /* :717 */
int vc_launch_kernel_indirect_s(void *kernel, void *indirectArgs, size_t offset,
                                unsigned blockX, unsigned blockY, unsigned blockZ,
                                const vc_kernel_arg *args, int argCount,
                                void *stream);                          /* :730 */
const char *vc_error_string(int err);                /* vcErrorString  :743 */

/* Extensions of the runtime API (no reference counterpart). */
int vc_get_kernel(const char *name, void **outKernel);
int vc_kernel_set_constant(void *kernel, const char *name, long long value);
/* Sticky device-side error word of the hot kernels (bounded waits that ran
 * out, bad launch shapes): 0 when clean. `clear` resets it. */
int vc_kernel_error(int clear);
/* Launch a kernel whose single thread waits on an mbarrier that nothing
 * arrives on, bounded to `timeout_us`; returns the error word it set. Used to
 * test the bounded-wait path without hanging a GPU. */
int vc_selftest_bounded_wait(unsigned timeout_us);
/* Run the bounds-checked vadd (the form VC_CHECK_BOUNDS=1 selects) over 1024
 * elements of real memory, telling it the output holds 1000: returns the
 * error word it set (4, out of bounds, when the check refused indices
 * 1000..1023 and wrote the rest), 100 when the output is not as expected, -1
 * on a CUDA error. */
int vc_selftest_bounds_check(void);

/* ---- 2. native hot-path entries --------------------------------------- */

/* c[i] = a[i] + b[i], i < n. Replaces vadd (test/vadd.vc:12-17). */
int vc_vadd_f32(const float *a, const float *b, float *c, int64_t n,
                void *stream);

/* *out = sum of x[0..n) (device double). fp32 per-thread runs, fp64 block
 * and final combine, deterministic order. Scratch: runtime-owned per-device
 * partials buffer. Replaces the sum of test/reduce.vc scaled to one scalar. */
int vc_sum_f32(const float *x, int64_t n, double *out, void *stream);

/* No counterpart in the reference. Same result as vc_sum_f32 (same kernel,
 * grid and summation order) for callers that cannot allocate device memory at
 * call time (a process whose device budget is fully reserved up front, a
 * latency-critical loop that must stay out of the driver allocator, a
 * library callback that must not allocate as a side effect). Allocates
 * nothing: its block partials live in a fixed 8 KiB array compiled into the
 * library (1024 partial slots; a device that would need more blocks is
 * refused with VC_INVALID_VALUE). All calls share that array: calls that
 * overlap on the GPU race. The first call on a device looks up the array's
 * address; make it before any stream capture. Runs on the runtime's current
 * device (vc_set_device), as vc_sum_f32 does. */
int vc_sum_f32_noalloc(const float *x, int64_t n, double *out, void *stream);

/* Fused: c = a + b and *out = sum(c) in one pass (12 bytes per element). */
int vc_vadd_sum_f32(const float *a, const float *b, float *c, int64_t n,
                    double *out, void *stream);

/* ---- Cross-GPU sum without a library collective (one process per GPU).
 * The reference's reduce is single-device (test/reduce.vc); its multi-GPU
 * form here combines the per-GPU partials, which a library all-reduce would
 * otherwise do after the kernel, inside the sum kernel itself over NVLink:
 * each rank allocates one mailbox (vc_peer_mailbox_alloc), exports it
 * (vc_peer_ipc_get_handle), imports every other rank's
 * (vc_peer_ipc_open, handles exchanged by any host channel), and passes
 * all `world` mailbox addresses, in rank order with its own at `rank`, to
 * vc_vadd_sum_f32_allreduce. That kernel writes c = a + b, and *out = the
 * sum over all ranks of sum(c): its last block stores this GPU's sum into
 * every mailbox with peer stores, then waits for the other ranks' (bounded:
 * after 2 s it gives NaN and records a timeout, see vc_kernel_error). Every
 * rank must make the same sequence of calls with the same increasing
 * `epoch` (>= 1), one per call. world <= 8. */
#define VC_IPC_HANDLE_BYTES 64
int vc_peer_mailbox_alloc(void **mailbox);
int vc_peer_mailbox_free(void *mailbox);
int vc_peer_ipc_get_handle(const void *dev_ptr, void *handle /* VC_IPC_HANDLE_BYTES */);
int vc_peer_ipc_open(const void *handle, void **dev_ptr);
int vc_peer_ipc_close(void *dev_ptr);
int vc_vadd_sum_f32_allreduce(const float *a, const float *b, float *c, int64_t n,
                              double *out, void *const *mailboxes, int rank, int world,
                              unsigned long long epoch, void *stream);

/* Demo block reduce: out[g] = tree sum of in[g*block .. g*block+block) with
 * the reference's pairing order (test/reduce.vc:11-38), for g < groups. */
int vc_block_reduce_f32(const float *in, float *out, int n, int block,
                        int groups, void *stream);

/* D[M][N] (fp32, row stride ldd) = A[M][K] * B + Cin (Cin optional, fp32,
 * row stride ldc). A is row-major (stride lda). b_kn = 1: B is [K][N]
 * row-major (stride ldb, the demos' layout); b_kn = 0: B is [N][K]
 * row-major. dtype VC_DTYPE_F16 or VC_DTYPE_BF16, fp32 accumulate.
 * Replaces wmma_gemm (test/wmma_gemm.vc:19-33) and matmulCoopmat
 * (examples/matmul_coopmat_bench.vc:60-110).
 * dtype VC_DTYPE_F32: A and B are fp32, computed on the tensor cores from a
 * hi/lo split of each operand (hi*hi in tf32, the two correction products in
 * bf16; at most ~2^-17 relative per product, rounded to nearest); replaces
 * matmulTiled (examples/matmul_bench.vc:22-54).
 * Cin may be D itself (in place, ldc == ldd); it must not otherwise overlap
 * D, since one tile's stores may land on another tile's addend. */
int vc_gemm(const void *A, const void *B, float *D, const float *Cin, int M,
            int N, int K, int64_t lda, int64_t ldb, int64_t ldd, int64_t ldc,
            int dtype, int b_kn, void *stream);

/* Flash-attention forward over BH independent [N][d] slices:
 * O = softmax_2(scale_log2 * Q K^T) V, where softmax_2 exponentiates in base
 * 2 (scale_log2 = log2(e)/sqrt(d) gives the ordinary softmax(QK^T/sqrt(d))).
 * causal != 0 masks key j > query i. dtype F32 (SIMT path, d <= 256),
 * F16 or BF16 (tcgen05 path, d in {64, 128}); O has the input dtype.
 * Replaces flashAttn (examples/flash_attn.vc:56-126). */
int vc_flash_fwd(const void *Q, const void *K, const void *V, void *O, int BH,
                 int N, int d, float scale_log2, int causal, int dtype,
                 void *stream);

#ifdef __cplusplus
}
#endif

#endif /* VC_B200_H */
