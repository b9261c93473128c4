//===- VCRuntime.h - VC runtime API, CUDA/B200 implementation -------------===//
//
// Drop-in replacement for the VC runtime header
// (include/vc/Runtime/VCRuntime.h in junka/vkcuda). Host programs written
// against that header -- including the host C++ the VC compiler generates
// for `kernel<<<grid, block>>>(args)` (lib/Codegen/ASTToHost.cpp:1197-1320) --
// compile and link against libVCRuntime built from this tree unchanged.
//
// Every declaration keeps the reference's name, parameter list, enum order and
// struct layout, because callers are compiled separately and bind by C++
// mangled name and by byte layout. The implementation underneath is the CUDA
// runtime on NVIDIA B200 (sm_100a) instead of Vulkan:
//   * device pointers returned by vcMalloc are real device addresses;
//   * streams are CUDA streams, events are CUDA events;
//   * kernels are looked up by entry name in a registry of hand-written
//     sm_100a kernels (flashAttn, wmma_gemm, matmulCoopmat, matmulTiled, vadd,
//     blockReduce) plus native entries with explicit shapes ("vc.gemm",
//     "vc.flash_fwd", "vc.vadd", "vc.sum", "vc.vadd_sum");
//   * storage images and the Vulkan SC offline-pipeline API are not provided
//     (they return InvalidValue).
//
// Launch grids keep the reference meaning: gridDim/blockDim are ELEMENT
// counts and the workgroup count is ceil(grid / block) per axis.
//
//===----------------------------------------------------------------------===//

#ifndef VC_RUNTIME_VCRUNTIME_H
#define VC_RUNTIME_VCRUNTIME_H

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace vc {

// Opaque handles. NULL stream = the current device's default stream.
struct VCBuffer;
using VCBufferHandle = VCBuffer *;
struct VCKernel;
using VCKernelHandle = VCKernel *;
struct VCStream;
using VCStreamHandle = VCStream *;
struct VCImage;
using VCImageHandle = VCImage *;
struct VCGraph;
using VCGraphHandle = VCGraph *;
struct VCEvent;
using VCEventHandle = VCEvent *;

// Error codes; numeric values are part of the ABI (reference VCRuntime.h:64-74).
enum class VCError {
  Success = 0,
  InvalidValue,
  OutOfMemory,
  InvalidKernel,
  InvalidDevice,
  InitializationError,
  MapFailed,
  NotReady,
  Unknown,
};

// Copy direction (reference VCRuntime.h:77-81).
enum class VCMemcpyKind {
  HostToDevice,
  DeviceToHost,
  DeviceToDevice,
};

// Storage-image pixel formats (reference VCRuntime.h:83-122). Declared so that
// code naming them still compiles; images themselves are not supported here.
enum class VCPixelFormat {
  R32G32B32A32Float,
  R16G16B16A16Float,
  R32G32B32A32Sint,
  R32Sint,
  R32Uint,
  R16Float,
  Rg16Float,
  R11G11B10Float,
  Rgba8Unorm,
  R16Sint,
  Rg16Sint,
  R32Float,
  Rg32Float,
  R8Unorm,
  Rg8Unorm,
  Rgba8Snorm,
  Rgba16Sint,
  Rgba8Sint,
  R8Sint,
  R32G32B32A32Uint,
  Rgba16Uint,
  Rgba8Uint,
  R8Uint,
};

// Initialise the runtime: enumerate CUDA devices, select device 0.
// Repeated calls return Success.
VCError vcInit();

// Synchronise every device, release runtime-owned resources and print the
// VC_PROFILE summary table when profiling is on.
VCError vcShutdown();

// Number of CUDA devices. Initialises lazily; a failed initialisation reports
// a count of 0 with Success (the reference behaviour).
VCError vcGetDeviceCount(int *count);

// Current device index (per host thread).
VCError vcGetDevice(int *device);

// Select the current device; InvalidDevice when out of range.
VCError vcSetDevice(int device);

// Subset of cudaDeviceProp; layout identical to the reference struct.
struct VCDeviceProperties {
  char name[256];
  size_t totalGlobalMem;
  size_t sharedMemPerBlock;
  size_t sharedMemPerMultiprocessor;
  int warpSize;
  int maxThreadsPerBlock;
  int maxThreadsDim[3];
  int maxGridSize[3];
  int clockRate;           // kHz (real value on CUDA)
  int multiProcessorCount; // SM count (148 on B200)
  int major;               // compute capability major
  int minor;               // compute capability minor
};

VCError vcGetDeviceProperties(VCDeviceProperties *out, int device);

// Block size that maximises occupancy for `kernel` (cudaOccupancy* on the
// registry kernel backing the handle).
VCError vcOccupancyMaxPotentialBlockSize(int *minGridSize, int *blockSize,
                                         VCKernelHandle kernel,
                                         size_t dynamicSharedMemPerBlock,
                                         int blockSizeLimit);

// Device printf is native in CUDA; this only records the flag. Must precede
// vcInit (InvalidValue afterwards, as in the reference).
VCError vcEnableKernelPrintf(int enable);

enum class VCMemoryType {
  Unregistered,
  Device,
  Host,
  Managed,
};

struct VCPointerAttributes {
  VCMemoryType memoryType = VCMemoryType::Unregistered;
  void *devicePointer = nullptr;
  void *hostPointer = nullptr;
  size_t size = 0;
};

// Attributes of any address inside a VC allocation (base + offset allowed);
// Unregistered for everything else.
VCError vcPointerGetAttributes(VCPointerAttributes *out, const void *ptr);

VCError vcMalloc(void **devPtr, size_t bytes);
VCError vcMallocHost(void **hostPtr, size_t bytes);
VCError vcMallocManaged(void **devPtr, size_t bytes);
VCError vcMallocManagedS(void **devPtr, size_t bytes, VCStreamHandle stream);
VCError vcFree(void *devPtr);
VCError vcMallocAsync(void **devPtr, size_t bytes, VCStreamHandle stream);
VCError vcMallocHostAsync(void **hostPtr, size_t bytes, VCStreamHandle stream);
VCError vcFreeAsync(void *devPtr, VCStreamHandle stream);

// Storage images: not supported on this runtime (InvalidValue).
VCError vcCreateImage2D(VCImageHandle *out, uint32_t width, uint32_t height,
                        VCPixelFormat fmt);
VCError vcCreateImage1D(VCImageHandle *out, uint32_t width,
                        VCPixelFormat fmt);
VCError vcCreateImage3D(VCImageHandle *out, uint32_t width, uint32_t height,
                        uint32_t depth, VCPixelFormat fmt);
VCError vcCreateImage2DArray(VCImageHandle *out, uint32_t width,
                             uint32_t height, uint32_t layers,
                             VCPixelFormat fmt);
VCError vcDestroyImage(VCImageHandle img);
VCError vcMemcpyToImage(VCImageHandle img, const void *hostData);
VCError vcMemcpyFromImage(void *hostData, VCImageHandle img);

// Copies. H2D and D2H block; D2D is asynchronous on the stream.
VCError vcMemcpy(void *dst, const void *src, size_t count, VCMemcpyKind kind);
VCError vcMemcpyS(void *dst, const void *src, size_t count, VCMemcpyKind kind,
                  VCStreamHandle stream);
// Asynchronous copy. H2D from pageable memory is staged before return, so the
// caller may reuse `src`; H2D from vcMallocHost memory is a direct DMA and
// `src` must stay untouched until the stream passes the copy. D2H needs a
// stream synchronisation before `dst` is read.
VCError vcMemcpyAsyncS(void *dst, const void *src, size_t count,
                       VCMemcpyKind kind, VCStreamHandle stream);
VCError vcMemcpyAsync(void *dst, const void *src, size_t count,
                      VCMemcpyKind kind);

// Peer copies over NVLink (cudaMemcpyPeer[Async]); the async form is truly
// stream-ordered. `stream` must belong to dstDevice.
VCError vcMemcpyPeer(void *dst, int dstDevice, const void *src, int srcDevice,
                     size_t bytes);
VCError vcMemcpyPeerAsync(void *dst, int dstDevice, const void *src,
                          int srcDevice, size_t bytes,
                          VCStreamHandle stream);

// Byte fills; `count` must be a multiple of 4 (reference contract).
VCError vcMemset(void *devPtr, int value, size_t count);
VCError vcMemsetS(void *devPtr, int value, size_t count, VCStreamHandle stream);
VCError vcMemsetAsyncS(void *devPtr, int value, size_t count,
                       VCStreamHandle stream);
VCError vcMemsetAsync(void *devPtr, int value, size_t count);

// 2D pitched copies and fills (DeviceToDevice only, as in the reference).
VCError vcMemcpy2D(void *dst, size_t dpitch, const void *src, size_t spitch,
                   size_t width, size_t height, VCMemcpyKind kind);
VCError vcMemcpy2DS(void *dst, size_t dpitch, const void *src, size_t spitch,
                    size_t width, size_t height, VCMemcpyKind kind,
                    VCStreamHandle stream);
VCError vcMemcpy2DAsync(void *dst, size_t dpitch, const void *src, size_t spitch,
                        size_t width, size_t height, VCMemcpyKind kind,
                        VCStreamHandle stream);
VCError vcMemset2D(void *dst, size_t pitch, int value, size_t width,
                   size_t height);
VCError vcMemset2DAsync(void *dst, size_t pitch, int value, size_t width,
                        size_t height, VCStreamHandle stream);

// Synchronisation. Waits are bounded by VC_SYNC_TIMEOUT_MS when set (NotReady
// is returned when the deadline passes; the work keeps running).
VCError vcDeviceSynchronize();
VCError vcStreamCreate(VCStreamHandle *out);
VCError vcStreamDestroy(VCStreamHandle stream);
VCError vcStreamSynchronize(VCStreamHandle stream);
VCError vcStreamQuery(VCStreamHandle stream, int *done);

using VCHostFn = void (*)(void *userData);
VCError vcLaunchHostFunc(VCStreamHandle stream, VCHostFn fn, void *userData);

// Events (CUDA events with timing).
VCError vcEventCreate(VCEventHandle *out);
VCError vcEventDestroy(VCEventHandle event);
VCError vcEventRecord(VCEventHandle event, VCStreamHandle stream);
VCError vcStreamWaitEvent(VCStreamHandle stream, VCEventHandle event);
VCError vcEventQuery(VCEventHandle event, int *done);
VCError vcEventSynchronize(VCEventHandle event);
// InvalidValue when either event was never recorded.
VCError vcEventElapsedTime(float *ms, VCEventHandle start, VCEventHandle end);

// Graphs: recording captures the default stream of the current device into a
// CUDA graph; launch replays the instantiated graph.
VCError vcGraphCreate(VCGraphHandle *out);
VCError vcGraphDestroy(VCGraphHandle graph);
VCError vcGraphBeginRecord(VCGraphHandle graph);
VCError vcGraphEndRecord(VCGraphHandle graph);
VCError vcGraphLaunch(VCGraphHandle graph, VCStreamHandle stream);
VCError vcGraphReset(VCGraphHandle graph);

// Kernel loading. The module words are checked for the SPIR-V magic when
// given (nullptr/0 is accepted and means "look up by name only"); the kernel
// is resolved by `entryPoint` in the registry. InvalidKernel for unknown
// entries (with a stderr line naming the entry).
VCError vcLoadKernel(const uint32_t *spirvWords, size_t wordCount,
                     const char *entryPoint, VCKernelHandle *outKernel);
VCError vcLoadKernelFromFile(const char *path, const char *entryPoint,
                             VCKernelHandle *outKernel);
VCError vcReleaseKernel(VCKernelHandle kernel);

struct VCKernelArg {
  enum Kind { Pointer, Scalar, Image } kind = Pointer;
  const void *data = nullptr;
  size_t size = 0;
};

VCError vcLaunchKernel(VCKernelHandle kernel, unsigned gridDim,
                       unsigned blockDim, const VCKernelArg *args,
                       int argCount);
VCError vcLaunchKernel2D(VCKernelHandle kernel, unsigned gridDimX,
                         unsigned gridDimY, unsigned blockDimX,
                         unsigned blockDimY, const VCKernelArg *args,
                         int argCount);
VCError vcLaunchKernelS(VCKernelHandle kernel, unsigned gridDim,
                        unsigned blockDim, const VCKernelArg *args,
                        int argCount, VCStreamHandle stream);
VCError vcLaunchKernel2DS(VCKernelHandle kernel, unsigned gridDimX,
                          unsigned gridDimY, unsigned blockDimX,
                          unsigned blockDimY, const VCKernelArg *args,
                          int argCount, VCStreamHandle stream);
// Indirect launch: the three uint32 workgroup counts are read from the device
// buffer at `offset` (one small D2H read on the stream) before the launch.
VCError vcLaunchKernelIndirectS(VCKernelHandle kernel, void *indirectArgs,
                                size_t offset, unsigned blockX,
                                unsigned blockY, unsigned blockZ,
                                const VCKernelArg *args, int argCount,
                                VCStreamHandle stream);
VCError vcLaunchKernelIndirect(VCKernelHandle kernel, void *indirectArgs,
                               size_t offset, unsigned blockX,
                               unsigned blockY, unsigned blockZ,
                               const VCKernelArg *args, int argCount);

const char *vcErrorString(VCError err);

//----------------------------------------------------------------------------
// Extensions (no counterpart in the reference header).
//----------------------------------------------------------------------------

// Resolve a registry kernel by name without a module.
VCError vcGetKernel(const char *name, VCKernelHandle *outKernel);

// Override one of the compile-time constants a legacy demo kernel bakes in
// (flashAttn: NHEAD, SEQ, HDIM, BR, BC; matmulCoopmat: L). The reference
// fixes these with #define in the .vc source, so they are not launch args.
VCError vcKernelSetConstant(VCKernelHandle kernel, const char *name,
                            long long value);

} // namespace vc

#endif // VC_RUNTIME_VCRUNTIME_H
