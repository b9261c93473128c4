// runtime.cpp - the VC runtime API (include/vc/Runtime/VCRuntime.h) on the
// CUDA runtime, replacing the Vulkan implementation of the reference
// (lib/Runtime/VCRuntime.cpp; API wrappers at :5023-5644).
//
// What maps to what:
//   vcMalloc / vcMallocHost / vcMallocManaged -> cudaMalloc / cudaMallocHost /
//     cudaMallocManaged, recorded in an allocation registry (base -> kind,
//     size, device) that serves vcPointerGetAttributes and bounds checks.
//   streams -> non-blocking CUDA streams; NULL -> legacy default stream of the
//     current device (or the capture stream while a graph records).
//   events -> CUDA events with timing, plus a "recorded" flag so that
//     vcEventElapsedTime reports InvalidValue for a never-recorded event, as
//     the reference does.
//   graphs -> CUDA stream capture of the default stream; H2D copies made
//     while recording are snapshotted into graph-owned pinned staging.
//   kernels -> a registry of hand-written sm_100a kernels keyed by entry
//     name (the reference keys SPIR-V modules by entry point,
//     VCRuntime.cpp:4255-4282).
//   vcLaunchHostFunc -> cudaLaunchHostFunc with a trampoline onto a runtime
//     worker thread, so the callback may call back into the runtime as the
//     reference allows (VCRuntime.h:536-542).
// Environment: VC_PROFILE=1 (per-op GPU timings, table at vcShutdown),
// VC_DEBUG=1 (diagnostics), VC_POISON=1 (outputs filled with NaN canaries
// before each registry launch), VC_SYNC_TIMEOUT_MS=<ms> (bounded host waits that
// return NotReady), VC_FAULT_INJECT=malloc:N,launch:N,memcpy:N (the Nth call
// of that kind fails, for host-side failure tests).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <fstream>
#include <initializer_list>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/vc/Runtime/VCRuntime.h"
#include "../../include/vc_b200.h"
#include "internal.h"

namespace vc {

// Handle structs (opaque in the public header).
struct VCEvent {
  cudaEvent_t ev = nullptr;
  int device = 0;
  bool recorded = false;
};

struct VCGraph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaStream_t capture = nullptr;
  int device = 0;
  bool recording = false;
  std::vector<void *> staging;  // pinned snapshots of H2D sources
};

struct KernelEntry;
struct VCKernel {
  const KernelEntry *entry = nullptr;
  std::map<std::string, long long> constants;
};

}  // namespace vc

using namespace vc;

namespace {

// ------------------------------------------------------------------ state
struct AllocInfo {
  VCMemoryType kind;
  size_t size;
  int device;
};

struct ProfileAgg {
  long calls = 0;
  double total_ms = 0.0;
  double max_ms = 0.0;
};

struct PendingSpan {
  std::string name;
  cudaEvent_t a, b;
  int device;
};

struct DeferredFree {
  void *ptr;
  cudaEvent_t ev;
  int device;
};

struct Scratch {
  double *partials = nullptr;
  unsigned int *ticket = nullptr;
  int capacity = 0;
};

struct State {
  std::mutex mu;
  bool initialized = false;
  int device_count = 0;
  bool printf_flag = false;
  bool profile = false;
  bool debug = false;
  bool poison = false;  // VC_POISON=1: NaN canaries in outputs before launches
  bool check_bounds = false;  // VC_CHECK_BOUNDS=1: device-side index checks
  long sync_timeout_ms = 0;
  std::map<uintptr_t, AllocInfo> allocs;
  std::unordered_map<void *, int> stream_device;
  std::map<int, VCGraph *> recording;  // device -> graph being recorded
  std::vector<PendingSpan> spans;
  std::map<std::string, ProfileAgg> profile_table;
  std::vector<DeferredFree> deferred;
  std::map<std::pair<int, void *>, Scratch> scratch;
  std::unordered_map<std::string, int> fault_at;     // kind -> Nth call fails
  std::unordered_map<std::string, int> fault_count;  // kind -> calls so far
  bool fault_parsed = false;
};

State &st() {
  static State *s = new State();  // never destroyed: safe during exit
  return *s;
}

thread_local int t_device = 0;

void parse_faults_locked(State &s) {
  if (s.fault_parsed) return;
  s.fault_parsed = true;
  const char *env = std::getenv("VC_FAULT_INJECT");
  if (!env) return;
  std::string spec(env);
  size_t pos = 0;
  while (pos < spec.size()) {
    size_t end = spec.find(',', pos);
    if (end == std::string::npos) end = spec.size();
    std::string item = spec.substr(pos, end - pos);
    size_t colon = item.find(':');
    if (colon != std::string::npos) {
      int n = std::atoi(item.c_str() + colon + 1);
      if (n > 0) s.fault_at[item.substr(0, colon)] = n;
    }
    pos = end + 1;
  }
}

// True when this call of `kind` is the one VC_FAULT_INJECT asks to fail.
bool inject_fault(const char *kind) {
  State &s = st();
  std::lock_guard<std::mutex> lk(s.mu);
  parse_faults_locked(s);
  auto it = s.fault_at.find(kind);
  if (it == s.fault_at.end()) return false;
  int n = ++s.fault_count[kind];
  if (n == it->second) {
    std::fprintf(stderr, "vc: injected fault: %s call %d\n", kind, n);
    return true;
  }
  return false;
}

VCError map_cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return VCError::Success;
  VCError out;
  switch (e) {
    case cudaErrorMemoryAllocation: out = VCError::OutOfMemory; break;
    case cudaErrorInvalidValue:
    case cudaErrorInvalidPitchValue:
    case cudaErrorInvalidMemcpyDirection:
    case cudaErrorInvalidResourceHandle:
    case cudaErrorInvalidConfiguration:
    case cudaErrorNotSupported: out = VCError::InvalidValue; break;
    case cudaErrorInvalidDevice: out = VCError::InvalidDevice; break;
    case cudaErrorNotReady: return VCError::NotReady;
    case cudaErrorNoDevice:
    case cudaErrorInsufficientDriver:
    case cudaErrorInitializationError: out = VCError::InitializationError; break;
    case cudaErrorInvalidDeviceFunction:
    case cudaErrorNoKernelImageForDevice:
    case cudaErrorLaunchOutOfResources: out = VCError::InvalidKernel; break;
    default: out = VCError::Unknown; break;
  }
  std::fprintf(stderr, "vc: %s: %s\n", what, cudaGetErrorString(e));
  return out;
}

bool ensure_init() {
  if (st().initialized) return true;
  return vcInit() == VCError::Success;
}

void use_current_device() { cudaSetDevice(t_device); }

cudaStream_t resolve_stream(VCStreamHandle s) {
  if (s) return reinterpret_cast<cudaStream_t>(s);
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  auto it = S.recording.find(t_device);
  if (it != S.recording.end()) return it->second->capture;
  return nullptr;
}

int stream_device(VCStreamHandle s) {
  if (!s) return t_device;
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  auto it = S.stream_device.find(reinterpret_cast<void *>(s));
  return it == S.stream_device.end() ? t_device : it->second;
}

bool lookup_alloc(const void *p, uintptr_t *base, AllocInfo *info) {
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  auto it = S.allocs.upper_bound(a);
  if (it == S.allocs.begin()) return false;
  --it;
  if (a >= it->first + (it->second.size ? it->second.size : 1)) return false;
  if (base) *base = it->first;
  if (info) *info = it->second;
  return true;
}

// Bytes available from p to the end of its registered allocation, or
// SIZE_MAX when p is not a VC allocation (foreign memory is not checked).
size_t bytes_available(const void *p) {
  uintptr_t base;
  AllocInfo info;
  if (!lookup_alloc(p, &base, &info)) return SIZE_MAX;
  return info.size - (reinterpret_cast<uintptr_t>(p) - base);
}

// Bounded host wait on a stream (VC_SYNC_TIMEOUT_MS), NotReady on timeout.
VCError wait_stream(cudaStream_t s) {
  const long limit = st().sync_timeout_ms;
  if (limit <= 0) return map_cuda(cudaStreamSynchronize(s), "stream synchronize");
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(limit);
  for (;;) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return VCError::Success;
    if (e != cudaErrorNotReady) return map_cuda(e, "stream query");
    if (std::chrono::steady_clock::now() > deadline) {
      std::fprintf(stderr, "vc: stream wait exceeded VC_SYNC_TIMEOUT_MS=%ld\n", limit);
      return VCError::NotReady;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void harvest_locked(State &S, bool block) {
  std::vector<PendingSpan> keep;
  for (auto &sp : S.spans) {
    cudaSetDevice(sp.device);
    if (block) cudaEventSynchronize(sp.b);
    if (cudaEventQuery(sp.b) == cudaSuccess) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, sp.a, sp.b);
      auto &agg = S.profile_table[sp.name];
      agg.calls += 1;
      agg.total_ms += ms;
      if (ms > agg.max_ms) agg.max_ms = ms;
      cudaEventDestroy(sp.a);
      cudaEventDestroy(sp.b);
    } else {
      keep.push_back(sp);
    }
  }
  S.spans.swap(keep);
  std::vector<DeferredFree> still;
  for (auto &d : S.deferred) {
    cudaSetDevice(d.device);
    if (block) cudaEventSynchronize(d.ev);
    if (cudaEventQuery(d.ev) == cudaSuccess) {
      cudaFree(d.ptr);
      cudaEventDestroy(d.ev);
    } else {
      still.push_back(d);
    }
  }
  S.deferred.swap(still);
  cudaSetDevice(t_device);
}

void harvest(bool block) {
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  harvest_locked(S, block);
}

// VC_PROFILE span around one operation on `s`.
struct ProfileScope {
  cudaEvent_t a = nullptr, b = nullptr;
  cudaStream_t s;
  const char *name;
  bool on;
  ProfileScope(const char *n, cudaStream_t stream) : s(stream), name(n), on(st().profile) {
    if (!on) return;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, s);
  }
  ~ProfileScope() {
    if (!on) return;
    cudaEventRecord(b, s);
    State &S = st();
    std::lock_guard<std::mutex> lk(S.mu);
    S.spans.push_back({name, a, b, t_device});
  }
};

// Worker thread for vcLaunchHostFunc callbacks.
struct HostFnQueue {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<std::pair<VCHostFn, void *>> q;
  std::thread worker;
  bool started = false;
  void start() {
    if (started) return;
    started = true;
    worker = std::thread([this] {
      for (;;) {
        std::pair<VCHostFn, void *> item;
        {
          std::unique_lock<std::mutex> lk(mu);
          cv.wait(lk, [this] { return !q.empty(); });
          item = q.front();
          q.pop_front();
        }
        if (!item.first) return;
        item.first(item.second);
      }
    });
    worker.detach();
  }
};

HostFnQueue &hostfn_queue() {
  static HostFnQueue *q = new HostFnQueue();
  return *q;
}

void CUDART_CB hostfn_trampoline(void *p) {
  auto *item = static_cast<std::pair<VCHostFn, void *> *>(p);
  HostFnQueue &q = hostfn_queue();
  {
    std::lock_guard<std::mutex> lk(q.mu);
    q.q.push_back(*item);
  }
  q.cv.notify_one();
  delete item;
}

}  // namespace

// =================================================================== vc::
namespace vc {

VCError vcInit() {
  State &S = st();
  {
    std::lock_guard<std::mutex> lk(S.mu);
    if (S.initialized) return VCError::Success;
  }
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n <= 0) {
    if (std::getenv("VC_DEBUG"))
      std::fprintf(stderr, "vc: no CUDA device (%s)\n", cudaGetErrorString(e));
    cudaGetLastError();
    return VCError::InitializationError;
  }
  std::lock_guard<std::mutex> lk(S.mu);
  S.device_count = n;
  S.profile = std::getenv("VC_PROFILE") && std::atoi(std::getenv("VC_PROFILE")) != 0;
  S.debug = std::getenv("VC_DEBUG") && std::atoi(std::getenv("VC_DEBUG")) != 0;
  S.poison = std::getenv("VC_POISON") && std::atoi(std::getenv("VC_POISON")) != 0;
  S.check_bounds =
      std::getenv("VC_CHECK_BOUNDS") && std::atoi(std::getenv("VC_CHECK_BOUNDS")) != 0;
  S.sync_timeout_ms = std::getenv("VC_SYNC_TIMEOUT_MS") ? std::atol(std::getenv("VC_SYNC_TIMEOUT_MS")) : 0;
  parse_faults_locked(S);
  S.initialized = true;
  if (t_device >= n) t_device = 0;
  cudaSetDevice(t_device);
  if (S.debug) std::fprintf(stderr, "vc: initialised, %d CUDA device(s)\n", n);
  return VCError::Success;
}

VCError vcShutdown() {
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  if (!S.initialized) return VCError::Success;
  for (int d = 0; d < S.device_count; ++d) {
    cudaSetDevice(d);
    cudaDeviceSynchronize();
  }
  harvest_locked(S, true);
  if (S.profile && !S.profile_table.empty()) {
    std::fprintf(stderr, "vc profile: %-28s %8s %12s %12s\n", "op", "calls", "total_ms", "max_ms");
    for (auto &kv : S.profile_table)
      std::fprintf(stderr, "vc profile: %-28s %8ld %12.4f %12.4f\n", kv.first.c_str(),
                   kv.second.calls, kv.second.total_ms, kv.second.max_ms);
    S.profile_table.clear();
  }
  for (auto &kv : S.scratch) {
    cudaSetDevice(kv.first.first);
    cudaFree(kv.second.partials);
    cudaFree(kv.second.ticket);
  }
  S.scratch.clear();
  for (auto &kv : S.allocs) {
    cudaSetDevice(kv.second.device);
    void *p = reinterpret_cast<void *>(kv.first);
    if (kv.second.kind == VCMemoryType::Host) cudaFreeHost(p);
    else cudaFree(p);
  }
  S.allocs.clear();
  S.initialized = false;
  cudaSetDevice(t_device);
  return VCError::Success;
}

VCError vcEnableKernelPrintf(int enable) {
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  if (S.initialized) return VCError::InvalidValue;
  S.printf_flag = enable != 0;
  return VCError::Success;
}

VCError vcGetDeviceCount(int *count) {
  if (!count) return VCError::InvalidValue;
  if (!ensure_init()) {
    *count = 0;
    return VCError::Success;
  }
  *count = st().device_count;
  return VCError::Success;
}

VCError vcGetDevice(int *device) {
  if (!device) return VCError::InvalidValue;
  if (!st().initialized) return VCError::InitializationError;
  *device = t_device;
  return VCError::Success;
}

VCError vcSetDevice(int device) {
  if (!st().initialized) return VCError::InitializationError;
  if (device < 0 || device >= st().device_count) return VCError::InvalidDevice;
  t_device = device;
  return map_cuda(cudaSetDevice(device), "set device");
}

VCError vcGetDeviceProperties(VCDeviceProperties *out, int device) {
  if (!st().initialized) return VCError::InitializationError;
  if (!out) return VCError::InvalidValue;
  if (device < 0 || device >= st().device_count) return VCError::InvalidDevice;
  cudaDeviceProp p;
  VCError e = map_cuda(cudaGetDeviceProperties(&p, device), "device properties");
  if (e != VCError::Success) return e;
  std::memset(out, 0, sizeof(*out));
  std::snprintf(out->name, sizeof(out->name), "%s", p.name);
  out->totalGlobalMem = p.totalGlobalMem;
  out->sharedMemPerBlock = p.sharedMemPerBlockOptin;
  out->sharedMemPerMultiprocessor = p.sharedMemPerMultiprocessor;
  out->warpSize = p.warpSize;
  out->maxThreadsPerBlock = p.maxThreadsPerBlock;
  for (int i = 0; i < 3; ++i) {
    out->maxThreadsDim[i] = p.maxThreadsDim[i];
    out->maxGridSize[i] = p.maxGridSize[i];
  }
  int clk = 0;
  cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device);
  out->clockRate = clk;
  out->multiProcessorCount = p.multiProcessorCount;
  out->major = p.major;
  out->minor = p.minor;
  return VCError::Success;
}

VCError vcOccupancyMaxPotentialBlockSize(int *minGridSize, int *blockSize,
                                         VCKernelHandle kernel,
                                         size_t dynamicSharedMemPerBlock,
                                         int blockSizeLimit) {
  if (!st().initialized) return VCError::InitializationError;
  if (!kernel) return VCError::InvalidKernel;
  if (!minGridSize || !blockSize) return VCError::InvalidValue;
  int dev = t_device, sms = 0, smem = 0, maxthr = 1024, thr_sm = 2048;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&maxthr, cudaDevAttrMaxThreadsPerBlock, dev);
  cudaDeviceGetAttribute(&thr_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
  if (dynamicSharedMemPerBlock > (size_t)smem) return VCError::OutOfMemory;
  int limit = blockSizeLimit > 0 && blockSizeLimit < maxthr ? blockSizeLimit : maxthr;
  int bs = 1;
  while (bs * 2 <= limit) bs *= 2;
  if (bs < 32) return VCError::OutOfMemory;
  *blockSize = bs;
  *minGridSize = sms * (thr_sm / bs);
  return VCError::Success;
}

VCError vcPointerGetAttributes(VCPointerAttributes *out, const void *ptr) {
  if (!st().initialized) return VCError::InitializationError;
  if (!out) return VCError::InvalidValue;
  *out = VCPointerAttributes{};
  uintptr_t base;
  AllocInfo info;
  if (!ptr || !lookup_alloc(ptr, &base, &info)) return VCError::Success;
  out->memoryType = info.kind;
  out->size = info.size;
  void *b = reinterpret_cast<void *>(base);
  if (info.kind == VCMemoryType::Device) {
    out->devicePointer = b;
  } else {
    out->devicePointer = b;
    out->hostPointer = b;
  }
  return VCError::Success;
}

static VCError alloc_common(void **p, size_t bytes, VCMemoryType kind) {
  if (!p) return VCError::InvalidValue;
  if (inject_fault("malloc")) return VCError::OutOfMemory;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  void *ptr = nullptr;
  cudaError_t e;
  const size_t n = bytes ? bytes : 1;
  if (kind == VCMemoryType::Device) e = cudaMalloc(&ptr, n);
  else if (kind == VCMemoryType::Host) e = cudaMallocHost(&ptr, n);
  else e = cudaMallocManaged(&ptr, n);
  if (e != cudaSuccess) return map_cuda(e, "allocation");
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  S.allocs[reinterpret_cast<uintptr_t>(ptr)] = AllocInfo{kind, bytes, t_device};
  *p = ptr;
  return VCError::Success;
}

VCError vcMalloc(void **devPtr, size_t bytes) { return alloc_common(devPtr, bytes, VCMemoryType::Device); }
VCError vcMallocHost(void **hostPtr, size_t bytes) { return alloc_common(hostPtr, bytes, VCMemoryType::Host); }
VCError vcMallocManaged(void **devPtr, size_t bytes) { return alloc_common(devPtr, bytes, VCMemoryType::Managed); }
VCError vcMallocManagedS(void **devPtr, size_t bytes, VCStreamHandle) { return vcMallocManaged(devPtr, bytes); }
VCError vcMallocAsync(void **devPtr, size_t bytes, VCStreamHandle) { return vcMalloc(devPtr, bytes); }
VCError vcMallocHostAsync(void **hostPtr, size_t bytes, VCStreamHandle) { return vcMallocHost(hostPtr, bytes); }

VCError vcFree(void *ptr) {
  if (!ptr) return VCError::Success;
  State &S = st();
  AllocInfo info;
  {
    std::lock_guard<std::mutex> lk(S.mu);
    auto it = S.allocs.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == S.allocs.end()) return VCError::InvalidValue;
    info = it->second;
    S.allocs.erase(it);
  }
  cudaSetDevice(info.device);
  cudaError_t e = info.kind == VCMemoryType::Host ? cudaFreeHost(ptr) : cudaFree(ptr);
  cudaSetDevice(t_device);
  return map_cuda(e, "free");
}

VCError vcFreeAsync(void *ptr, VCStreamHandle stream) {
  if (!ptr) return VCError::Success;
  State &S = st();
  AllocInfo info;
  {
    std::lock_guard<std::mutex> lk(S.mu);
    auto it = S.allocs.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == S.allocs.end()) return VCError::InvalidValue;
    info = it->second;
    S.allocs.erase(it);
  }
  if (info.kind == VCMemoryType::Host) return map_cuda(cudaFreeHost(ptr), "free host");
  // Released once the work already queued on `stream` has completed; reclaimed
  // at the next synchronisation point (the reference contract).
  cudaEvent_t ev;
  cudaSetDevice(info.device);
  cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  cudaEventRecord(ev, resolve_stream(stream));
  std::lock_guard<std::mutex> lk(S.mu);
  S.deferred.push_back({ptr, ev, info.device});
  cudaSetDevice(t_device);
  return VCError::Success;
}

VCError vcCreateImage2D(VCImageHandle *, uint32_t, uint32_t, VCPixelFormat) { return VCError::InvalidValue; }
VCError vcCreateImage1D(VCImageHandle *, uint32_t, VCPixelFormat) { return VCError::InvalidValue; }
VCError vcCreateImage3D(VCImageHandle *, uint32_t, uint32_t, uint32_t, VCPixelFormat) { return VCError::InvalidValue; }
VCError vcCreateImage2DArray(VCImageHandle *, uint32_t, uint32_t, uint32_t, VCPixelFormat) { return VCError::InvalidValue; }
VCError vcDestroyImage(VCImageHandle img) { return img ? VCError::InvalidValue : VCError::Success; }
VCError vcMemcpyToImage(VCImageHandle, const void *) { return VCError::InvalidValue; }
VCError vcMemcpyFromImage(void *, VCImageHandle) { return VCError::InvalidValue; }

static cudaMemcpyKind cuda_kind(VCMemcpyKind k) {
  switch (k) {
    case VCMemcpyKind::HostToDevice: return cudaMemcpyHostToDevice;
    case VCMemcpyKind::DeviceToHost: return cudaMemcpyDeviceToHost;
    default: return cudaMemcpyDeviceToDevice;
  }
}

// Capture-aware async copy: during graph recording, H2D sources are
// snapshotted into pinned staging owned by the graph.
static VCError copy_async(void *dst, const void *src, size_t count, VCMemcpyKind kind,
                          cudaStream_t s) {
  State &S = st();
  VCGraph *g = nullptr;
  {
    std::lock_guard<std::mutex> lk(S.mu);
    auto it = S.recording.find(t_device);
    if (it != S.recording.end() && it->second->capture == s) g = it->second;
  }
  if (g && kind == VCMemcpyKind::DeviceToHost) return VCError::InvalidValue;
  if (g && kind == VCMemcpyKind::HostToDevice) {
    void *stage = nullptr;
    VCError e = map_cuda(cudaMallocHost(&stage, count), "graph staging");
    if (e != VCError::Success) return e;
    std::memcpy(stage, src, count);
    g->staging.push_back(stage);
    src = stage;
  }
  ProfileScope prof(kind == VCMemcpyKind::HostToDevice ? "memcpy H2D"
                    : kind == VCMemcpyKind::DeviceToHost ? "memcpy D2H" : "memcpy D2D", s);
  return map_cuda(cudaMemcpyAsync(dst, src, count, cuda_kind(kind), s), "memcpy");
}

VCError vcMemcpyS(void *dst, const void *src, size_t count, VCMemcpyKind kind,
                  VCStreamHandle stream) {
  if (!dst || !src) return VCError::InvalidValue;
  if (inject_fault("memcpy")) return VCError::Unknown;
  if (!ensure_init()) return VCError::InitializationError;
  if (count == 0) return VCError::Success;
  use_current_device();
  cudaStream_t s = resolve_stream(stream);
  VCError e = copy_async(dst, src, count, kind, s);
  if (e != VCError::Success) return e;
  if (kind == VCMemcpyKind::DeviceToDevice) return VCError::Success;
  return wait_stream(s);  // H2D and D2H block (reference contract)
}

VCError vcMemcpy(void *dst, const void *src, size_t count, VCMemcpyKind kind) {
  return vcMemcpyS(dst, src, count, kind, nullptr);
}

VCError vcMemcpyAsyncS(void *dst, const void *src, size_t count, VCMemcpyKind kind,
                       VCStreamHandle stream) {
  if (!dst || !src) return VCError::InvalidValue;
  if (inject_fault("memcpy")) return VCError::Unknown;
  if (!ensure_init()) return VCError::InitializationError;
  if (count == 0) return VCError::Success;
  use_current_device();
  return copy_async(dst, src, count, kind, resolve_stream(stream));
}

VCError vcMemcpyAsync(void *dst, const void *src, size_t count, VCMemcpyKind kind) {
  return vcMemcpyAsyncS(dst, src, count, kind, nullptr);
}

static VCError peer_common(void *dst, int dstDevice, const void *src, int srcDevice,
                           size_t bytes) {
  if (!dst || !src) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  const int n = st().device_count;
  if (dstDevice < 0 || dstDevice >= n || srcDevice < 0 || srcDevice >= n)
    return VCError::InvalidDevice;
  AllocInfo di, si;
  if (lookup_alloc(dst, nullptr, &di) && di.device != dstDevice) return VCError::InvalidValue;
  if (lookup_alloc(src, nullptr, &si) && si.device != srcDevice) return VCError::InvalidValue;
  if (bytes > bytes_available(dst) || bytes > bytes_available(src)) return VCError::InvalidValue;
  if (dstDevice != srcDevice) {
    int can = 0;
    cudaDeviceCanAccessPeer(&can, dstDevice, srcDevice);
    if (can) {
      cudaSetDevice(dstDevice);
      cudaError_t e = cudaDeviceEnablePeerAccess(srcDevice, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
    }
  }
  return VCError::Success;
}

VCError vcMemcpyPeer(void *dst, int dstDevice, const void *src, int srcDevice, size_t bytes) {
  VCError e = peer_common(dst, dstDevice, src, srcDevice, bytes);
  if (e != VCError::Success) return e;
  if (bytes == 0) return VCError::Success;
  cudaSetDevice(dstDevice);
  e = map_cuda(cudaMemcpyPeerAsync(dst, dstDevice, src, srcDevice, bytes, nullptr), "peer copy");
  if (e == VCError::Success) e = wait_stream(nullptr);
  cudaSetDevice(t_device);
  return e;
}

VCError vcMemcpyPeerAsync(void *dst, int dstDevice, const void *src, int srcDevice,
                          size_t bytes, VCStreamHandle stream) {
  VCError e = peer_common(dst, dstDevice, src, srcDevice, bytes);
  if (e != VCError::Success) return e;
  if (stream_device(stream) != dstDevice) return VCError::InvalidValue;
  if (bytes == 0) return VCError::Success;
  cudaSetDevice(dstDevice);
  e = map_cuda(cudaMemcpyPeerAsync(dst, dstDevice, src, srcDevice, bytes, resolve_stream(stream)),
               "peer copy");
  cudaSetDevice(t_device);
  return e;
}

VCError vcMemsetAsyncS(void *ptr, int value, size_t count, VCStreamHandle stream) {
  if (!ptr) return VCError::InvalidValue;
  if (count % 4 != 0) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  if (count > bytes_available(ptr)) return VCError::InvalidValue;
  use_current_device();
  cudaStream_t s = resolve_stream(stream);
  ProfileScope prof("memset", s);
  return map_cuda(cudaMemsetAsync(ptr, value & 0xff, count, s), "memset");
}

VCError vcMemsetS(void *ptr, int value, size_t count, VCStreamHandle stream) {
  VCError e = vcMemsetAsyncS(ptr, value, count, stream);
  if (e != VCError::Success) return e;
  return wait_stream(resolve_stream(stream));
}
VCError vcMemset(void *ptr, int value, size_t count) { return vcMemsetS(ptr, value, count, nullptr); }
VCError vcMemsetAsync(void *ptr, int value, size_t count) { return vcMemsetAsyncS(ptr, value, count, nullptr); }

VCError vcMemcpy2DAsync(void *dst, size_t dpitch, const void *src, size_t spitch,
                        size_t width, size_t height, VCMemcpyKind kind, VCStreamHandle stream) {
  if (kind != VCMemcpyKind::DeviceToDevice) return VCError::InvalidValue;
  if (!dst || !src) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  if (width == 0 || height == 0) return VCError::Success;
  if (width > dpitch || width > spitch) return VCError::InvalidValue;
  const size_t need_d = (height - 1) * dpitch + width, need_s = (height - 1) * spitch + width;
  if (need_d > bytes_available(dst) || need_s > bytes_available(src)) return VCError::InvalidValue;
  use_current_device();
  cudaStream_t s = resolve_stream(stream);
  ProfileScope prof("memcpy2D D2D", s);
  return map_cuda(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height,
                                    cudaMemcpyDeviceToDevice, s), "memcpy2D");
}

VCError vcMemcpy2DS(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width,
                    size_t height, VCMemcpyKind kind, VCStreamHandle stream) {
  VCError e = vcMemcpy2DAsync(dst, dpitch, src, spitch, width, height, kind, stream);
  if (e != VCError::Success) return e;
  return wait_stream(resolve_stream(stream));
}

VCError vcMemcpy2D(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width,
                   size_t height, VCMemcpyKind kind) {
  return vcMemcpy2DS(dst, dpitch, src, spitch, width, height, kind, nullptr);
}

VCError vcMemset2DAsync(void *dst, size_t pitch, int value, size_t width, size_t height,
                        VCStreamHandle stream) {
  if (!dst) return VCError::InvalidValue;
  if (width % 4 != 0) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  if (width == 0 || height == 0) return VCError::Success;
  if (width > pitch) return VCError::InvalidValue;
  if ((height - 1) * pitch + width > bytes_available(dst)) return VCError::InvalidValue;
  use_current_device();
  cudaStream_t s = resolve_stream(stream);
  ProfileScope prof("memset2D", s);
  return map_cuda(cudaMemset2DAsync(dst, pitch, value & 0xff, width, height, s), "memset2D");
}

VCError vcMemset2D(void *dst, size_t pitch, int value, size_t width, size_t height) {
  VCError e = vcMemset2DAsync(dst, pitch, value, width, height, nullptr);
  if (e != VCError::Success) return e;
  return wait_stream(resolve_stream(nullptr));
}

VCError vcDeviceSynchronize() {
  if (!st().initialized) return VCError::InitializationError;
  use_current_device();
  VCError e;
  if (st().sync_timeout_ms > 0) {
    // Bounded: poll the legacy stream and every stream created here.
    std::vector<cudaStream_t> streams{nullptr};
    {
      std::lock_guard<std::mutex> lk(st().mu);
      for (auto &kv : st().stream_device)
        if (kv.second == t_device) streams.push_back(reinterpret_cast<cudaStream_t>(kv.first));
    }
    e = VCError::Success;
    for (cudaStream_t s : streams) {
      e = wait_stream(s);
      if (e != VCError::Success) break;
    }
    if (e == VCError::Success) e = map_cuda(cudaDeviceSynchronize(), "device synchronize");
  } else {
    e = map_cuda(cudaDeviceSynchronize(), "device synchronize");
  }
  harvest(false);
  return e;
}

VCError vcStreamCreate(VCStreamHandle *out) {
  if (!out) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  cudaStream_t s;
  VCError e = map_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
  if (e != VCError::Success) return e;
  {
    std::lock_guard<std::mutex> lk(st().mu);
    st().stream_device[reinterpret_cast<void *>(s)] = t_device;
  }
  *out = reinterpret_cast<VCStreamHandle>(s);
  return VCError::Success;
}

VCError vcStreamDestroy(VCStreamHandle stream) {
  if (!stream) return VCError::InvalidValue;
  {
    std::lock_guard<std::mutex> lk(st().mu);
    st().stream_device.erase(reinterpret_cast<void *>(stream));
  }
  return map_cuda(cudaStreamDestroy(reinterpret_cast<cudaStream_t>(stream)), "stream destroy");
}

VCError vcStreamSynchronize(VCStreamHandle stream) {
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  VCError e = wait_stream(resolve_stream(stream));
  harvest(false);
  return e;
}

VCError vcStreamQuery(VCStreamHandle stream, int *done) {
  if (!done) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  cudaError_t e = cudaStreamQuery(resolve_stream(stream));
  if (e == cudaSuccess) { *done = 1; return VCError::Success; }
  if (e == cudaErrorNotReady) { cudaGetLastError(); *done = 0; return VCError::Success; }
  return map_cuda(e, "stream query");
}

VCError vcLaunchHostFunc(VCStreamHandle stream, VCHostFn fn, void *userData) {
  if (!fn) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  hostfn_queue().start();
  auto *item = new std::pair<VCHostFn, void *>(fn, userData);
  cudaError_t e = cudaLaunchHostFunc(resolve_stream(stream), hostfn_trampoline, item);
  if (e != cudaSuccess) delete item;
  return map_cuda(e, "host function");
}

VCError vcEventCreate(VCEventHandle *out) {
  if (!out) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  auto *ev = new VCEvent();
  ev->device = t_device;
  VCError e = map_cuda(cudaEventCreate(&ev->ev), "event create");
  if (e != VCError::Success) { delete ev; return e; }
  *out = ev;
  return VCError::Success;
}

VCError vcEventDestroy(VCEventHandle event) {
  if (!event) return VCError::InvalidValue;
  cudaEventDestroy(event->ev);
  delete event;
  return VCError::Success;
}

VCError vcEventRecord(VCEventHandle event, VCStreamHandle stream) {
  if (!event) return VCError::InvalidValue;
  use_current_device();
  VCError e = map_cuda(cudaEventRecord(event->ev, resolve_stream(stream)), "event record");
  if (e == VCError::Success) event->recorded = true;
  return e;
}

VCError vcStreamWaitEvent(VCStreamHandle stream, VCEventHandle event) {
  if (!event) return VCError::InvalidValue;
  use_current_device();
  return map_cuda(cudaStreamWaitEvent(resolve_stream(stream), event->ev, 0), "stream wait event");
}

VCError vcEventQuery(VCEventHandle event, int *done) {
  if (!event || !done) return VCError::InvalidValue;
  cudaError_t e = cudaEventQuery(event->ev);
  if (e == cudaSuccess) { *done = 1; return VCError::Success; }
  if (e == cudaErrorNotReady) { cudaGetLastError(); *done = 0; return VCError::Success; }
  return map_cuda(e, "event query");
}

VCError vcEventSynchronize(VCEventHandle event) {
  if (!event) return VCError::InvalidValue;
  const long limit = st().sync_timeout_ms;
  if (limit <= 0) return map_cuda(cudaEventSynchronize(event->ev), "event synchronize");
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(limit);
  for (;;) {
    cudaError_t e = cudaEventQuery(event->ev);
    if (e == cudaSuccess) return VCError::Success;
    if (e != cudaErrorNotReady) return map_cuda(e, "event query");
    if (std::chrono::steady_clock::now() > deadline) return VCError::NotReady;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

VCError vcEventElapsedTime(float *ms, VCEventHandle start, VCEventHandle end) {
  if (!start || !end || !ms) return VCError::InvalidValue;
  if (!start->recorded || !end->recorded) return VCError::InvalidValue;
  cudaError_t e = cudaEventElapsedTime(ms, start->ev, end->ev);
  if (e == cudaErrorNotReady) { cudaGetLastError(); return VCError::NotReady; }
  return map_cuda(e, "event elapsed time");
}

VCError vcGraphCreate(VCGraphHandle *out) {
  if (!out) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  auto *g = new VCGraph();
  g->device = t_device;
  *out = g;
  return VCError::Success;
}

static void graph_release(VCGraph *g) {
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  g->exec = nullptr;
  g->graph = nullptr;
  for (void *p : g->staging) cudaFreeHost(p);
  g->staging.clear();
}

VCError vcGraphDestroy(VCGraphHandle graph) {
  if (!graph) return VCError::InvalidValue;
  if (graph->recording) vcGraphEndRecord(graph);
  graph_release(graph);
  if (graph->capture) cudaStreamDestroy(graph->capture);
  delete graph;
  return VCError::Success;
}

VCError vcGraphBeginRecord(VCGraphHandle graph) {
  if (!graph) return VCError::InvalidValue;
  if (graph->recording) return VCError::InvalidValue;
  State &S = st();
  {
    std::lock_guard<std::mutex> lk(S.mu);
    if (S.recording.count(t_device)) return VCError::InvalidValue;
  }
  use_current_device();
  graph_release(graph);
  if (!graph->capture) {
    VCError e = map_cuda(cudaStreamCreateWithFlags(&graph->capture, cudaStreamNonBlocking),
                         "graph stream");
    if (e != VCError::Success) return e;
  }
  // Work already queued on the default stream precedes the graph's replay;
  // make the capture stream start after it.
  cudaStreamSynchronize(nullptr);
  VCError e = map_cuda(cudaStreamBeginCapture(graph->capture, cudaStreamCaptureModeRelaxed),
                       "begin capture");
  if (e != VCError::Success) return e;
  graph->device = t_device;
  graph->recording = true;
  std::lock_guard<std::mutex> lk(S.mu);
  S.recording[t_device] = graph;
  return VCError::Success;
}

VCError vcGraphEndRecord(VCGraphHandle graph) {
  if (!graph || !graph->recording) return VCError::InvalidValue;
  {
    std::lock_guard<std::mutex> lk(st().mu);
    st().recording.erase(graph->device);
  }
  graph->recording = false;
  VCError e = map_cuda(cudaStreamEndCapture(graph->capture, &graph->graph), "end capture");
  if (e != VCError::Success) return e;
  return map_cuda(cudaGraphInstantiate(&graph->exec, graph->graph, 0), "graph instantiate");
}

VCError vcGraphLaunch(VCGraphHandle graph, VCStreamHandle stream) {
  if (!graph || !graph->exec || graph->recording) return VCError::InvalidValue;
  use_current_device();
  cudaStream_t s = resolve_stream(stream);
  ProfileScope prof("graph launch", s);
  return map_cuda(cudaGraphLaunch(graph->exec, s), "graph launch");
}

VCError vcGraphReset(VCGraphHandle graph) {
  if (!graph) return VCError::InvalidValue;
  if (graph->recording) return VCError::InvalidValue;
  graph_release(graph);
  return VCError::Success;
}

const char *vcErrorString(VCError err) {
  switch (err) {
    case VCError::Success: return "success";
    case VCError::InvalidValue: return "invalid value";
    case VCError::OutOfMemory: return "out of memory";
    case VCError::InvalidKernel: return "invalid kernel";
    case VCError::InvalidDevice: return "invalid device";
    case VCError::InitializationError: return "initialization error";
    case VCError::MapFailed: return "map failed";
    case VCError::NotReady: return "not ready";
    default: return "unknown error";
  }
}

}  // namespace vc

// ============================================================ kernel registry
namespace vc {

struct LaunchShape {
  unsigned wgx, wgy;  // workgroup counts (ceil(grid / block))
  unsigned bx, by;    // block sizes
};

using LaunchFn = VCError (*)(VCKernel &, const LaunchShape &, const VCKernelArg *, int,
                             cudaStream_t);

struct KernelEntry {
  const char *name;
  LaunchFn launch;
  std::vector<std::pair<const char *, long long>> constants;
};

}  // namespace vc

namespace {

// ---- argument decoding: Pointer args carry a device address, Scalar args
// point at `size` bytes that are read here (copied at launch).
bool arg_ptr(const VCKernelArg *a, int n, int i, const void **out) {
  if (i >= n || a[i].kind != VCKernelArg::Pointer) return false;
  *out = a[i].data;
  return true;
}
bool arg_i64(const VCKernelArg *a, int n, int i, long long *out) {
  if (i >= n || a[i].kind != VCKernelArg::Scalar || !a[i].data) return false;
  if (a[i].size == 4) { *out = *static_cast<const int32_t *>(a[i].data); return true; }
  if (a[i].size == 8) { *out = *static_cast<const int64_t *>(a[i].data); return true; }
  return false;
}
bool arg_f32(const VCKernelArg *a, int n, int i, float *out) {
  if (i >= n || a[i].kind != VCKernelArg::Scalar || !a[i].data) return false;
  if (a[i].size == 4) { *out = *static_cast<const float *>(a[i].data); return true; }
  if (a[i].size == 8) { *out = static_cast<float>(*static_cast<const double *>(a[i].data)); return true; }
  return false;
}

VCError bad_args(const char *k) {
  std::fprintf(stderr, "vc: kernel %s: argument list does not match the kernel\n", k);
  return VCError::InvalidValue;
}

VCError too_small(const char *k) {
  std::fprintf(stderr, "vc: kernel %s: a buffer is smaller than the launch needs\n", k);
  return VCError::InvalidValue;
}

long long konst(const VCKernel &k, const char *name) {
  auto it = k.constants.find(name);
  return it == k.constants.end() ? 0 : it->second;
}

VCError run(cudaError_t e, const char *what) { return map_cuda(e, what); }

// ---- VC_POISON=1: a NaN canary in every output before its kernel runs.
// With compute-sanitizer closed, this is how a kernel that leaves part of its
// output unwritten shows itself: the region the kernel's contract says it
// writes is filled with 0xFF bytes (NaN for fp32 / fp16 / bf16, -1 for
// integers) on the launch stream, so an element the kernel skips reads back
// as NaN instead of a stale plausible value. A region that shares memory with
// an input of the same launch (an in-place call) is left alone.
struct Span {
  const void *p;
  size_t bytes;
};
bool spans_overlap(const void *p, size_t bytes, std::initializer_list<Span> inputs) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(p), a1 = a0 + bytes;
  for (const Span &in : inputs) {
    if (!in.p || !in.bytes) continue;
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(in.p), b1 = b0 + in.bytes;
    if (a0 < b1 && b0 < a1) return true;
  }
  return false;
}
// Output of `rows` rows of `width` bytes, `pitch` bytes apart.
void poison_output(const char *kernel, void *p, size_t pitch, size_t width, size_t rows,
                   cudaStream_t s, std::initializer_list<Span> inputs) {
  if (!st().poison || !p || !width || !rows) return;
  const size_t span = (rows - 1) * pitch + width;
  if (spans_overlap(p, span, inputs)) return;
  cudaError_t e = rows == 1 ? cudaMemsetAsync(p, 0xFF, width, s)
                            : cudaMemset2DAsync(p, pitch, 0xFF, width, rows, s);
  if (st().debug)
    std::fprintf(stderr, "vc: poison %s output %p, %zu x %zu bytes (%s)\n", kernel, p, rows, width,
                 cudaGetErrorString(e));
}
void poison_output(const char *kernel, void *p, size_t bytes, cudaStream_t s,
                   std::initializer_list<Span> inputs) {
  poison_output(kernel, p, bytes, bytes, 1, s, inputs);
}

// ---- VC_CHECK_BOUNDS=1: the demo kernels (vadd, fillPattern, blockReduce
// and their native entries) run their bounds-checked forms, in which every
// global access is checked on the device against the extent the allocation
// registry records for its buffer; an index past it sets kErrOutOfBounds in
// the error word (vc_kernel_error) and is skipped. The host checks above each
// launch use the same extents, so a check that fires means the kernel's own
// index arithmetic went wrong. (The TMA kernels need no such form: their
// tensor maps bound every copy in hardware.)
int64_t elems_available(const void *p, size_t esz) {
  const size_t b = bytes_available(p);
  return b == SIZE_MAX ? INT64_MAX : (int64_t)(b / esz);
}
bool checking(const char *name) {
  if (!st().check_bounds) return false;
  if (st().debug) std::fprintf(stderr, "vc: bounds-checked %s launch\n", name);
  return true;
}
cudaError_t vadd_maybe_checked(const float *a, const float *b, float *c, int64_t n,
                               cudaStream_t s, const char *name) {
  if (checking(name))
    return vcb::launch_vadd_f32_checked(a, b, c, n, elems_available(a, 4), elems_available(b, 4),
                                        elems_available(c, 4), s);
  return vcb::launch_vadd_f32(a, b, c, n, s);
}
cudaError_t block_reduce_maybe_checked(const float *in, float *out, int n, int block, int groups,
                                       cudaStream_t s, const char *name) {
  if (checking(name))
    return vcb::launch_block_reduce_demo(in, out, n, block, groups, s, elems_available(in, 4),
                                         elems_available(out, 4));
  return vcb::launch_block_reduce_demo(in, out, n, block, groups, s);
}

// vadd(a, b, c, int n): c[i] = a[i] + b[i] for i < min(n, workgroups*block)
// (test/vadd.vc:12-17).
VCError k_vadd(VCKernel &, const LaunchShape &sh, const VCKernelArg *a, int n, cudaStream_t s) {
  const void *pa, *pb, *pc;
  long long cnt;
  if (!arg_ptr(a, n, 0, &pa) || !arg_ptr(a, n, 1, &pb) || !arg_ptr(a, n, 2, &pc) ||
      !arg_i64(a, n, 3, &cnt) || n != 4)
    return bad_args("vadd");
  long long covered = (long long)sh.wgx * sh.bx * sh.wgy * sh.by;
  long long m = cnt < covered ? cnt : covered;
  if (m <= 0) return VCError::Success;
  const size_t bytes = (size_t)m * 4;
  if (bytes > bytes_available(pa) || bytes > bytes_available(pb) || bytes > bytes_available(pc))
    return too_small("vadd");
  poison_output("vadd", const_cast<void *>(pc), bytes, s, {{pa, bytes}, {pb, bytes}});
  return run(vadd_maybe_checked((const float *)pa, (const float *)pb, (float *)pc, m, s, "vadd"),
             "vadd");
}

// fillPattern(int *a, int base, int n): a[i] = base + i for
// i < min(n, workgroups*block) (test/multigpu.vc:24-27).
VCError k_fill_pattern(VCKernel &, const LaunchShape &sh, const VCKernelArg *a, int n,
                       cudaStream_t s) {
  const void *pa;
  long long base, cnt;
  if (!arg_ptr(a, n, 0, &pa) || !arg_i64(a, n, 1, &base) || !arg_i64(a, n, 2, &cnt) || n != 3)
    return bad_args("fillPattern");
  long long covered = (long long)sh.wgx * sh.bx * sh.wgy * sh.by;
  long long m = cnt < covered ? cnt : covered;
  if (m <= 0) return VCError::Success;
  if ((size_t)m * 4 > bytes_available(pa)) return too_small("fillPattern");
  poison_output("fillPattern", const_cast<void *>(pa), (size_t)m * 4, s, {});
  if (checking("fillPattern"))
    return run(vcb::launch_fill_pattern_checked((int *)pa, (int)base, m, elems_available(pa, 4), s),
               "fillPattern");
  return run(vcb::launch_fill_pattern((int *)pa, (int)base, m, s), "fillPattern");
}

// blockReduce(in, out, int N): out[g] = tree sum of block g (test/reduce.vc).
VCError k_block_reduce(VCKernel &, const LaunchShape &sh, const VCKernelArg *a, int n,
                       cudaStream_t s) {
  const void *pin, *pout;
  long long N;
  if (!arg_ptr(a, n, 0, &pin) || !arg_ptr(a, n, 1, &pout) || !arg_i64(a, n, 2, &N) || n != 3)
    return bad_args("blockReduce");
  if (sh.by != 1 || sh.wgy != 1 || sh.bx > 1024) return bad_args("blockReduce");
  const long long groups = sh.wgx;
  if ((size_t)groups * 4 > bytes_available(pout)) return too_small("blockReduce");
  long long need = N < groups * (long long)sh.bx ? N : groups * (long long)sh.bx;
  if (need > 0 && (size_t)need * 4 > bytes_available(pin)) return too_small("blockReduce");
  poison_output("blockReduce", const_cast<void *>(pout), (size_t)groups * 4, s,
                {{pin, need > 0 ? (size_t)need * 4 : 0}});
  return run(block_reduce_maybe_checked((const float *)pin, (float *)pout, (int)N, (int)sh.bx,
                                        (int)groups, s, "blockReduce"),
             "blockReduce");
}

// flashAttn(Q, K, V, O, float scale, int causal) with the demo's compile-time
// NHEAD / SEQ / HDIM (examples/flash_attn.vc:50-54, 56-126). `scale` is in
// the exp2 domain; causal is on only for the value 1 (flash_attn.vc:100).
VCError k_flash_attn(VCKernel &k, const LaunchShape &sh, const VCKernelArg *a, int n,
                     cudaStream_t s) {
  const void *q, *kk, *v, *o;
  float scale;
  long long causal;
  if (!arg_ptr(a, n, 0, &q) || !arg_ptr(a, n, 1, &kk) || !arg_ptr(a, n, 2, &v) ||
      !arg_ptr(a, n, 3, &o) || !arg_f32(a, n, 4, &scale) || !arg_i64(a, n, 5, &causal) || n != 6)
    return bad_args("flashAttn");
  const long long nhead = konst(k, "NHEAD"), seq = konst(k, "SEQ"), hdim = konst(k, "HDIM"),
                  br = konst(k, "BR");
  if (sh.bx != (unsigned)br || (long long)sh.wgx * sh.bx != nhead * seq || sh.wgy != 1) {
    std::fprintf(stderr, "vc: flashAttn: launch grid must be NHEAD*SEQ=%lld elements of block BR=%lld\n",
                 nhead * seq, br);
    return VCError::InvalidValue;
  }
  const size_t bytes = (size_t)(nhead * seq * hdim) * 4;
  for (const void *p : {q, kk, v, o})
    if (bytes > bytes_available(p)) return too_small("flashAttn");
  vcb::FlashArgs f{q, kk, v, const_cast<void *>(o), (int)nhead, (int)seq, (int)hdim, scale,
                   causal == 1, 0};
  poison_output("flashAttn", const_cast<void *>(o), bytes, s, {{q, bytes}, {kk, bytes}, {v, bytes}});
  return run(vcb::launch_flash_fwd_f32(f, s), "flashAttn");
}

// D of a GEMM: M rows of N fp32 at row stride ldd (A, B, Cin are inputs).
void poison_gemm_output(const vcb::GemmArgs &g, size_t in_esz, cudaStream_t s, const char *name) {
  const size_t a_span = ((size_t)(g.M - 1) * g.lda + g.K) * in_esz;
  const size_t b_span = g.b_kn ? ((size_t)(g.K - 1) * g.ldb + g.N) * in_esz
                               : ((size_t)(g.N - 1) * g.ldb + g.K) * in_esz;
  const size_t c_span = g.Cin ? ((size_t)(g.M - 1) * g.ldc + g.N) * 4 : 0;
  poison_output(name, g.D, (size_t)g.ldd * 4, (size_t)g.N * 4, (size_t)g.M, s,
                {{g.A, a_span}, {g.B, b_span}, {g.Cin, c_span}});
}

VCError gemm_dispatch(const vcb::GemmArgs &g, cudaStream_t s, const char *name) {
  poison_gemm_output(g, 2, s, name);
  cudaError_t e = vcb::launch_gemm_tcgen05(g, s);
  if (e == cudaErrorNotSupported) {
    cudaGetLastError();
    e = vcb::launch_gemm_simt(g, s);
  }
  return run(e, name);
}

// fp32 A, B: the tensor-core path (three tf32 products per product) when
// TMA can take the strides, else the CUDA-core path.
VCError gemm_f32_dispatch(const vcb::GemmArgs &g, cudaStream_t s, const char *name) {
  poison_gemm_output(g, 4, s, name);
  cudaError_t e = vcb::launch_gemm_f32_tcgen05(g, s);
  if (e == cudaErrorNotSupported) {
    cudaGetLastError();
    e = vcb::launch_gemm_f32_simt(g, s);
  }
  return run(e, name);
}

// wmma_gemm(A, B, C, D): D = A*B + C for one 8x8x16 tile
// (test/wmma_gemm.vc:19-33): A 8x16 fp16 (ldm 16), B 16x8 fp16 (ldm 8), C/D
// 8x8 fp32 (ldm 8).
VCError k_wmma_gemm(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n, cudaStream_t s) {
  const void *A, *B, *C, *D;
  if (!arg_ptr(a, n, 0, &A) || !arg_ptr(a, n, 1, &B) || !arg_ptr(a, n, 2, &C) ||
      !arg_ptr(a, n, 3, &D) || n != 4)
    return bad_args("wmma_gemm");
  if (bytes_available(A) < 256 || bytes_available(B) < 256 || bytes_available(C) < 256 ||
      bytes_available(D) < 256)
    return too_small("wmma_gemm");
  vcb::GemmArgs g{A, B, (float *)D, (const float *)C, 8, 8, 16, 16, 8, 8, 8, false, true};
  return gemm_dispatch(g, s, "wmma_gemm");
}

// matmulCoopmat(A, B, C, int N): C[n][m] = sum_k A[n][k] B[k][m] over the
// 16x16 tiles the grid covers, row stride L (examples/matmul_coopmat_bench.vc
// :56-110). K runs in 16-steps up to N, as the reference's loop does.
VCError k_matmul_coopmat(VCKernel &k, const LaunchShape &sh, const VCKernelArg *a, int n,
                         cudaStream_t s) {
  const void *A, *B, *C;
  long long N;
  if (!arg_ptr(a, n, 0, &A) || !arg_ptr(a, n, 1, &B) || !arg_ptr(a, n, 2, &C) ||
      !arg_i64(a, n, 3, &N) || n != 4)
    return bad_args("matmulCoopmat");
  const long long L = konst(k, "L");
  const long long rows = (long long)sh.wgy * 16, cols = (long long)sh.wgx * 16;
  const long long kdim = ((N + 15) / 16) * 16;
  if (N <= 0 || rows <= 0 || cols <= 0) return VCError::Success;
  if (cols > L || kdim > L) return bad_args("matmulCoopmat");
  if ((size_t)((rows - 1) * L + kdim) * 2 > bytes_available(A) ||
      (size_t)((kdim - 1) * L + cols) * 2 > bytes_available(B) ||
      (size_t)((rows - 1) * L + cols) * 4 > bytes_available(C))
    return too_small("matmulCoopmat");
  vcb::GemmArgs g{A, B, (float *)C, nullptr, (int)rows, (int)cols, (int)kdim, L, L, L, 0, false, true};
  return gemm_dispatch(g, s, "matmulCoopmat");
}

// matmulTiled(A, B, C, int N): fp32 C = A*B, N x N row-major
// (examples/matmul_bench.vc:22-54), for the tiles the grid covers.
VCError k_matmul_tiled(VCKernel &, const LaunchShape &sh, const VCKernelArg *a, int n,
                       cudaStream_t s) {
  const void *A, *B, *C;
  long long N;
  if (!arg_ptr(a, n, 0, &A) || !arg_ptr(a, n, 1, &B) || !arg_ptr(a, n, 2, &C) ||
      !arg_i64(a, n, 3, &N) || n != 4)
    return bad_args("matmulTiled");
  if (N <= 0) return VCError::Success;
  long long rows = (long long)sh.wgy * sh.by, cols = (long long)sh.wgx * sh.bx;
  if (rows > N) rows = N;
  if (cols > N) cols = N;
  const size_t nn = (size_t)N * N * 4;
  if (nn > bytes_available(A) || nn > bytes_available(B) || nn > bytes_available(C))
    return too_small("matmulTiled");
  vcb::GemmArgs g{A, B, (float *)C, nullptr, (int)rows, (int)cols, (int)N, N, N, N, 0,
                  false, true};
  return gemm_f32_dispatch(g, s, "matmulTiled");
}

// ---- native entries (explicit shapes; grid and block are not used)
VCError k_native_vadd(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n, cudaStream_t s) {
  const void *pa, *pb, *pc;
  long long cnt;
  if (!arg_ptr(a, n, 0, &pa) || !arg_ptr(a, n, 1, &pb) || !arg_ptr(a, n, 2, &pc) ||
      !arg_i64(a, n, 3, &cnt) || n != 4 || cnt < 0)
    return bad_args("vc.vadd");
  const size_t bytes = (size_t)cnt * 4;
  if (bytes > bytes_available(pa) || bytes > bytes_available(pb) || bytes > bytes_available(pc))
    return too_small("vc.vadd");
  poison_output("vc.vadd", const_cast<void *>(pc), bytes, s, {{pa, bytes}, {pb, bytes}});
  return run(vadd_maybe_checked((const float *)pa, (const float *)pb, (float *)pc, cnt, s, "vc.vadd"),
             "vc.vadd");
}

VCError sum_common(const float *x, const float *b, float *c, long long cnt, double *out,
                   cudaStream_t s, const char *name) {
  double *partials;
  unsigned int *ticket;
  int cap;
  cudaError_t e = vcb::reduce_scratch(s, &partials, &ticket, &cap);
  if (e != cudaSuccess) return run(e, name);
  const size_t bytes = (size_t)cnt * 4;
  poison_output(name, out, 8, s, {{x, bytes}, {b, b ? bytes : 0}, {c, c ? bytes : 0}});
  if (c) poison_output(name, c, bytes, s, {{x, bytes}, {b, bytes}});
  return run(vcb::launch_sum_f32(x, b, c, cnt, out, partials, ticket, cap, s), name);
}

VCError k_native_sum(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n, cudaStream_t s) {
  const void *x, *out;
  long long cnt;
  if (!arg_ptr(a, n, 0, &x) || !arg_i64(a, n, 1, &cnt) || !arg_ptr(a, n, 2, &out) || n != 3 ||
      cnt < 0)
    return bad_args("vc.sum");
  if ((size_t)cnt * 4 > bytes_available(x) || 8 > bytes_available(out)) return too_small("vc.sum");
  return sum_common((const float *)x, nullptr, nullptr, cnt, (double *)out, s, "vc.sum");
}

VCError k_native_vadd_sum(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n,
                          cudaStream_t s) {
  const void *pa, *pb, *pc, *out;
  long long cnt;
  if (!arg_ptr(a, n, 0, &pa) || !arg_ptr(a, n, 1, &pb) || !arg_ptr(a, n, 2, &pc) ||
      !arg_i64(a, n, 3, &cnt) || !arg_ptr(a, n, 4, &out) || n != 5 || cnt < 0)
    return bad_args("vc.vadd_sum");
  const size_t bytes = (size_t)cnt * 4;
  if (bytes > bytes_available(pa) || bytes > bytes_available(pb) || bytes > bytes_available(pc) ||
      8 > bytes_available(out))
    return too_small("vc.vadd_sum");
  return sum_common((const float *)pa, (const float *)pb, (float *)pc, cnt, (double *)out, s,
                    "vc.vadd_sum");
}

VCError k_native_block_reduce(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n,
                              cudaStream_t s) {
  const void *pin, *pout;
  long long N, block, groups;
  if (!arg_ptr(a, n, 0, &pin) || !arg_ptr(a, n, 1, &pout) || !arg_i64(a, n, 2, &N) ||
      !arg_i64(a, n, 3, &block) || !arg_i64(a, n, 4, &groups) || n != 5)
    return bad_args("vc.block_reduce");
  if (block <= 0 || block > 1024 || groups <= 0) return bad_args("vc.block_reduce");
  if ((size_t)groups * 4 > bytes_available(pout)) return too_small("vc.block_reduce");
  poison_output("vc.block_reduce", const_cast<void *>(pout), (size_t)groups * 4, s,
                {{pin, N > 0 ? (size_t)N * 4 : 0}});
  return run(block_reduce_maybe_checked((const float *)pin, (float *)pout, (int)N, (int)block,
                                        (int)groups, s, "vc.block_reduce"),
             "vc.block_reduce");
}

VCError gemm_checked(const vcb::GemmArgs &g, int dtype, cudaStream_t s) {
  if (dtype != VC_DTYPE_F16 && dtype != VC_DTYPE_BF16 && dtype != VC_DTYPE_F32)
    return VCError::InvalidValue;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return VCError::InvalidValue;
  if (g.lda < g.K || g.ldd < g.N || (g.b_kn ? g.ldb < g.N : g.ldb < g.K)) return VCError::InvalidValue;
  if (g.Cin && g.ldc < g.N) return VCError::InvalidValue;
  const size_t esz = dtype == VC_DTYPE_F32 ? 4 : 2;
  const size_t a_need = ((size_t)(g.M - 1) * g.lda + g.K) * esz;
  const size_t b_need = g.b_kn ? ((size_t)(g.K - 1) * g.ldb + g.N) * esz
                               : ((size_t)(g.N - 1) * g.ldb + g.K) * esz;
  const size_t d_need = ((size_t)(g.M - 1) * g.ldd + g.N) * 4;
  if (a_need > bytes_available(g.A) || b_need > bytes_available(g.B) || d_need > bytes_available(g.D))
    return too_small("vc.gemm");
  if (g.Cin && ((size_t)(g.M - 1) * g.ldc + g.N) * 4 > bytes_available(g.Cin))
    return too_small("vc.gemm");
  if (dtype == VC_DTYPE_F32) return gemm_f32_dispatch(g, s, "vc.gemm");
  return gemm_dispatch(g, s, "vc.gemm");
}

VCError k_native_gemm(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n, cudaStream_t s) {
  const void *A, *B, *D, *Cin;
  long long M, N, K, lda, ldb, ldd, ldc, dtype, b_kn;
  if (n != 13 || !arg_ptr(a, n, 0, &A) || !arg_ptr(a, n, 1, &B) || !arg_ptr(a, n, 2, &D) ||
      !arg_ptr(a, n, 3, &Cin) || !arg_i64(a, n, 4, &M) || !arg_i64(a, n, 5, &N) ||
      !arg_i64(a, n, 6, &K) || !arg_i64(a, n, 7, &lda) || !arg_i64(a, n, 8, &ldb) ||
      !arg_i64(a, n, 9, &ldd) || !arg_i64(a, n, 10, &ldc) || !arg_i64(a, n, 11, &dtype) ||
      !arg_i64(a, n, 12, &b_kn))
    return bad_args("vc.gemm");
  vcb::GemmArgs g{A, B, (float *)D, (const float *)Cin, (int)M, (int)N, (int)K, lda, ldb, ldd,
                  ldc, dtype == VC_DTYPE_BF16, b_kn != 0};
  return gemm_checked(g, (int)dtype, s);
}

VCError flash_checked(const vcb::FlashArgs &f, cudaStream_t s) {
  if (f.BH <= 0 || f.N <= 0 || f.d <= 0) return VCError::InvalidValue;
  const size_t esz = f.dtype == VC_DTYPE_F32 ? 4 : 2;
  const size_t bytes = (size_t)f.BH * f.N * f.d * esz;
  for (const void *p : {f.Q, f.K, f.V, (const void *)f.O})
    if (!p || bytes > bytes_available(p)) return too_small("vc.flash_fwd");
  poison_output("vc.flash_fwd", f.O, bytes, s, {{f.Q, bytes}, {f.K, bytes}, {f.V, bytes}});
  if (f.dtype == VC_DTYPE_F32) return run(vcb::launch_flash_fwd_f32(f, s), "vc.flash_fwd");
  if (f.dtype == VC_DTYPE_F16 || f.dtype == VC_DTYPE_BF16)
    return run(vcb::launch_flash_fwd_tcgen05(f, s), "vc.flash_fwd");
  return VCError::InvalidValue;
}

VCError k_native_flash(VCKernel &, const LaunchShape &, const VCKernelArg *a, int n, cudaStream_t s) {
  const void *Q, *K, *V, *O;
  long long BH, N, d, causal, dtype;
  float scale;
  if (n != 10 || !arg_ptr(a, n, 0, &Q) || !arg_ptr(a, n, 1, &K) || !arg_ptr(a, n, 2, &V) ||
      !arg_ptr(a, n, 3, &O) || !arg_i64(a, n, 4, &BH) || !arg_i64(a, n, 5, &N) ||
      !arg_i64(a, n, 6, &d) || !arg_f32(a, n, 7, &scale) || !arg_i64(a, n, 8, &causal) ||
      !arg_i64(a, n, 9, &dtype))
    return bad_args("vc.flash_fwd");
  vcb::FlashArgs f{Q, K, V, const_cast<void *>(O), (int)BH, (int)N, (int)d, scale, causal != 0,
                   (int)dtype};
  return flash_checked(f, s);
}

const std::vector<KernelEntry> &registry() {
  static const std::vector<KernelEntry> r = {
      {"vadd", k_vadd, {}},
      {"blockReduce", k_block_reduce, {}},
      {"fillPattern", k_fill_pattern, {}},
      {"flashAttn", k_flash_attn, {{"NHEAD", 2}, {"SEQ", 64}, {"HDIM", 16}, {"BR", 16}, {"BC", 16}}},
      {"wmma_gemm", k_wmma_gemm, {}},
      {"matmulCoopmat", k_matmul_coopmat, {{"L", 1024}}},
      {"matmulTiled", k_matmul_tiled, {}},
      {"matmul", k_matmul_tiled, {}},  // test/matmul.vc: the same contract
      {"vc.vadd", k_native_vadd, {}},
      {"vc.sum", k_native_sum, {}},
      {"vc.vadd_sum", k_native_vadd_sum, {}},
      {"vc.block_reduce", k_native_block_reduce, {}},
      {"vc.gemm", k_native_gemm, {}},
      {"vc.flash_fwd", k_native_flash, {}},
  };
  return r;
}

const KernelEntry *find_entry(const char *name) {
  if (!name) return nullptr;
  for (const auto &e : registry())
    if (std::strcmp(e.name, name) == 0) return &e;
  return nullptr;
}

VCKernel *make_kernel(const KernelEntry *e) {
  auto *k = new VCKernel();
  k->entry = e;
  for (auto &c : e->constants) k->constants[c.first] = c.second;
  return k;
}

// ---- GLSL-backend modules (entry "main"): which demo kernel is this?
// The VC compiler's GLSL backend gives every pointer parameter its own storage
// buffer block `layout(set = 0, binding = i) buffer Bi { T name[]; }` in
// parameter order and gathers the scalar parameters, in order, into one push
// constant block (lib/Codegen/ASTToGLSL.cpp:955-1008); glslc keeps those
// member names in the module (OpMemberName). The module's interface, read
// back here as "name:type,... ; name:type,..." (storage buffers by binding,
// then push constants), identifies the demo kernel it was compiled from.
struct SpvInterfaceReader {
  std::map<uint32_t, std::map<uint32_t, std::string>> member_names;  // struct -> member -> name
  std::map<uint32_t, std::vector<uint32_t>> struct_members;          // struct -> member type ids
  std::map<uint32_t, std::string> scalar_types;                      // id -> "f32" / "i32" / ...
  std::map<uint32_t, uint32_t> runtime_array_elem;                   // id -> element type
  std::map<uint32_t, std::pair<uint32_t, uint32_t>> pointers;        // id -> (storage class, type)
  std::map<uint32_t, uint32_t> bindings;                             // variable -> binding
  std::vector<std::pair<uint32_t, uint32_t>> variables;              // (pointer type, id)

  static std::string literal(const uint32_t *w, size_t n) {
    std::string out;
    for (size_t i = 0; i < n; ++i)
      for (int b = 0; b < 4; ++b) {
        const char c = static_cast<char>((w[i] >> (8 * b)) & 0xFFu);
        if (!c) return out;
        out.push_back(c);
      }
    return out;
  }

  bool read(const uint32_t *words, size_t count) {
    for (size_t i = 5; i < count;) {
      const uint32_t op = words[i] & 0xFFFFu, wc = words[i] >> 16;
      if (wc == 0 || i + wc > count) return false;
      const uint32_t *a = words + i + 1;
      const size_t na = wc - 1;
      switch (op) {
        case 6:  // OpMemberName
          if (na >= 3) member_names[a[0]][a[1]] = literal(a + 2, na - 2);
          break;
        case 21:  // OpTypeInt
          if (na >= 3) scalar_types[a[0]] = (a[2] ? "i" : "u") + std::to_string(a[1]);
          break;
        case 22:  // OpTypeFloat
          if (na >= 2) scalar_types[a[0]] = "f" + std::to_string(a[1]);
          break;
        case 29:  // OpTypeRuntimeArray
          if (na >= 2) runtime_array_elem[a[0]] = a[1];
          break;
        case 30:  // OpTypeStruct
          if (na >= 1) struct_members[a[0]].assign(a + 1, a + na);
          break;
        case 32:  // OpTypePointer
          if (na >= 3) pointers[a[0]] = {a[1], a[2]};
          break;
        case 59:  // OpVariable
          if (na >= 3) variables.push_back({a[0], a[1]});
          break;
        case 71:  // OpDecorate ... Binding
          if (na >= 3 && a[1] == 33u) bindings[a[0]] = a[2];
          break;
        default:
          break;
      }
      i += wc;
    }
    return true;
  }

  // A scalar type, or a runtime array of one (one level only: a malformed
  // module may declare an array of itself).
  std::string type_name(uint32_t id) const {
    auto ra = runtime_array_elem.find(id);
    if (ra != runtime_array_elem.end()) id = ra->second;
    auto it = scalar_types.find(id);
    return it != scalar_types.end() ? it->second : "?";
  }

  // "a:f32,b:f32,c:f32;n:i32" (storage buffers by binding; push constants).
  std::string signature() const {
    std::map<uint32_t, std::string> buffers;  // binding -> "name:type"
    std::string push;
    for (const auto &v : variables) {
      auto pt = pointers.find(v.first);
      if (pt == pointers.end()) continue;
      const uint32_t storage = pt->second.first, st = pt->second.second;
      auto sm = struct_members.find(st);
      if (sm == struct_members.end()) continue;
      auto names = member_names.find(st);
      auto member = [&](size_t m) {
        std::string nm = "?";
        if (names != member_names.end()) {
          auto it = names->second.find(static_cast<uint32_t>(m));
          if (it != names->second.end()) nm = it->second;
        }
        return nm + ":" + type_name(sm->second[m]);
      };
      if (storage == 12u || storage == 2u) {  // StorageBuffer, or Uniform + BufferBlock
        auto b = bindings.find(v.second);
        if (b != bindings.end() && sm->second.size() == 1) buffers[b->second] = member(0);
      } else if (storage == 9u) {  // PushConstant
        for (size_t m = 0; m < sm->second.size(); ++m) push += (m ? "," : "") + member(m);
      }
    }
    std::string out;
    for (const auto &b : buffers) out += (out.empty() ? "" : ",") + b.second;
    return out + ";" + push;
  }
};

// Interfaces of the demo kernels as their GLSL modules carry them.
const char *glsl_kernel_for(const std::string &sig) {
  static const std::pair<const char *, const char *> table[] = {
      {"a:f32,b:f32,c:f32;n:i32", "vadd"},                       // test/vadd.vc:12
      {"inBuf:f32,outBuf:f32;N:i32", "blockReduce"},             // test/reduce.vc:11
      {"Q:f32,K:f32,V:f32,O:f32;scale:f32,causal:i32", "flashAttn"},  // flash_attn.vc:56
      {"A:f32,B:f32,C:f32;N:i32", "matmulTiled"},                // matmul_bench.vc:22, test/matmul.vc:12
      {"a:i32;base:i32,n:i32", "fillPattern"},                   // test/multigpu.vc:24
  };
  for (const auto &t : table)
    if (sig == t.first) return t.second;
  return nullptr;
}

uint64_t fnv1a64(const uint32_t *w, size_t n) {
  uint64_t h = 1469598103934665603ull;
  const uint8_t *p = reinterpret_cast<const uint8_t *>(w);
  for (size_t i = 0; i < n * 4; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

}  // namespace

namespace vc {

VCError vcGetKernel(const char *name, VCKernelHandle *outKernel) {
  if (!outKernel || !name) return VCError::InvalidValue;
  const KernelEntry *e = find_entry(name);
  if (!e) {
    std::fprintf(stderr, "vc: no kernel named '%s' in the registry\n", name);
    return VCError::InvalidKernel;
  }
  *outKernel = make_kernel(e);
  return VCError::Success;
}

// The reference refuses, with InvalidValue, any module that is missing, shorter
// than the 5-word SPIR-V header or without the SPIR-V magic number, before it
// looks at the entry point (lib/Runtime/VCRuntime.cpp:4261-4268). Callers that
// hold no module resolve a kernel by name with vcGetKernel instead.
VCError vcLoadKernel(const uint32_t *spirvWords, size_t wordCount, const char *entryPoint,
                     VCKernelHandle *outKernel) {
  if (!outKernel) return VCError::InvalidValue;
  if (!spirvWords || wordCount < 5 || spirvWords[0] != 0x07230203u) {
    std::fprintf(stderr,
                 "vc: kernel '%s': input is not a SPIR-V binary (no 0x07230203 magic word)\n",
                 entryPoint ? entryPoint : "?");
    return VCError::InvalidValue;
  }
  const char *name = entryPoint ? entryPoint : "main";
  const KernelEntry *e = find_entry(name);
  if (!e && std::strcmp(name, "main") == 0) {
    // A GLSL-backend module: identify the kernel by its interface.
    SpvInterfaceReader reader;
    const std::string sig = reader.read(spirvWords, wordCount) ? reader.signature() : "";
    const char *kernel = sig.empty() ? nullptr : glsl_kernel_for(sig);
    if (kernel) {
      e = find_entry(kernel);
      const char *dbg = std::getenv("VC_DEBUG");  // loading needs no vcInit
      if (st().debug || (dbg && std::atoi(dbg) != 0))
        std::fprintf(stderr, "vc: module 'main' with interface %s is %s\n", sig.c_str(), kernel);
    } else {
      std::fprintf(stderr,
                   "vc: entry 'main': interface '%s' (module fingerprint %016llx) matches no "
                   "kernel here\n",
                   sig.c_str(), (unsigned long long)fnv1a64(spirvWords, wordCount));
      return VCError::InvalidKernel;
    }
  }
  if (!e) {
    std::fprintf(stderr, "vc: no kernel named '%s' in the registry\n", name);
    return VCError::InvalidKernel;
  }
  *outKernel = make_kernel(e);
  return VCError::Success;
}

VCError vcLoadKernelFromFile(const char *path, const char *entryPoint, VCKernelHandle *outKernel) {
  if (!outKernel || !path) return VCError::InvalidValue;
  std::ifstream f(path, std::ios::binary);
  if (!f) return VCError::InvalidValue;
  std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  // Whole words, the last one zero-padded, as the reference reads a file
  // (VCRuntime.cpp:4378-4387); vcLoadKernel then judges the module.
  std::vector<uint32_t> words((bytes.size() + 3) / 4, 0u);
  if (!bytes.empty()) std::memcpy(words.data(), bytes.data(), bytes.size());
  return vcLoadKernel(words.data(), words.size(), entryPoint, outKernel);
}

VCError vcReleaseKernel(VCKernelHandle kernel) {
  delete kernel;
  return VCError::Success;
}

VCError vcKernelSetConstant(VCKernelHandle kernel, const char *name, long long value) {
  if (!kernel || !name) return VCError::InvalidValue;
  auto it = kernel->constants.find(name);
  if (it == kernel->constants.end()) return VCError::InvalidValue;
  if (value <= 0) return VCError::InvalidValue;
  it->second = value;
  return VCError::Success;
}

VCError vcLaunchKernel2DS(VCKernelHandle kernel, unsigned gridDimX, unsigned gridDimY,
                          unsigned blockDimX, unsigned blockDimY, const VCKernelArg *args,
                          int argCount, VCStreamHandle stream) {
  if (!kernel || !kernel->entry) return VCError::InvalidKernel;
  if (blockDimX == 0 || blockDimY == 0 || argCount < 0 || (argCount > 0 && !args))
    return VCError::InvalidValue;
  if (inject_fault("launch")) return VCError::Unknown;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  LaunchShape sh{(gridDimX + blockDimX - 1) / blockDimX, (gridDimY + blockDimY - 1) / blockDimY,
                 blockDimX, blockDimY};
  cudaStream_t s = resolve_stream(stream);
  ProfileScope prof(kernel->entry->name, s);
  return kernel->entry->launch(*kernel, sh, args, argCount, s);
}

VCError vcLaunchKernelS(VCKernelHandle kernel, unsigned gridDim, unsigned blockDim,
                        const VCKernelArg *args, int argCount, VCStreamHandle stream) {
  return vcLaunchKernel2DS(kernel, gridDim, 1, blockDim, 1, args, argCount, stream);
}

VCError vcLaunchKernel(VCKernelHandle kernel, unsigned gridDim, unsigned blockDim,
                       const VCKernelArg *args, int argCount) {
  return vcLaunchKernelS(kernel, gridDim, blockDim, args, argCount, nullptr);
}

VCError vcLaunchKernel2D(VCKernelHandle kernel, unsigned gridDimX, unsigned gridDimY,
                         unsigned blockDimX, unsigned blockDimY, const VCKernelArg *args,
                         int argCount) {
  return vcLaunchKernel2DS(kernel, gridDimX, gridDimY, blockDimX, blockDimY, args, argCount,
                           nullptr);
}

VCError vcLaunchKernelIndirectS(VCKernelHandle kernel, void *indirectArgs, size_t offset,
                                unsigned blockX, unsigned blockY, unsigned blockZ,
                                const VCKernelArg *args, int argCount, VCStreamHandle stream) {
  if (!kernel) return VCError::InvalidKernel;
  if (!indirectArgs || blockZ == 0) return VCError::InvalidValue;
  if (offset + 12 > bytes_available(indirectArgs)) return VCError::InvalidValue;
  if (!ensure_init()) return VCError::InitializationError;
  use_current_device();
  cudaStream_t s = resolve_stream(stream);
  uint32_t wg[3] = {0, 0, 0};
  VCError e = map_cuda(cudaMemcpyAsync(wg, static_cast<char *>(indirectArgs) + offset, 12,
                                       cudaMemcpyDeviceToHost, s), "indirect args");
  if (e == VCError::Success) e = wait_stream(s);
  if (e != VCError::Success) return e;
  if (wg[0] == 0 || wg[1] == 0 || wg[2] == 0) return VCError::Success;
  if (wg[2] != 1) return VCError::InvalidValue;
  return vcLaunchKernel2DS(kernel, wg[0] * blockX, wg[1] * blockY, blockX, blockY, args,
                           argCount, stream);
}

VCError vcLaunchKernelIndirect(VCKernelHandle kernel, void *indirectArgs, size_t offset,
                               unsigned blockX, unsigned blockY, unsigned blockZ,
                               const VCKernelArg *args, int argCount) {
  return vcLaunchKernelIndirectS(kernel, indirectArgs, offset, blockX, blockY, blockZ, args,
                                 argCount, nullptr);
}

}  // namespace vc

// ====================================================== runtime-owned scratch
namespace vcb {

cudaError_t reduce_scratch(cudaStream_t stream, double **partials, unsigned int **ticket,
                           int *capacity) {
  int dev = 0;
  cudaGetDevice(&dev);
  State &S = st();
  std::lock_guard<std::mutex> lk(S.mu);
  auto key = std::make_pair(dev, reinterpret_cast<void *>(stream));
  auto it = S.scratch.find(key);
  if (it == S.scratch.end()) {
    Scratch sc;
    sc.capacity = stream_max_blocks();
    cudaError_t e = cudaMalloc(&sc.partials, sizeof(double) * sc.capacity);
    if (e != cudaSuccess) return e;
    e = cudaMalloc(&sc.ticket, sizeof(unsigned int));
    if (e != cudaSuccess) { cudaFree(sc.partials); return e; }
    e = cudaMemset(sc.ticket, 0, sizeof(unsigned int));
    if (e != cudaSuccess) return e;
    it = S.scratch.emplace(key, sc).first;
  }
  *partials = it->second.partials;
  *ticket = it->second.ticket;
  *capacity = it->second.capacity;
  return cudaSuccess;
}

void *tensor_map_encoder() {
  static void *fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                         cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
  });
  return fn;
}

}  // namespace vcb

// ================================================================ flat C ABI
extern "C" {

static inline int E(VCError e) { return static_cast<int>(e); }
static inline VCStreamHandle S(void *s) { return reinterpret_cast<VCStreamHandle>(s); }

int vc_init(void) { return E(vcInit()); }
int vc_shutdown(void) { return E(vcShutdown()); }
int vc_get_device_count(int *count) { return E(vcGetDeviceCount(count)); }
int vc_get_device(int *device) { return E(vcGetDevice(device)); }
int vc_set_device(int device) { return E(vcSetDevice(device)); }
int vc_get_device_properties(vc_device_properties *out, int device) {
  static_assert(sizeof(vc_device_properties) == sizeof(VCDeviceProperties), "layout");
  return E(vcGetDeviceProperties(reinterpret_cast<VCDeviceProperties *>(out), device));
}
int vc_occupancy_max_potential_block_size(int *minGridSize, int *blockSize, void *kernel,
                                          size_t dynSmem, int blockSizeLimit) {
  return E(vcOccupancyMaxPotentialBlockSize(minGridSize, blockSize,
                                            static_cast<VCKernelHandle>(kernel), dynSmem,
                                            blockSizeLimit));
}
int vc_pointer_get_attributes(vc_pointer_attributes *out, const void *ptr) {
  static_assert(sizeof(vc_pointer_attributes) == sizeof(VCPointerAttributes), "layout");
  if (!out) return E(VCError::InvalidValue);
  VCPointerAttributes a;
  VCError e = vcPointerGetAttributes(&a, ptr);
  out->memoryType = static_cast<int>(a.memoryType);
  out->devicePointer = a.devicePointer;
  out->hostPointer = a.hostPointer;
  out->size = a.size;
  return E(e);
}
int vc_malloc(void **p, size_t bytes) { return E(vcMalloc(p, bytes)); }
int vc_malloc_host(void **p, size_t bytes) { return E(vcMallocHost(p, bytes)); }
int vc_malloc_managed(void **p, size_t bytes) { return E(vcMallocManaged(p, bytes)); }
int vc_free(void *p) { return E(vcFree(p)); }
int vc_malloc_async(void **p, size_t bytes, void *s) { return E(vcMallocAsync(p, bytes, S(s))); }
int vc_free_async(void *p, void *s) { return E(vcFreeAsync(p, S(s))); }
static bool kind_ok(int k) { return k >= 0 && k <= 2; }
int vc_memcpy(void *dst, const void *src, size_t count, int kind) {
  if (!kind_ok(kind)) return E(VCError::InvalidValue);
  return E(vcMemcpy(dst, src, count, static_cast<VCMemcpyKind>(kind)));
}
int vc_memcpy_s(void *dst, const void *src, size_t count, int kind, void *s) {
  if (!kind_ok(kind)) return E(VCError::InvalidValue);
  return E(vcMemcpyS(dst, src, count, static_cast<VCMemcpyKind>(kind), S(s)));
}
int vc_memcpy_async_s(void *dst, const void *src, size_t count, int kind, void *s) {
  if (!kind_ok(kind)) return E(VCError::InvalidValue);
  return E(vcMemcpyAsyncS(dst, src, count, static_cast<VCMemcpyKind>(kind), S(s)));
}
int vc_memcpy_async(void *dst, const void *src, size_t count, int kind) {
  if (!kind_ok(kind)) return E(VCError::InvalidValue);
  return E(vcMemcpyAsync(dst, src, count, static_cast<VCMemcpyKind>(kind)));
}
int vc_memcpy_peer(void *dst, int dd, const void *src, int sd, size_t bytes) {
  return E(vcMemcpyPeer(dst, dd, src, sd, bytes));
}
int vc_memcpy_peer_async(void *dst, int dd, const void *src, int sd, size_t bytes, void *s) {
  return E(vcMemcpyPeerAsync(dst, dd, src, sd, bytes, S(s)));
}
int vc_memset(void *p, int v, size_t count) { return E(vcMemset(p, v, count)); }
int vc_memset_async_s(void *p, int v, size_t count, void *s) { return E(vcMemsetAsyncS(p, v, count, S(s))); }
int vc_memcpy_2d_async(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width,
                       size_t height, int kind, void *s) {
  if (!kind_ok(kind)) return E(VCError::InvalidValue);
  return E(vcMemcpy2DAsync(dst, dpitch, src, spitch, width, height,
                           static_cast<VCMemcpyKind>(kind), S(s)));
}
int vc_memset_2d_async(void *dst, size_t pitch, int v, size_t width, size_t height, void *s) {
  return E(vcMemset2DAsync(dst, pitch, v, width, height, S(s)));
}
int vc_device_synchronize(void) { return E(vcDeviceSynchronize()); }
int vc_stream_create(void **out) {
  return E(vcStreamCreate(reinterpret_cast<VCStreamHandle *>(out)));
}
int vc_stream_destroy(void *s) { return E(vcStreamDestroy(S(s))); }
int vc_stream_synchronize(void *s) { return E(vcStreamSynchronize(S(s))); }
int vc_stream_query(void *s, int *done) { return E(vcStreamQuery(S(s), done)); }
int vc_launch_host_func(void *s, void (*fn)(void *), void *user) {
  return E(vcLaunchHostFunc(S(s), fn, user));
}
int vc_event_create(void **out) { return E(vcEventCreate(reinterpret_cast<VCEventHandle *>(out))); }
int vc_event_destroy(void *ev) { return E(vcEventDestroy(static_cast<VCEventHandle>(ev))); }
int vc_event_record(void *ev, void *s) { return E(vcEventRecord(static_cast<VCEventHandle>(ev), S(s))); }
int vc_stream_wait_event(void *s, void *ev) {
  return E(vcStreamWaitEvent(S(s), static_cast<VCEventHandle>(ev)));
}
int vc_event_query(void *ev, int *done) { return E(vcEventQuery(static_cast<VCEventHandle>(ev), done)); }
int vc_event_synchronize(void *ev) { return E(vcEventSynchronize(static_cast<VCEventHandle>(ev))); }
int vc_event_elapsed_time(float *ms, void *a, void *b) {
  return E(vcEventElapsedTime(ms, static_cast<VCEventHandle>(a), static_cast<VCEventHandle>(b)));
}
int vc_graph_create(void **out) { return E(vcGraphCreate(reinterpret_cast<VCGraphHandle *>(out))); }
int vc_graph_destroy(void *g) { return E(vcGraphDestroy(static_cast<VCGraphHandle>(g))); }
int vc_graph_begin_record(void *g) { return E(vcGraphBeginRecord(static_cast<VCGraphHandle>(g))); }
int vc_graph_end_record(void *g) { return E(vcGraphEndRecord(static_cast<VCGraphHandle>(g))); }
int vc_graph_launch(void *g, void *s) { return E(vcGraphLaunch(static_cast<VCGraphHandle>(g), S(s))); }
int vc_graph_reset(void *g) { return E(vcGraphReset(static_cast<VCGraphHandle>(g))); }
int vc_load_kernel(const uint32_t *words, size_t n, const char *entry, void **out) {
  return E(vcLoadKernel(words, n, entry, reinterpret_cast<VCKernelHandle *>(out)));
}
int vc_load_kernel_from_file(const char *path, const char *entry, void **out) {
  return E(vcLoadKernelFromFile(path, entry, reinterpret_cast<VCKernelHandle *>(out)));
}
int vc_release_kernel(void *k) { return E(vcReleaseKernel(static_cast<VCKernelHandle>(k))); }
int vc_launch_kernel(void *k, unsigned grid, unsigned block, const vc_kernel_arg *args, int n) {
  static_assert(sizeof(vc_kernel_arg) == sizeof(VCKernelArg), "layout");
  return E(vcLaunchKernel(static_cast<VCKernelHandle>(k), grid, block,
                          reinterpret_cast<const VCKernelArg *>(args), n));
}
int vc_launch_kernel_s(void *k, unsigned grid, unsigned block, const vc_kernel_arg *args, int n,
                       void *s) {
  return E(vcLaunchKernelS(static_cast<VCKernelHandle>(k), grid, block,
                           reinterpret_cast<const VCKernelArg *>(args), n, S(s)));
}
int vc_launch_kernel_2d_s(void *k, unsigned gx, unsigned gy, unsigned bx, unsigned by,
                          const vc_kernel_arg *args, int n, void *s) {
  return E(vcLaunchKernel2DS(static_cast<VCKernelHandle>(k), gx, gy, bx, by,
                             reinterpret_cast<const VCKernelArg *>(args), n, S(s)));
}
int vc_launch_kernel_indirect_s(void *k, void *ind, size_t offset, unsigned bx, unsigned by,
                                unsigned bz, const vc_kernel_arg *args, int n, void *s) {
  return E(vcLaunchKernelIndirectS(static_cast<VCKernelHandle>(k), ind, offset, bx, by, bz,
                                   reinterpret_cast<const VCKernelArg *>(args), n, S(s)));
}
const char *vc_error_string(int err) {
  if (err < 0 || err > static_cast<int>(VCError::Unknown)) return "unknown error";
  return vcErrorString(static_cast<VCError>(err));
}
int vc_get_kernel(const char *name, void **out) {
  return E(vcGetKernel(name, reinterpret_cast<VCKernelHandle *>(out)));
}
int vc_kernel_set_constant(void *k, const char *name, long long value) {
  return E(vcKernelSetConstant(static_cast<VCKernelHandle>(k), name, value));
}
int vc_kernel_error(int clear) {
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  int codes[5] = {vcb::stream_kernels_error(clear), vcb::gemm_tcgen05_error(clear),
                  vcb::gemm_f32_error(clear), vcb::flash_tcgen05_error(clear),
                  vcb::selftest_error(clear)};
  for (int c : codes)
    if (c != 0) return c;
  return 0;
}
int vc_selftest_bounds_check(void) {
  if (!ensure_init()) return -1;
  use_current_device();
  // 1024 elements each, all of them real memory; the checked vadd is told c
  // holds 1000, so indices 1000..1023 must be refused on the device.
  constexpr int64_t kN = 1024, kLimit = 1000;
  float *buf = nullptr;
  if (cudaMalloc(&buf, 3 * kN * sizeof(float)) != cudaSuccess) return -1;
  float *a = buf, *b = buf + kN, *c = buf + 2 * kN;
  int rc = -1;
  std::vector<float> ha(kN), hc(kN);
  for (int64_t i = 0; i < kN; ++i) ha[i] = (float)i;
  vcb::stream_kernels_error(1);
  if (cudaMemcpy(a, ha.data(), kN * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
      cudaMemcpy(b, ha.data(), kN * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
      cudaMemset(c, 0xFF, kN * 4) == cudaSuccess &&
      vcb::launch_vadd_f32_checked(a, b, c, kN, kN, kN, kLimit, nullptr) == cudaSuccess &&
      cudaDeviceSynchronize() == cudaSuccess &&
      cudaMemcpy(hc.data(), c, kN * 4, cudaMemcpyDeviceToHost) == cudaSuccess) {
    rc = vcb::stream_kernels_error(1);  // expected: kErrOutOfBounds (4)
    for (int64_t i = 0; i < kN && rc == 4; ++i) {
      uint32_t bits;
      std::memcpy(&bits, &hc[i], 4);
      const bool want_written = i < kLimit;
      if (want_written ? hc[i] != 2.0f * (float)i : bits != 0xFFFFFFFFu) rc = 100;
    }
  }
  cudaFree(buf);
  return rc;
}
int vc_selftest_bounded_wait(unsigned timeout_us) {
  if (!ensure_init()) return -1;
  use_current_device();
  vcb::selftest_error(1);
  cudaError_t e = vcb::launch_selftest_bounded_wait(timeout_us, nullptr);
  if (e != cudaSuccess) return -1;
  if (cudaStreamSynchronize(nullptr) != cudaSuccess) return -1;
  return vcb::selftest_error(1);
}

int vc_vadd_f32(const float *a, const float *b, float *c, int64_t n, void *s) {
  if (!a || !b || !c || n < 0) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  const size_t bytes = (size_t)n * 4;
  poison_output("vc_vadd_f32", c, bytes, reinterpret_cast<cudaStream_t>(s), {{a, bytes}, {b, bytes}});
  return E(map_cuda(vadd_maybe_checked(a, b, c, n, reinterpret_cast<cudaStream_t>(s), "vc_vadd_f32"),
                    "vc_vadd_f32"));
}
int vc_sum_f32(const float *x, int64_t n, double *out, void *s) {
  if (!x || !out || n < 0) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  return E(sum_common(x, nullptr, nullptr, n, out, reinterpret_cast<cudaStream_t>(s), "vc_sum_f32"));
}
// No reference counterpart: vc_sum_f32 for callers that cannot allocate (see
// include/vc_b200.h). Same prologue and error mapping as vc_sum_f32; the
// scratch is the static device array of stream_kernels.cu.
int vc_sum_f32_noalloc(const float *x, int64_t n, double *out, void *s) {
  if (!x || !out || n < 0) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  int needed = 0;
  cudaError_t e = vcb::launch_sum_f32_noalloc(x, n, out, reinterpret_cast<cudaStream_t>(s), &needed);
  if (e == cudaErrorInvalidValue && needed > vcb::noalloc_sum_capacity()) {
    std::fprintf(stderr,
                 "vc_sum_f32_noalloc: this device needs %d block partials; the static scratch "
                 "holds %d\n", needed, vcb::noalloc_sum_capacity());
    return E(VCError::InvalidValue);
  }
  return E(map_cuda(e, "vc_sum_f32_noalloc"));
}
int vc_vadd_sum_f32(const float *a, const float *b, float *c, int64_t n, double *out, void *s) {
  if (!a || !b || !c || !out || n < 0) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  return E(sum_common(a, b, c, n, out, reinterpret_cast<cudaStream_t>(s), "vc_vadd_sum_f32"));
}
int vc_peer_mailbox_alloc(void **mailbox) {
  if (!mailbox) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, sizeof(vcb::PeerMailbox));
  if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(vcb::PeerMailbox));
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return E(map_cuda(e, "vc_peer_mailbox_alloc"));
  }
  *mailbox = p;
  return VC_SUCCESS;
}
int vc_peer_mailbox_free(void *mailbox) {
  if (!mailbox) return VC_SUCCESS;
  if (!ensure_init()) return E(VCError::InitializationError);
  return E(map_cuda(cudaFree(mailbox), "vc_peer_mailbox_free"));
}
int vc_peer_ipc_get_handle(const void *dev_ptr, void *handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == VC_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr));
  if (e != cudaSuccess) return E(map_cuda(e, "vc_peer_ipc_get_handle"));
  std::memcpy(handle, &h, sizeof(h));
  return VC_SUCCESS;
}
int vc_peer_ipc_open(const void *handle, void **dev_ptr) {
  if (!handle || !dev_ptr) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return E(map_cuda(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                    "vc_peer_ipc_open"));
}
int vc_peer_ipc_close(void *dev_ptr) {
  if (!dev_ptr) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  return E(map_cuda(cudaIpcCloseMemHandle(dev_ptr), "vc_peer_ipc_close"));
}
int vc_vadd_sum_f32_allreduce(const float *a, const float *b, float *c, int64_t n, double *out,
                              void *const *mailboxes, int rank, int world,
                              unsigned long long epoch, void *s) {
  if (!a || !b || !c || !out || n < 0 || !mailboxes || world < 1 ||
      world > vcb::kMaxPeers || rank < 0 || rank >= world || epoch == 0)
    return E(VCError::InvalidValue);
  vcb::PeerExchange px{};
  for (int i = 0; i < world; ++i) {
    if (!mailboxes[i]) return E(VCError::InvalidValue);
    px.mbox[i] = static_cast<vcb::PeerMailbox *>(mailboxes[i]);
  }
  px.rank = rank;
  px.world = world;
  px.epoch = epoch;
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
  double *partials;
  unsigned int *ticket;
  int cap;
  cudaError_t e = vcb::reduce_scratch(st, &partials, &ticket, &cap);
  if (e != cudaSuccess) return E(run(e, "vc_vadd_sum_f32_allreduce"));
  return E(run(vcb::launch_sum_f32(a, b, c, n, out, partials, ticket, cap, st, &px),
               "vc_vadd_sum_f32_allreduce"));
}
int vc_block_reduce_f32(const float *in, float *out, int n, int block, int groups, void *s) {
  if (!in || !out || n < 0 || block <= 0 || block > 1024 || groups <= 0) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  poison_output("vc_block_reduce_f32", out, (size_t)groups * 4, reinterpret_cast<cudaStream_t>(s),
                {{in, (size_t)n * 4}});
  return E(map_cuda(block_reduce_maybe_checked(in, out, n, block, groups,
                                               reinterpret_cast<cudaStream_t>(s),
                                               "vc_block_reduce_f32"),
                    "vc_block_reduce_f32"));
}
int vc_gemm(const void *A, const void *B, float *D, const float *Cin, int M, int N, int K,
            int64_t lda, int64_t ldb, int64_t ldd, int64_t ldc, int dtype, int b_kn, void *s) {
  if (!A || !B || !D) return E(VCError::InvalidValue);
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  vcb::GemmArgs g{A, B, D, Cin, M, N, K, lda, ldb, ldd, ldc, dtype == VC_DTYPE_BF16, b_kn != 0};
  return E(gemm_checked(g, dtype, reinterpret_cast<cudaStream_t>(s)));
}
int vc_flash_fwd(const void *Q, const void *K, const void *V, void *O, int BH, int N, int d,
                 float scale_log2, int causal, int dtype, void *s) {
  if (!ensure_init()) return E(VCError::InitializationError);
  use_current_device();
  vcb::FlashArgs f{Q, K, V, O, BH, N, d, scale_log2, causal != 0, dtype};
  return E(flash_checked(f, reinterpret_cast<cudaStream_t>(s)));
}

}  // extern "C"
