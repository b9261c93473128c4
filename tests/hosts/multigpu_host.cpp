// A compiled C++ host program on the vc:: runtime API in the form the VC
// compiler's host emitter produces for test/multigpu.vc (see vadd_host.cpp):
// device count, current device 0, out-of-range vcSetDevice refused,
// fillPattern(base 1000) on device 0, vcMemcpyPeer 0 -> 0, and with two or
// more devices: vcMemcpyPeer 0 -> 1 over NVLink, fillPattern(base 2000) on
// device 1, and a device-1 buffer freed while device 0 is current
// (test/multigpu.vc:24-150). Prints which half ran.
#include "vc/Runtime/VCRuntime.h"
#include <cstdio>
#include <cstring>
#include <cmath>
using namespace vc;

static const uint32_t __vc_spirv_fillPattern[] = {
  0x07230203, 0x00010000, 0x00000000, 0x00000002, 0x00000000, 0x00020011, 0x00000001, 0x0003000e,
  0x00000000, 0x00000001, 0x0006000f, 0x00000005, 0x00000001, 0x6c6c6966, 0x74746150, 0x006e7265
};
static const size_t __vc_spirv_fillPattern_len = 16;
static VCKernelHandle __vc_k_fillPattern = nullptr;

static int fill(int *buf, int base, int n) {
  if (!__vc_k_fillPattern)
    vcLoadKernel(__vc_spirv_fillPattern, __vc_spirv_fillPattern_len, "fillPattern",
                 &__vc_k_fillPattern);
  auto __vc_a1 = (base);
  auto __vc_a2 = (n);
  VCKernelArg __args[3] = {{VCKernelArg::Pointer, buf, 0},
                           {VCKernelArg::Scalar, &__vc_a1, sizeof(__vc_a1)},
                           {VCKernelArg::Scalar, &__vc_a2, sizeof(__vc_a2)}};
  return vcLaunchKernel(__vc_k_fillPattern, (n + 255) / 256 * 256, 256, __args, 3) ==
         VCError::Success;
}

static int fail(const char *why) {
  printf("multigpu: FAIL (%s)\n", why);
  vcShutdown();
  return 1;
}

int main() {
  vcInit();
  int devCount = 0;
  if (vcGetDeviceCount(&devCount) != VCError::Success || devCount < 1) return fail("no devices");
  printf("device count: %d\n", devCount);
  int cur = -1;
  if (vcGetDevice(&cur) != VCError::Success || cur != 0) return fail("default device != 0");
  if (vcSetDevice(devCount) == VCError::Success) return fail("out-of-range device accepted");
  if (vcSetDevice(0) != VCError::Success) return fail("vcSetDevice(0)");
  const int N = 1024;
  const size_t bytes = N * sizeof(int);
  int *buf0 = 0, *buf0b = 0;
  if (vcMalloc((void **)&buf0, bytes) != VCError::Success) return fail("malloc device 0");
  if (!fill(buf0, 1000, N)) return fail("launch device 0");
  vcDeviceSynchronize();
  vcMalloc((void **)&buf0b, bytes);
  if (vcMemcpyPeer(buf0b, 0, buf0, 0, bytes) != VCError::Success) return fail("peer copy 0->0");
  int check[N];
  vcMemcpy(check, buf0b, bytes, VCMemcpyKind::DeviceToHost);
  for (int i = 0; i < N; ++i)
    if (check[i] != 1000 + i) return fail("peer 0->0 data");
  if (devCount >= 2) {
    vcSetDevice(1);
    int *buf1 = 0;
    if (vcMalloc((void **)&buf1, bytes) != VCError::Success) return fail("malloc device 1");
    if (vcMemcpyPeer(buf1, 1, buf0, 0, bytes) != VCError::Success) return fail("peer copy 0->1");
    vcMemcpy(check, buf1, bytes, VCMemcpyKind::DeviceToHost);
    for (int i = 0; i < N; ++i)
      if (check[i] != 1000 + i) return fail("peer 0->1 data");
    if (!fill(buf1, 2000, N)) return fail("launch device 1");
    vcDeviceSynchronize();
    vcMemcpy(check, buf1, bytes, VCMemcpyKind::DeviceToHost);
    for (int i = 0; i < N; ++i)
      if (check[i] != 2000 + i) return fail("device 1 launch data");
    vcSetDevice(0);
    if (vcFree(buf1) != VCError::Success) return fail("free device-1 buffer from device 0");
    printf("multigpu: 0->1 peer copy + device-1 launch verified\n");
  } else {
    printf("multigpu: single device, peer copy 0->0 verified\n");
  }
  vcSetDevice(0);
  vcFree(buf0);
  vcFree(buf0b);
  vcReleaseKernel(__vc_k_fillPattern);
  vcShutdown();
  printf("multigpu: PASS\n");
  return 0;
}
