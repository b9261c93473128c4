// A compiled C++ host program on the vc:: runtime API, written in the form the
// VC compiler's host emitter produces for test/vadd.vc (runtime header,
// `using namespace vc`, an embedded SPIR-V module per kernel, a lazily loaded
// kernel handle and a VCKernelArg launch; lib/Codegen/ASTToHost.cpp:238-248,
// 406-428, 1261-1318). It links against libVCRuntime.so unchanged and checks
// the demo's own condition: c[i] == a[i] + b[i] exactly (test/vadd.vc:40-43).
#include "vc/Runtime/VCRuntime.h"
#include <cstdio>
#include <cstring>
#include <cmath>
using namespace vc;

// SPIR-V module of the kernel (header, capability, memory model, entry point).
static const uint32_t __vc_spirv_vadd[] = {
  0x07230203, 0x00010000, 0x00000000, 0x00000002, 0x00000000, 0x00020011, 0x00000001, 0x0003000e,
  0x00000000, 0x00000001, 0x0005000f, 0x00000005, 0x00000001, 0x64646176, 0x00000000
};
static const size_t __vc_spirv_vadd_len = 15;
static VCKernelHandle __vc_k_vadd = nullptr;

int main() {
  vcInit();
  const int N = 64;
  float hA[64], hB[64], hC[64];
  for (int i = 0; i < N; i++) { hA[i] = 1.0f * i; hB[i] = 2.0f; }
  void *dA = 0, *dB = 0, *dC = 0;
  int bytes = N * 4;
  vcMalloc(&dA, bytes);
  vcMalloc(&dB, bytes);
  vcMalloc(&dC, bytes);
  vcMemcpy(dA, hA, bytes, VCMemcpyKind::HostToDevice);
  vcMemcpy(dB, hB, bytes, VCMemcpyKind::HostToDevice);
  {
    if (!__vc_k_vadd) vcLoadKernel(__vc_spirv_vadd, __vc_spirv_vadd_len, "vadd", &__vc_k_vadd);
    auto __vc_a3 = (N);
    VCKernelArg __args[4] = {{VCKernelArg::Pointer, dA, 0}, {VCKernelArg::Pointer, dB, 0},
                             {VCKernelArg::Pointer, dC, 0},
                             {VCKernelArg::Scalar, &__vc_a3, sizeof(__vc_a3)}};
    if (vcLaunchKernel(__vc_k_vadd, N, 32, __args, 4) != VCError::Success) {
      printf("vector_add: FAIL (launch)\n");
      return 1;
    }
  }
  vcDeviceSynchronize();
  vcMemcpy(hC, dC, bytes, VCMemcpyKind::DeviceToHost);
  int ok = 1;
  for (int i = 0; i < N; i++)
    if (hC[i] != hA[i] + hB[i]) ok = 0;
  printf("vector_add: %s\n", ok ? "PASS" : "FAIL");
  vcFree(dA);
  vcFree(dB);
  vcFree(dC);
  vcReleaseKernel(__vc_k_vadd);
  vcShutdown();
  return ok ? 0 : 1;
}
