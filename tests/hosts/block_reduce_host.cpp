// A compiled C++ host program on the vc:: runtime API in the form the VC
// compiler's host emitter produces for test/reduce.vc (see vadd_host.cpp).
// gridDim is an element count (N), the runtime launches ceil(N / block)
// workgroups, and each partial must equal the sequential float sum of its
// block exactly (test/reduce.vc:64-75). A second case runs 64-thread blocks
// over a ragged N (the last block partly empty).
#include "vc/Runtime/VCRuntime.h"
#include <cstdio>
#include <cstring>
#include <cmath>
#include <vector>
using namespace vc;

static const uint32_t __vc_spirv_blockReduce[] = {
  0x07230203, 0x00010000, 0x00000000, 0x00000002, 0x00000000, 0x00020011, 0x00000001, 0x0003000e,
  0x00000000, 0x00000001, 0x0006000f, 0x00000005, 0x00000001, 0x636f6c62, 0x6465526b, 0x00656375
};
static const size_t __vc_spirv_blockReduce_len = 16;
static VCKernelHandle __vc_k_blockReduce = nullptr;

static int runCase(int N, int block) {
  const int numBlocks = (N + block - 1) / block;
  std::vector<float> hIn(N), hOut(numBlocks, 0.0f);
  for (int i = 0; i < N; i++) hIn[i] = 1.0f * i;
  void *dIn = 0, *dOut = 0;
  vcMalloc(&dIn, N * 4);
  vcMalloc(&dOut, numBlocks * 4);
  vcMemcpy(dIn, hIn.data(), N * 4, VCMemcpyKind::HostToDevice);
  {
    if (!__vc_k_blockReduce)
      vcLoadKernel(__vc_spirv_blockReduce, __vc_spirv_blockReduce_len, "blockReduce",
                   &__vc_k_blockReduce);
    auto __vc_a2 = (N);
    VCKernelArg __args[3] = {{VCKernelArg::Pointer, dIn, 0}, {VCKernelArg::Pointer, dOut, 0},
                             {VCKernelArg::Scalar, &__vc_a2, sizeof(__vc_a2)}};
    if (vcLaunchKernel(__vc_k_blockReduce, N, block, __args, 3) != VCError::Success) return 0;
  }
  vcDeviceSynchronize();
  vcMemcpy(hOut.data(), dOut, numBlocks * 4, VCMemcpyKind::DeviceToHost);
  int ok = 1;
  for (int b = 0; b < numBlocks; b++) {
    int lo = b * block, hi = (b + 1) * block;
    if (hi > N) hi = N;
    float expect = 0.0f;
    for (int i = lo; i < hi; i++) expect += hIn[i];
    if (hOut[b] != expect) ok = 0;
  }
  vcFree(dIn);
  vcFree(dOut);
  return ok;
}

int main() {
  vcInit();
  int ok = runCase(128, 32) && runCase(1000, 64);
  printf("block_reduce: %s\n", ok ? "PASS" : "FAIL");
  vcReleaseKernel(__vc_k_blockReduce);
  vcShutdown();
  return ok ? 0 : 1;
}
