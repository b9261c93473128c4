// A compiled C++ host program on the vc:: runtime API in the form the VC
// compiler's host emitter produces for examples/matmul_coopmat_bench.vc (see
// vadd_host.cpp): fp16 A and B with row stride L = 1024 (:56), integer inputs
// (:138-143), grid ((N/16)*32, N/16) elements of 32-thread blocks (:116-117),
// the launch timed between two vcEvents on the default stream, and the N x N
// corner of C checked exactly against an fp64 loop (:168-184), for
// N = 128, 256, 512, 1024 (:225) after a warm-up launch.
#include "vc/Runtime/VCRuntime.h"
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>
using namespace vc;
using __half = _Float16;

#define L 1024
#define COOP_GX(N) (((N) / 16) * 32)
#define COOP_GY(N) ((N) / 16)

static const uint32_t __vc_spirv_matmulCoopmat[] = {
  0x07230203, 0x00010000, 0x00000000, 0x00000002, 0x00000000, 0x00020011, 0x00000001, 0x0003000e,
  0x00000000, 0x00000001, 0x0007000f, 0x00000005, 0x00000001, 0x6d74616d, 0x6f436c75, 0x616d706f,
  0x00000074
};
static const size_t __vc_spirv_matmulCoopmat_len = 17;
static VCKernelHandle __vc_k_matmulCoopmat = nullptr;

static VCError launch(void *dA, void *dB, void *dC, int N) {
  if (!__vc_k_matmulCoopmat)
    vcLoadKernel(__vc_spirv_matmulCoopmat, __vc_spirv_matmulCoopmat_len, "matmulCoopmat",
                 &__vc_k_matmulCoopmat);
  auto __vc_a3 = (N);
  VCKernelArg __args[4] = {{VCKernelArg::Pointer, dA, 0}, {VCKernelArg::Pointer, dB, 0},
                           {VCKernelArg::Pointer, dC, 0},
                           {VCKernelArg::Scalar, &__vc_a3, sizeof(__vc_a3)}};
  return vcLaunchKernel2D(__vc_k_matmulCoopmat, COOP_GX(N), COOP_GY(N), 32, 1, __args, 4);
}

static int runSize(int N) {
  int abytes = N * L * 2, cbytes = N * L * 4;
  __half *hA = (__half *)malloc(abytes);
  __half *hB = (__half *)malloc(abytes);
  float *hC = (float *)malloc(cbytes);
  for (int n = 0; n < N; n++)
    for (int m = 0; m < L; m++) {
      hA[n * L + m] = (__half)((n * 3 + m * 5) % 7);
      hB[n * L + m] = (__half)((n * 2 + m * 3) % 7);
    }
  void *dA = 0, *dB = 0, *dC = 0;
  vcMalloc(&dA, abytes);
  vcMalloc(&dB, abytes);
  vcMalloc(&dC, cbytes);
  vcMemcpy(dA, hA, abytes, VCMemcpyKind::HostToDevice);
  vcMemcpy(dB, hB, abytes, VCMemcpyKind::HostToDevice);
  VCEventHandle start = 0, end = 0;
  vcEventCreate(&start);
  vcEventCreate(&end);
  vcEventRecord(start, 0);
  VCError le = launch(dA, dB, dC, N);
  vcEventRecord(end, 0);
  vcEventSynchronize(end);
  float ms = 0.0f;
  VCError te = vcEventElapsedTime(&ms, start, end);
  vcEventDestroy(start);
  vcEventDestroy(end);
  vcMemcpy(hC, dC, cbytes, VCMemcpyKind::DeviceToHost);
  int ok = le == VCError::Success && te == VCError::Success;
  for (int n = 0; n < N && ok; n++)
    for (int m = 0; m < N; m++) {
      double ref = 0.0;
      for (int k = 0; k < N; k++) ref += (double)hA[n * L + k] * (double)hB[k * L + m];
      if (ref != (double)hC[n * L + m]) {
        printf("  N=%d [%d][%d] got %.1f want %.1f\n", N, n, m, (double)hC[n * L + m], ref);
        ok = 0;
        break;
      }
    }
  double gflops = te == VCError::Success ? 2.0 * N * (double)N * N / ((double)ms * 1e6) : 0.0;
  printf("  N=%4d  %8.4f ms   %8.2f GFLOPS   %s\n", N, ms, gflops, ok ? "PASS" : "FAIL");
  vcFree(dA);
  vcFree(dB);
  vcFree(dC);
  free(hA);
  free(hB);
  free(hC);
  return ok;
}

int main() {
  vcInit();
  {
    int w = 16, ab = w * L * 2, cb = w * L * 4;
    void *dA = 0, *dB = 0, *dC = 0;
    vcMalloc(&dA, ab);
    vcMalloc(&dB, ab);
    vcMalloc(&dC, cb);
    vcMemset(dA, 0, ab);
    vcMemset(dB, 0, ab);
    launch(dA, dB, dC, w);
    vcDeviceSynchronize();
    vcFree(dA);
    vcFree(dB);
    vcFree(dC);
  }
  int sizes[4] = {128, 256, 512, 1024};
  int allOk = 1;
  for (int i = 0; i < 4; i++)
    if (!runSize(sizes[i])) allOk = 0;
  printf("matmul_coopmat_bench: %s\n", allOk ? "PASS" : "FAIL");
  vcReleaseKernel(__vc_k_matmulCoopmat);
  vcShutdown();
  return allOk ? 0 : 1;
}
