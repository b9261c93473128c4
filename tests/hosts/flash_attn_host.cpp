// A compiled C++ host program on the vc:: runtime API in the form the VC
// compiler's host emitter produces for examples/flash_attn.vc (see
// vadd_host.cpp). Shapes are the demo's #defines (NHEAD 2, SEQ 64, HDIM 16,
// BR 16; flash_attn.vc:50-54), the grid is NHEAD*SEQ elements of block BR
// (:226), `scale` is in the exp2 domain (:211), and both cases (causal 0 and
// 1, seeds 12345 + causal, :202) must match the fp64 host reference within
// 1e-4 (:230-236). Inputs and the reference come from the oracle library
// (the demo's generator and referenceAttn restated in oracle/oracle.c).
#include "vc/Runtime/VCRuntime.h"
#include <cstdio>
#include <cstring>
#include <cmath>
using namespace vc;

extern "C" {
void oracle_fa_inputs(uint32_t seed, int64_t elems, float *Q, float *K, float *V);
void oracle_attention(const float *Q, const float *K, const float *V, float *O, int BH, int N,
                      int d, float scale_log2, int causal, int bh_begin, int bh_end,
                      int row_begin, int row_end, int threads);
}

#define SEQ 64
#define HDIM 16
#define NHEAD 2
#define BR 16

static const uint32_t __vc_spirv_flashAttn[] = {
  0x07230203, 0x00010000, 0x00000000, 0x00000002, 0x00000000, 0x00020011, 0x00000001, 0x0003000e,
  0x00000000, 0x00000001, 0x0006000f, 0x00000005, 0x00000001, 0x73616c66, 0x74744168, 0x0000006e
};
static const size_t __vc_spirv_flashAttn_len = 16;
static VCKernelHandle __vc_k_flashAttn = nullptr;

static int runCase(int causal) {
  const int ELEMS = NHEAD * SEQ * HDIM;
  static float hQ[ELEMS], hK[ELEMS], hV[ELEMS], hO[ELEMS], hRef[ELEMS];
  oracle_fa_inputs(12345u + (unsigned int)causal, ELEMS, hQ, hK, hV);
  float scale = float(1.4426950408889634 / std::sqrt(double(HDIM)));
  oracle_attention(hQ, hK, hV, hRef, NHEAD, SEQ, HDIM, scale, causal, 0, NHEAD, 0, SEQ, 1);
  void *dQ = 0, *dK = 0, *dV = 0, *dO = 0;
  int bytes = ELEMS * 4;
  vcMalloc(&dQ, bytes);
  vcMalloc(&dK, bytes);
  vcMalloc(&dV, bytes);
  vcMalloc(&dO, bytes);
  vcMemcpy(dQ, hQ, bytes, VCMemcpyKind::HostToDevice);
  vcMemcpy(dK, hK, bytes, VCMemcpyKind::HostToDevice);
  vcMemcpy(dV, hV, bytes, VCMemcpyKind::HostToDevice);
  {
    if (!__vc_k_flashAttn)
      vcLoadKernel(__vc_spirv_flashAttn, __vc_spirv_flashAttn_len, "flashAttn", &__vc_k_flashAttn);
    auto __vc_a4 = (scale);
    auto __vc_a5 = (causal);
    VCKernelArg __args[6] = {{VCKernelArg::Pointer, dQ, 0}, {VCKernelArg::Pointer, dK, 0},
                             {VCKernelArg::Pointer, dV, 0}, {VCKernelArg::Pointer, dO, 0},
                             {VCKernelArg::Scalar, &__vc_a4, sizeof(__vc_a4)},
                             {VCKernelArg::Scalar, &__vc_a5, sizeof(__vc_a5)}};
    if (vcLaunchKernel2D(__vc_k_flashAttn, NHEAD * SEQ, 1, BR, 1, __args, 6) != VCError::Success)
      return 0;
  }
  vcDeviceSynchronize();
  vcMemcpy(hO, dO, bytes, VCMemcpyKind::DeviceToHost);
  int ok = 1;
  float worst = 0.0f;
  for (int i = 0; i < ELEMS; i++) {
    float diff = std::fabs(double(hO[i] - hRef[i]));
    if (diff > worst) worst = diff;
    if (diff > 1.0e-4f) ok = 0;
  }
  printf("  causal=%d worst_abs_err=%.3e\n", causal, double(worst));
  vcFree(dQ);
  vcFree(dK);
  vcFree(dV);
  vcFree(dO);
  return ok;
}

int main() {
  vcInit();
  printf("flash_attn: heads=%d seq=%d dim=%d\n", NHEAD, SEQ, HDIM);
  int ok = 1;
  if (!runCase(0)) ok = 0;
  if (!runCase(1)) ok = 0;
  printf("flash_attn: %s\n", ok ? "PASS" : "FAIL");
  vcReleaseKernel(__vc_k_flashAttn);
  vcShutdown();
  return ok ? 0 : 1;
}
