// TEST INFRASTRUCTURE.  Definition of the reference's C launcher
// (declared at src/attn_kernel.h:18-20 of JoursBleu/rocm_attn) that runs
// this repository's C oracle on host memory, so the reference's own
// known-answer test (src/tests/attn_test.cpp:51-98) checks the oracle
// against the reference's CPU attention (src/tests/attn_test.cpp:10-49).
#include "attn_kernel.h"

extern "C" void attn_oracle_forward(const float* q, const float* k, const float* v, float* out, int B, int H,
                                    int Sq, int Skv, int D, int causal, float scale);

extern "C" void launch_attn_forward(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq,
                                    int Skv, int D, bool causal, AttnDType dtype, hipStream_t) {
  if (dtype != ATTN_F32) return;  // the known-answer test is fp32 only
  attn_oracle_forward(static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
                      static_cast<float*>(out), B, H, Sq, Skv, D, causal ? 1 : 0, 0.f);
}
