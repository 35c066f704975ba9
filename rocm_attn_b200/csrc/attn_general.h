// Internal interface between the C ABI dispatcher (attn_kernel.cu) and the
// general attention kernel (attn_general.cu).
#pragma once

#include <cuda_runtime.h>

namespace ra {

// Largest head dimension the general kernel takes.
constexpr int kGeneralMaxHeadDim = 256;

// Attention forward on contiguous q [BH, Sq, D], k/v [BH, Skv, D] -> out
// [BH, Sq, D] in dtype 0 = fp16, 1 = bf16, 2 = fp32 (AttnDType values), fp32
// arithmetic, any 1 <= D <= kGeneralMaxHeadDim, Sq, Skv >= 1.  Returns 0 when
// the launch was queued, -1 otherwise.
int launch_attn_general(const void* q, const void* k, const void* v, void* out, int BH, int Sq, int Skv, int D,
                        bool causal, float scale, int dtype, cudaStream_t stream);

}  // namespace ra
