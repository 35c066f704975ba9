// Internal interface between the C ABI dispatcher (attn_kernel.cu) and the
// general attention kernel (attn_general.cu).
#pragma once

#include <cuda_runtime.h>

#include <vector>

namespace ra {

// Largest head dimension the general kernel takes.
constexpr int kGeneralMaxHeadDim = 256;

// Element strides of q, k and v over (batch, head, row); the head dim of each
// is contiguous.
struct GeneralStrides {
  long long q[3], k[3], v[3];
};

// Attention forward on q [B, H, Sq, D], k/v [B, H, Skv, D] (strided as
// given) -> out [B, H, Sq, D] contiguous, in dtype 0 = fp16, 1 = bf16,
// 2 = fp32 (AttnDType values), fp32 arithmetic, any 1 <= D <=
// kGeneralMaxHeadDim, Sq, Skv >= 1.  Returns 0 when the launch was queued,
// -1 otherwise.
int launch_attn_general(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv,
                        int D, bool causal, float scale, int dtype, const GeneralStrides& strides,
                        cudaStream_t stream);

// Bounds of the short-sequence kernels (one warp per (batch, head) slice): D
// in {16, 32, 64, 128}, Skv <= kSmallMaxKeys, and Sq <= 16 for fp16/bf16
// (warp-level tensor cores) or, for the SIMT kernel, Sq <= 32 rows at D <= 32,
// 16 at D = 64, 8 at D = 128 (and at D = 128 only Skv <= 16: with more keys
// its fp32 K and V do not fit in shared memory).
constexpr int kSmallMaxKeys = 64;

// True when launch_attn_small takes a problem of these sizes.
bool small_kernel_takes(int Sq, int Skv, int D, int dtype);

// Same contract as launch_attn_general for problems small_kernel_takes, and
// buffers whose bases and strides keep each row 16-byte aligned; returns -2
// (nothing launched) when they do not.
int launch_attn_small(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv, int D,
                      bool causal, float scale, int dtype, const GeneralStrides& strides, cudaStream_t stream);

// Grouped launches of the warp-level tensor-core short kernel (fp16/bf16,
// Sq <= 16): problems with the same dtype, head dim and 16-key group count
// (small_mma_group_key) run in one grid, up to kSmallGroupMax per grid, each
// slice computed exactly as a single launch computes it.
constexpr int kSmallGroupMax = 16;
struct SmallProblem {
  const void *q, *k, *v;
  void* out;
  int B, H, Sq, Skv;
  bool causal;
  float scale;
  GeneralStrides st;
};
// The group key of a problem: its 16-key group count (1, 2 or 4), or 0 when
// it does not take the warp-level tensor-core short kernel.
int small_mma_group_key(int Sq, int Skv, int D, int dtype);
// Launches the n problems (all of head dim D, dtype 0 or 1 and one group
// key) as few grids as kSmallGroupMax allows.  Problems whose rows are not
// 16-byte aligned are not launched; their indices go to *fallback.  Returns
// 0, or -1 if a grid could not be launched.
int launch_attn_small_grouped(const SmallProblem* p, int n, int D, int dtype, cudaStream_t stream,
                              std::vector<int>* fallback);

// Mid-length sequences on warp-level tensor cores (fp16/bf16, 16-byte aligned
// rows): every D = 16 / 32 problem, and D = 64 with Sq <= kMidMaxQueries and
// Skv <= kMidMaxKeys.
#ifndef RA_MID_MAX_QUERIES
#define RA_MID_MAX_QUERIES 64
#endif
constexpr int kMidMaxQueries = RA_MID_MAX_QUERIES;
constexpr int kMidMaxKeys = 256;
bool mid_kernel_takes(int Sq, int Skv, int D, int dtype);
int launch_attn_mid(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv, int D,
                    bool causal, float scale, int dtype, const GeneralStrides& strides, cudaStream_t stream);

}  // namespace ra
