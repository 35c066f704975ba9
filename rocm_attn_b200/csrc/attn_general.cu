// General attention forward for the shapes the tensor-core kernel does not
// take: fp32 inputs, head dims other than 64 and 128 (1..256), and fp16/bf16
// pointers that are not 16-byte aligned (TMA needs aligned bases).
//
// Covers the reference's remaining kernels on this path: the fp32 and
// D=16 fp16 routes of its launcher (src/attn_kernel_torch.cu:625-689, the
// simple kernel :36-97 and the WMMA D=16 kernel :356-621).  The math is the
// reference's: s = (q . k) * scale, masked when causal and key > query
// (top-left, src/attn_kernel_torch.cu:54,263), softmax in base 2 with a
// running fp32 max and sum (:269-298), O = P V / sum (:333-354), and a row
// with no unmasked key gives 0 (:335-336).
//
// Layout: q [B, H, Sq, D], k/v [B, H, Skv, D] with any (batch, head, row)
// strides and a contiguous head dim; o [B, H, Sq, D] contiguous.
// CTA: 64 query rows of one (batch, head) and 256 threads, four per row;
// thread t4 of a row owns the dims d = t4 + 4 i, so the four threads of a row
// read four consecutive shared-memory banks.  Keys are staged in blocks of 32
// (16 when D > 128) as fp32, zero beyond D; a row's four partial dot products
// are summed with two butterfly shuffles.  Every accumulation is fp32.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "attn_general.h"

namespace ra {

namespace {

constexpr int kRows = 64;    // query rows per CTA
constexpr int kThreads = 256;

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// kDMax: a multiple of 4 with D <= kDMax; each thread holds kDMax / 4 dims.
template <typename T, int kDMax, bool kCausal>
__global__ void __launch_bounds__(kThreads) attn_general_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                const T* __restrict__ v, T* __restrict__ o, int H,
                                                                int Sq, int Skv, int D, float scale_log2,
                                                                const GeneralStrides st) {
  constexpr int kPer = kDMax / 4;
  constexpr int kKeys = kDMax > 128 ? 16 : 32;  // keys per staged block (static shared memory <= 33 KB)
  constexpr int kStride = kDMax + 1;            // padded row of a staged key
  __shared__ float sK[kKeys * kStride];
  __shared__ float sV[kKeys * kStride];

  const int row_blocks = (Sq + kRows - 1) / kRows;
  const int bh = static_cast<int>(blockIdx.x / row_blocks);
  const int rb = static_cast<int>(blockIdx.x % row_blocks);
  const int row = rb * kRows + static_cast<int>(threadIdx.x) / 4;
  const int t4 = threadIdx.x & 3;
  const bool live = row < Sq;
  const long long b = bh / H, h = bh - b * H;
  const long long q_base = b * st.q[0] + h * st.q[1] + static_cast<long long>(live ? row : 0) * st.q[2];
  const long long k_base = b * st.k[0] + h * st.k[1], v_base = b * st.v[0] + h * st.v[1];
  const size_t o_base = (static_cast<size_t>(bh) * Sq + (live ? row : 0)) * D;

  float qr[kPer], acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = t4 + 4 * i;
    qr[i] = (live && d < D) ? to_f32(q[q_base + d]) * scale_log2 : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;

  // Keys this CTA needs: all of them, or up to its last query row when causal.
  const int last_row = min(Sq - 1, rb * kRows + kRows - 1);
  const int key_end = kCausal ? min(Skv, last_row + 1) : Skv;

  for (int k0 = 0; k0 < key_end; k0 += kKeys) {
    __syncthreads();  // the previous block's keys are no longer read
    for (int e = threadIdx.x; e < kKeys * kDMax; e += kThreads) {
      const int kk = e / kDMax, d = e - kk * kDMax;
      const int key = k0 + kk;
      const bool in = key < Skv && d < D;
      sK[kk * kStride + d] = in ? to_f32(k[k_base + key * st.k[2] + d]) : 0.f;
      sV[kk * kStride + d] = in ? to_f32(v[v_base + key * st.v[2] + d]) : 0.f;
    }
    __syncthreads();

    float s[kKeys];
#pragma unroll
    for (int kk = 0; kk < kKeys; ++kk) {
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < kPer; ++i) part = fmaf(qr[i], sK[kk * kStride + t4 + 4 * i], part);
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      const int key = k0 + kk;
      const bool masked = key >= Skv || (kCausal && key > row);
      s[kk] = masked ? -INFINITY : part;
    }
    float mb = m;
#pragma unroll
    for (int kk = 0; kk < kKeys; ++kk) mb = fmaxf(mb, s[kk]);
    if (mb == -INFINITY) continue;  // every key of the block is masked for this row
    const float alpha = exp2f(m - mb);  // m == -inf gives 0
    l *= alpha;
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] *= alpha;
    m = mb;
#pragma unroll
    for (int kk = 0; kk < kKeys; ++kk) {
      const float p = exp2f(s[kk] - m);
      l += p;
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc[i] = fmaf(p, sV[kk * kStride + t4 + 4 * i], acc[i]);
    }
  }

  if (live) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = t4 + 4 * i;
      if (d < D) o[o_base + d] = from_f32<T>(acc[i] * inv);
    }
  }
}

template <typename T, int kDMax>
int launch_typed(const void* q, const void* k, const void* v, void* out, int BH, int H, int Sq, int Skv, int D,
                 bool causal, float scale_log2, const GeneralStrides& st, cudaStream_t stream) {
  const long long blocks = static_cast<long long>((Sq + kRows - 1) / kRows) * BH;
  if (blocks > 0x7fffffffLL) return -1;
  const dim3 grid(static_cast<unsigned>(blocks));
  if (causal)
    attn_general_kernel<T, kDMax, true><<<grid, kThreads, 0, stream>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<T*>(out), H, Sq,
        Skv, D, scale_log2, st);
  else
    attn_general_kernel<T, kDMax, false><<<grid, kThreads, 0, stream>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<T*>(out), H, Sq,
        Skv, D, scale_log2, st);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <typename T>
int launch_dims(const void* q, const void* k, const void* v, void* out, int BH, int H, int Sq, int Skv, int D,
                bool causal, float scale_log2, const GeneralStrides& st, cudaStream_t stream) {
  if (D <= 16) return launch_typed<T, 16>(q, k, v, out, BH, H, Sq, Skv, D, causal, scale_log2, st, stream);
  if (D <= 32) return launch_typed<T, 32>(q, k, v, out, BH, H, Sq, Skv, D, causal, scale_log2, st, stream);
  if (D <= 64) return launch_typed<T, 64>(q, k, v, out, BH, H, Sq, Skv, D, causal, scale_log2, st, stream);
  if (D <= 128) return launch_typed<T, 128>(q, k, v, out, BH, H, Sq, Skv, D, causal, scale_log2, st, stream);
  return launch_typed<T, 256>(q, k, v, out, BH, H, Sq, Skv, D, causal, scale_log2, st, stream);
}

}  // namespace

int launch_attn_general(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv,
                        int D, bool causal, float scale, int dtype, const GeneralStrides& st, cudaStream_t stream) {
  const long long BH = static_cast<long long>(B) * H;
  if (B <= 0 || H <= 0 || BH > 0x7fffffffLL || Sq <= 0 || Skv <= 0 || D <= 0 || D > kGeneralMaxHeadDim) return -1;
  const int bh = static_cast<int>(BH);
  const float scale_log2 = scale * 1.4426950408889634f;
  switch (dtype) {
    case 0: return launch_dims<__half>(q, k, v, out, bh, H, Sq, Skv, D, causal, scale_log2, st, stream);
    case 1: return launch_dims<__nv_bfloat16>(q, k, v, out, bh, H, Sq, Skv, D, causal, scale_log2, st, stream);
    case 2: return launch_dims<float>(q, k, v, out, bh, H, Sq, Skv, D, causal, scale_log2, st, stream);
    default: return -1;
  }
}

}  // namespace ra
