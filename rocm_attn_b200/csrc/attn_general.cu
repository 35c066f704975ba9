// The attention kernels for the calls the tcgen05 kernel does not take well
// (dispatch in attn_kernel.cu, launch_attn_forward_strided):
//   attn_small_mma_kernel  fp16/bf16, <= 16 queries, <= 64 keys: one warp per
//                          (batch, head) slice on warp-level tensor cores;
//   attn_mid_mma_kernel    fp16/bf16 at D = 16 / 32 and short D = 64: 64-row
//                          FlashAttention-2-style tiles on warp-level tensor
//                          cores, K/V streamed in 64-key chunks;
//   attn_small_kernel      <= 32 queries, <= 64 keys in any dtype: one warp per
//                          slice, SIMT fp32;
//   attn_general_kernel    everything else: fp32 inputs, head dims 1..256,
//                          buffers TMA cannot describe.
//
// Together they cover the reference's remaining kernels on this path: the
// fp32 and D=16 fp16 routes of its launcher (src/attn_kernel_torch.cu:625-689,
// the simple kernel :36-97 and the WMMA D=16 kernel :356-621).  The math is
// the reference's: s = (q . k) * scale, masked when causal and key > query
// (top-left, src/attn_kernel_torch.cu:54,263), softmax in base 2 with an fp32
// running max and sum (:269-298), O = P V / sum (:333-354), and a row with no
// unmasked key gives 0 (:335-336).  Every accumulation is fp32; the
// warp-level tensor-core kernels round P to the input type for P V, as the
// tcgen05 kernel does.
//
// Layout: q [B, H, Sq, D], k/v [B, H, Skv, D] with any (batch, head, row)
// strides and a contiguous head dim; o [B, H, Sq, D] contiguous.
//
// attn_general_kernel: 64 query rows of one (batch, head) per CTA and 256
// threads, four per row; thread t4 of a row owns the dims d = t4 + 4 i, so the
// four threads of a row read four consecutive shared-memory banks.  Keys are
// staged in blocks of 32 (16 when D > 128) as fp32, zero beyond D; a row's
// four partial dot products are summed with two butterfly shuffles.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "attn_general.h"

#include <atomic>
#include <mutex>
#include <vector>

namespace ra {

namespace {

constexpr int kRows = 64;    // query rows per CTA
constexpr int kThreads = 256;
constexpr int kMaxDevices = 64;

// Multiprocessor count of the current device, read once per device (0 when
// it cannot be read).
int current_sm_count() {
  static std::atomic<int> cached[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Raises the dynamic shared-memory limit of one kernel to `smem` bytes on the
// current device, once per device, and with `max_carveout` asks for the
// largest shared-memory share of the SM (so shared memory does not cap the
// CTAs per SM below what the registers allow); one static instance per
// kernel.
struct SmemOptIn {
  std::atomic<bool> done[kMaxDevices] = {};
  std::mutex mu;
  template <typename Kernel>
  bool ensure(Kernel kern, int smem, bool max_carveout = false) {
    if (smem <= 48 * 1024 && !max_carveout) return true;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    if (done[dev].load(std::memory_order_acquire)) return true;
    std::lock_guard<std::mutex> g(mu);
    if (!done[dev].load(std::memory_order_relaxed)) {
      if (smem > 48 * 1024 &&
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return false;
      if (max_carveout && cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                               static_cast<int>(cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
        return false;
      done[dev].store(true, std::memory_order_release);
    }
    return true;
  }
};

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

// ---------------------------------------------------------------------------
// Short sequences (Sq <= 32, Skv <= 64): one warp per (batch, head) slice,
// kSmallWarps warps per CTA walking the slices with a grid stride.  A warp
// converts its slice's K and V to fp32 in its own shared-memory region; lane l
// takes query row l / kLpr and the contiguous dims [kPer * (l % kLpr),
// kPer * (l % kLpr + 1)), kLpr = 32 / (rows rounded up to a power of two).
// With at most 64 keys a row keeps all its scores in registers: one max, one
// exponential per key and one pass over V, with no running rescale.
// This replaces a 128- or 256-row tensor-core unit per slice, which for the
// reference's 16-row inference shapes would be 88-94% padding.
// ---------------------------------------------------------------------------
constexpr int kSmallWarps = 4;

// 8 consecutive elements of a 16-byte aligned fp16/bf16/fp32 row as fp32.
__device__ __forceinline__ void load_f32x8(const void* src, int dtype, float* dst) {
  if (dtype == 2) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
    dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
    return;
  }
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if (dtype == 0) {
      __half2 h;
      memcpy(&h, &w[i], 4);
      f = __half22float2(h);
    } else {
      __nv_bfloat162 h;
      memcpy(&h, &w[i], 4);
      f = __bfloat1622float2(h);
    }
    dst[2 * i] = f.x;
    dst[2 * i + 1] = f.y;
  }
}

// Lanes per query row of the short-sequence kernel at head dim D (each lane
// holds 32 dims, 16 at D = 16): the warp covers 32 / lanes rows.
__host__ __device__ constexpr int small_lanes_per_row(int D) { return D <= 32 ? 1 : D / 32; }

// Largest dynamic shared memory a CTA may opt in to on sm_100 (227 KiB).
constexpr int kMaxDynamicSmem = 232448;

// Key capacity of the SIMT short-sequence kernel for Skv keys (16 or 64).
__host__ __device__ constexpr int small_simt_keys(int Skv) { return Skv <= 16 ? 16 : 64; }

// Dynamic shared memory of the SIMT short-sequence kernel: every warp holds
// its slice's K and V as fp32.  At D = 128 with 64 keys this is 256 KiB, above
// the limit, so those problems run the general kernel.
__host__ __device__ constexpr int small_simt_smem_bytes(int D, int keys) {
  return kSmallWarps * 2 * keys * D * static_cast<int>(sizeof(float));
}

// kD: the head dim (16, 32, 64 or 128); kKeys: the key capacity (16 or 64).
// dtype and causal are the same for the whole launch.
template <int kD, int kKeys>
__global__ void __launch_bounds__(kSmallWarps * 32) attn_small_kernel(const void* __restrict__ q,
                                                                      const void* __restrict__ k,
                                                                      const void* __restrict__ v,
                                                                      void* __restrict__ o, int dtype, bool causal,
                                                                      int BH, int H, int Sq, int Skv,
                                                                      float scale_log2, const GeneralStrides st) {
  constexpr int kLpr = small_lanes_per_row(kD);
  constexpr int kPer = kD / kLpr;
  static_assert(kPer % 8 == 0, "lane runs are whole chunks of 8 elements");
  extern __shared__ __align__(16) unsigned char small_smem[];
  const int esize = dtype == 2 ? 4 : 2;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  float* sK = reinterpret_cast<float*>(small_smem) + static_cast<size_t>(warp) * 2 * kKeys * kD;
  float* sV = sK + kKeys * kD;
  const int row = lane / kLpr, d0 = (lane % kLpr) * kPer;
  const bool live = row < Sq;
  const char* qb = static_cast<const char*>(q);
  const char* kb = static_cast<const char*>(k);
  const char* vb = static_cast<const char*>(v);

  for (int bh = blockIdx.x * kSmallWarps + warp; bh < BH; bh += gridDim.x * kSmallWarps) {
    const long long b = bh / H, h = bh - b * H;
    const long long k0 = b * st.k[0] + h * st.k[1], v0 = b * st.v[0] + h * st.v[1];
    __syncwarp();  // the previous slice's keys are no longer read
    for (int e = lane; e < Skv * (kD / 8); e += 32) {
      const int key = e / (kD / 8), c = (e - key * (kD / 8)) * 8;
      float a[8], w[8];
      load_f32x8(kb + (k0 + key * st.k[2] + c) * esize, dtype, a);
      load_f32x8(vb + (v0 + key * st.v[2] + c) * esize, dtype, w);
      float4* dk = reinterpret_cast<float4*>(sK + key * kD + c);
      float4* dv = reinterpret_cast<float4*>(sV + key * kD + c);
      dk[0] = make_float4(a[0], a[1], a[2], a[3]);
      dk[1] = make_float4(a[4], a[5], a[6], a[7]);
      dv[0] = make_float4(w[0], w[1], w[2], w[3]);
      dv[1] = make_float4(w[4], w[5], w[6], w[7]);
    }
    __syncwarp();

    float qr[kPer];
    {
      const long long q0 = b * st.q[0] + h * st.q[1] + static_cast<long long>(live ? row : 0) * st.q[2] + d0;
#pragma unroll
      for (int i = 0; i < kPer; i += 8) load_f32x8(qb + (q0 + i) * esize, dtype, qr + i);
#pragma unroll
      for (int i = 0; i < kPer; ++i) qr[i] *= scale_log2;
    }
    const int key_end = causal ? min(Skv, row + 1) : Skv;
    float s[kKeys];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      s[j] = -INFINITY;
      if (j < Skv) {  // uniform across the warp
        const float4* kr = reinterpret_cast<const float4*>(sK + j * kD + d0);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < kPer / 4; ++i) {
          const float4 x = kr[i];
          a0 = fmaf(qr[4 * i], x.x, a0);
          a1 = fmaf(qr[4 * i + 1], x.y, a1);
          a0 = fmaf(qr[4 * i + 2], x.z, a0);
          a1 = fmaf(qr[4 * i + 3], x.w, a1);
        }
        float dot = a0 + a1;
#pragma unroll
        for (int off = 1; off < kLpr; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        if (j < key_end) s[j] = dot;
        m = fmaxf(m, s[j]);
      }
    }
    float l = 0.f;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      s[j] = j < Skv ? exp2f(s[j] - m) : 0.f;  // a masked key gives 0
      l += s[j];
    }
    float acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kKeys; ++j)
      if (j < Skv) {
        const float4* vr = reinterpret_cast<const float4*>(sV + j * kD + d0);
#pragma unroll
        for (int i = 0; i < kPer / 4; ++i) {
          const float4 x = vr[i];
          acc[4 * i] = fmaf(s[j], x.x, acc[4 * i]);
          acc[4 * i + 1] = fmaf(s[j], x.y, acc[4 * i + 1]);
          acc[4 * i + 2] = fmaf(s[j], x.z, acc[4 * i + 2]);
          acc[4 * i + 3] = fmaf(s[j], x.w, acc[4 * i + 3]);
        }
      }
    if (live) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const size_t o0 = (static_cast<size_t>(bh) * Sq + row) * kD + d0;
      if (dtype == 2) {
        float4* orow = reinterpret_cast<float4*>(static_cast<float*>(o) + o0);
#pragma unroll
        for (int i = 0; i < kPer / 4; ++i)
          orow[i] = make_float4(acc[4 * i] * inv, acc[4 * i + 1] * inv, acc[4 * i + 2] * inv, acc[4 * i + 3] * inv);
      } else {
        uint4* orow = reinterpret_cast<uint4*>(static_cast<char*>(o) + o0 * 2);
#pragma unroll
        for (int i = 0; i < kPer / 8; ++i) {
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float lo = acc[8 * i + 2 * u] * inv, hi = acc[8 * i + 2 * u + 1] * inv;
            if (dtype == 0) {
              const __half2 hh = __floats2half2_rn(lo, hi);
              memcpy(&w[u], &hh, 4);
            } else {
              const __nv_bfloat162 hh = __floats2bfloat162_rn(lo, hi);
              memcpy(&w[u], &hh, 4);
            }
          }
          orow[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
}

template <int kD, int kKeys>
int launch_small_typed(const void* q, const void* k, const void* v, void* out, int dtype, bool causal, int BH, int H,
                       int Sq, int Skv, float scale_log2, const GeneralStrides& st, cudaStream_t stream) {
  constexpr int smem = small_simt_smem_bytes(kD, kKeys);
  static_assert(smem <= kMaxDynamicSmem, "SIMT short-sequence kernel above the shared-memory limit");
  auto kern = attn_small_kernel<kD, kKeys>;
  static SmemOptIn opt_in;
  const int sms = current_sm_count();
  if (sms == 0 || !opt_in.ensure(kern, smem)) return -1;
  const long long need = (static_cast<long long>(BH) + kSmallWarps - 1) / kSmallWarps;
  const unsigned grid = static_cast<unsigned>(need < 32LL * sms ? need : 32LL * sms);
  kern<<<grid, kSmallWarps * 32, smem, stream>>>(q, k, v, out, dtype, causal, BH, H, Sq, Skv, scale_log2, st);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <int kD>
int launch_small_keys(const void* q, const void* k, const void* v, void* out, int dtype, bool causal, int BH, int H,
                      int Sq, int Skv, float scale_log2, const GeneralStrides& st, cudaStream_t stream) {
  if (Skv <= 16)
    return launch_small_typed<kD, 16>(q, k, v, out, dtype, causal, BH, H, Sq, Skv, scale_log2, st, stream);
  if constexpr (small_simt_smem_bytes(kD, 64) <= kMaxDynamicSmem)
    return launch_small_typed<kD, 64>(q, k, v, out, dtype, causal, BH, H, Sq, Skv, scale_log2, st, stream);
  return -2;  // does not fit in shared memory: the caller runs the general kernel
}

// ---------------------------------------------------------------------------
// Short sequences on the warp-level tensor-core path (fp16/bf16, Sq <= 16,
// Skv <= 64, D in {16, 32, 64, 128}): one warp per (batch, head) slice does
// S = Q K^T and O = P V with mma.sync m16n8k16 (fp32 accumulate).  Q, K and V
// are staged in the warp's shared memory in rows padded by 16 bytes (so the
// eight row addresses of an ldmatrix hit distinct banks) and read as
// fragments with ldmatrix (V transposed).  The accumulator fragments of S are
// the A fragments of P V after packing to 16-bit pairs, so P never leaves
// registers.  Row max and sum reduce over the four lanes of a row quad.
// ---------------------------------------------------------------------------
constexpr int kMmaWarps = 4;

// CTAs per SM the short tensor-core kernel is compiled for.  The kernel is
// bound by HBM latency, so more slices in flight per SM help: six CTAs (an
// 80-register cap) where that compiles without spills (D = 64 with up to 16
// keys, D <= 32 with up to 32; measured 5-7 % faster on the largest UnifoLM
// 16-row shapes), otherwise no bound.
template <int kD, int kNK>
constexpr int small_mma_min_blocks() {
  return ((kD == 64 && kNK == 1) || (kD <= 32 && kNK <= 2)) ? 6 : 1;
}

// 16-byte global -> shared copy that does not block the thread; with
// valid = false nothing is read and the 16 bytes are zero-filled.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
template <bool kBf16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kBf16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
template <bool kBf16>
__device__ __forceinline__ uint32_t pack16x2(float lo, float hi) {
  uint32_t w;
  if constexpr (kBf16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    memcpy(&w, &h, 4);
  } else {
    const __half2 h = __floats2half2_rn(lo, hi);
    memcpy(&w, &h, 4);
  }
  return w;
}

// One (batch, head) slice on one warp: qp, kp, vp point at its first row
// (row strides q_row, k_row, v_row elements), ob at its contiguous output;
// sQ, sK, sV are the warp's staging buffers.  kNK: 16-key groups (Skv <= 16 kNK).
template <bool kBf16, int kD, int kNK>
__device__ __forceinline__ void small_mma_slice(const uint16_t* __restrict__ qp, const uint16_t* __restrict__ kp,
                                                const uint16_t* __restrict__ vp, uint16_t* __restrict__ ob,
                                                bool causal, int Sq, int Skv, float scale_log2, long long q_row,
                                                long long k_row, long long v_row, uint16_t* sQ, uint16_t* sK,
                                                uint16_t* sV, int lane) {
  constexpr int kRow = kD + 8;        // padded row of a staged matrix, in 16-bit elements
  constexpr int kKeys = 16 * kNK;
  constexpr int kChunks = kD / 8;     // 16-byte chunks per row
  const int g = lane >> 2, t4 = lane & 3;  // row within an 8-row group, lane within the row quad
  const int mi = lane >> 3, ri = lane & 7; // ldmatrix: matrix and row this lane addresses
  __syncwarp();  // the previous slice's staging is no longer read
  // Stage Q (16 rows) and K, V (kKeys rows) with 16-byte asynchronous
  // copies, all in flight at once, zero-filled past Sq / Skv.
#pragma unroll
  for (int e = lane; e < (16 + 2 * kKeys) * kChunks; e += 32) {
    const int r = e / kChunks, c = (e - r * kChunks) * 8;
    const uint16_t* src;
    uint16_t* dst;
    bool in;
    if (r < 16) {
      in = r < Sq;
      src = qp + (in ? r : 0) * q_row + c;
      dst = sQ + r * kRow + c;
    } else if (r < 16 + kKeys) {
      const int key = r - 16;
      in = key < Skv;
      src = kp + (in ? key : 0) * k_row + c;
      dst = sK + key * kRow + c;
    } else {
      const int key = r - 16 - kKeys;
      in = key < Skv;
      src = vp + (in ? key : 0) * v_row + c;
      dst = sV + key * kRow + c;
    }
    cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dst)), src, in);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncwarp();

  // S = Q K^T: 2 * kNK n8 tiles of keys, kD / 16 k-steps over the head dim.
  float sf[2 * kNK][4];
#pragma unroll
  for (int n = 0; n < 2 * kNK; ++n) sf[n][0] = sf[n][1] = sf[n][2] = sf[n][3] = 0.f;
  const uint32_t q_base = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
  const uint32_t k_base = static_cast<uint32_t>(__cvta_generic_to_shared(sK));
  const uint32_t v_base = static_cast<uint32_t>(__cvta_generic_to_shared(sV));
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks) {
    uint32_t a[4];
    ldsm_x4(q_base + 2 * (((mi & 1) * 8 + ri) * kRow + ks * 16 + (mi >> 1) * 8), a);
#pragma unroll
    for (int nk = 0; nk < kNK; ++nk) {
      uint32_t bk[4];
      ldsm_x4(k_base + 2 * ((nk * 16 + (mi >> 1) * 8 + ri) * kRow + ks * 16 + (mi & 1) * 8), bk);
      mma16816<kBf16>(sf[2 * nk], a, bk[0], bk[1]);
      mma16816<kBf16>(sf[2 * nk + 1], a, bk[2], bk[3]);
    }
  }

  // Softmax over each row (rows g and g + 8 of this lane; its keys are
  // 8 n + 2 t4 and + 1 of every tile n).
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int n = 0; n < 2 * kNK; ++n) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = 8 * n + 2 * t4 + (e & 1);
      const int row = g + (e >> 1) * 8;
      const bool masked = key >= Skv || (causal && key > row);
      sf[n][e] = masked ? -INFINITY : sf[n][e] * scale_log2;
    }
    m0 = fmaxf(m0, fmaxf(sf[n][0], sf[n][1]));
    m1 = fmaxf(m1, fmaxf(sf[n][2], sf[n][3]));
  }
  m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
  m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int n = 0; n < 2 * kNK; ++n) {
    sf[n][0] = exp2f(sf[n][0] - m0);
    sf[n][1] = exp2f(sf[n][1] - m0);
    sf[n][2] = exp2f(sf[n][2] - m1);
    sf[n][3] = exp2f(sf[n][3] - m1);
    l0 += sf[n][0] + sf[n][1];
    l1 += sf[n][2] + sf[n][3];
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // O = P V: P's accumulator fragments are A fragments after packing.
  float of[kD / 8][4];
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) of[n][0] = of[n][1] = of[n][2] = of[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < kNK; ++kk) {
    const uint32_t a[4] = {pack16x2<kBf16>(sf[2 * kk][0], sf[2 * kk][1]),
                           pack16x2<kBf16>(sf[2 * kk][2], sf[2 * kk][3]),
                           pack16x2<kBf16>(sf[2 * kk + 1][0], sf[2 * kk + 1][1]),
                           pack16x2<kBf16>(sf[2 * kk + 1][2], sf[2 * kk + 1][3])};
#pragma unroll
    for (int dt = 0; dt < kD / 8; dt += 2) {
      uint32_t bv[4];
      ldsm_x4_trans(v_base + 2 * ((kk * 16 + (mi & 1) * 8 + ri) * kRow + (dt + (mi >> 1)) * 8), bv);
      mma16816<kBf16>(of[dt], a, bv[0], bv[1]);
      mma16816<kBf16>(of[dt + 1], a, bv[2], bv[3]);
    }
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) {
    const int col = 8 * n + 2 * t4;
    if (g < Sq) *reinterpret_cast<uint32_t*>(ob + g * kD + col) = pack16x2<kBf16>(of[n][0] * inv0, of[n][1] * inv0);
    if (g + 8 < Sq)
      *reinterpret_cast<uint32_t*>(ob + (g + 8) * kD + col) = pack16x2<kBf16>(of[n][2] * inv1, of[n][3] * inv1);
  }
}

// The warp's staging buffers in dynamic shared memory.
template <int kD, int kNK>
__device__ __forceinline__ uint16_t* small_mma_staging(unsigned char* smem, int warp) {
  return reinterpret_cast<uint16_t*>(smem) + static_cast<size_t>(warp) * (16 + 2 * 16 * kNK) * (kD + 8);
}

template <bool kBf16, int kD, int kNK>
__global__ void __launch_bounds__(kMmaWarps * 32, small_mma_min_blocks<kD, kNK>()) attn_small_mma_kernel(const uint16_t* __restrict__ q,
                                                                        const uint16_t* __restrict__ k,
                                                                        const uint16_t* __restrict__ v,
                                                                        uint16_t* __restrict__ o, bool causal,
                                                                        int BH, int H, int Sq, int Skv,
                                                                        float scale_log2, const GeneralStrides st) {
  extern __shared__ __align__(16) unsigned char mma_smem[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  uint16_t* sQ = small_mma_staging<kD, kNK>(mma_smem, warp);
  uint16_t* sK = sQ + 16 * (kD + 8);
  uint16_t* sV = sK + 16 * kNK * (kD + 8);
  for (int bh = blockIdx.x * kMmaWarps + warp; bh < BH; bh += gridDim.x * kMmaWarps) {
    const long long b = bh / H, h = bh - b * H;
    small_mma_slice<kBf16, kD, kNK>(q + b * st.q[0] + h * st.q[1], k + b * st.k[0] + h * st.k[1],
                                    v + b * st.v[0] + h * st.v[1], o + static_cast<size_t>(bh) * Sq * kD, causal,
                                    Sq, Skv, scale_log2, st.q[2], st.k[2], st.v[2], sQ, sK, sV, lane);
  }
}

// Several problems of one dtype, head dim and key-group count in one grid:
// slot i holds problem i and the running total of slices up to and
// including it; warps walk the global slice index and find its problem.
struct SmallSlot {
  const uint16_t *q, *k, *v;
  uint16_t* o;
  GeneralStrides st;
  long long slice_end;
  int H, Sq, Skv, causal;
  float scale_log2;
};
struct SmallGroupArgs {
  SmallSlot p[kSmallGroupMax];
  int n;
};

template <bool kBf16, int kD, int kNK>
__global__ void __launch_bounds__(kMmaWarps * 32, small_mma_min_blocks<kD, kNK>()) attn_small_mma_group_kernel(const __grid_constant__ SmallGroupArgs a) {
  extern __shared__ __align__(16) unsigned char mma_smem[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  uint16_t* sQ = small_mma_staging<kD, kNK>(mma_smem, warp);
  uint16_t* sK = sQ + 16 * (kD + 8);
  uint16_t* sV = sK + 16 * kNK * (kD + 8);
  const long long total = a.p[a.n - 1].slice_end;
  int pi = 0;  // a warp's slices only increase, so its problem index only moves forward
  for (long long s = static_cast<long long>(blockIdx.x) * kMmaWarps + warp; s < total;
       s += static_cast<long long>(gridDim.x) * kMmaWarps) {
    while (s >= a.p[pi].slice_end) ++pi;
    const SmallSlot& P = a.p[pi];
    const long long bh = s - (pi > 0 ? a.p[pi - 1].slice_end : 0);
    const long long b = bh / P.H, h = bh - b * P.H;
    small_mma_slice<kBf16, kD, kNK>(P.q + b * P.st.q[0] + h * P.st.q[1], P.k + b * P.st.k[0] + h * P.st.k[1],
                                    P.v + b * P.st.v[0] + h * P.st.v[1], P.o + bh * P.Sq * kD, P.causal != 0, P.Sq,
                                    P.Skv, P.scale_log2, P.st.q[2], P.st.k[2], P.st.v[2], sQ, sK, sV, lane);
  }
}

template <bool kBf16, int kD, int kNK>
int launch_small_mma_typed(const void* q, const void* k, const void* v, void* out, bool causal, int BH, int H, int Sq,
                           int Skv, float scale_log2, const GeneralStrides& st, cudaStream_t stream) {
  constexpr int smem = kMmaWarps * (16 + 2 * 16 * kNK) * (kD + 8) * 2;
  static_assert(smem <= kMaxDynamicSmem, "short-sequence tensor-core kernel above the shared-memory limit");
  auto kern = attn_small_mma_kernel<kBf16, kD, kNK>;
  static SmemOptIn opt_in;
  const int sms = current_sm_count();
  if (sms == 0 || !opt_in.ensure(kern, smem, true)) return -1;
  const long long need = (static_cast<long long>(BH) + kMmaWarps - 1) / kMmaWarps;
  const unsigned grid = static_cast<unsigned>(need < 32LL * sms ? need : 32LL * sms);
  kern<<<grid, kMmaWarps * 32, smem, stream>>>(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
                                               static_cast<const uint16_t*>(v), static_cast<uint16_t*>(out), causal,
                                               BH, H, Sq, Skv, scale_log2, st);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <bool kBf16, int kD, int kNK>
int launch_small_mma_group_typed(const SmallGroupArgs& a, cudaStream_t stream) {
  constexpr int smem = kMmaWarps * (16 + 2 * 16 * kNK) * (kD + 8) * 2;
  auto kern = attn_small_mma_group_kernel<kBf16, kD, kNK>;
  static SmemOptIn opt_in;
  const int sms = current_sm_count();
  if (sms == 0 || !opt_in.ensure(kern, smem, true)) return -1;
  const long long need = (a.p[a.n - 1].slice_end + kMmaWarps - 1) / kMmaWarps;
  const unsigned grid = static_cast<unsigned>(need < 32LL * sms ? need : 32LL * sms);
  kern<<<grid, kMmaWarps * 32, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <bool kBf16, int kD>
int launch_small_mma_group_d(const SmallGroupArgs& a, int nk, cudaStream_t stream) {
  switch (nk) {
    case 1: return launch_small_mma_group_typed<kBf16, kD, 1>(a, stream);
    case 2: return launch_small_mma_group_typed<kBf16, kD, 2>(a, stream);
    default: return launch_small_mma_group_typed<kBf16, kD, 4>(a, stream);
  }
}

template <bool kBf16>
int launch_small_mma_group(const SmallGroupArgs& a, int D, int nk, cudaStream_t stream) {
  switch (D) {
    case 16: return launch_small_mma_group_d<kBf16, 16>(a, nk, stream);
    case 32: return launch_small_mma_group_d<kBf16, 32>(a, nk, stream);
    case 64: return launch_small_mma_group_d<kBf16, 64>(a, nk, stream);
    default: return launch_small_mma_group_d<kBf16, 128>(a, nk, stream);
  }
}

template <bool kBf16, int kD>
int launch_small_mma_keys(const void* q, const void* k, const void* v, void* out, bool causal, int BH, int H, int Sq,
                          int Skv, float sl, const GeneralStrides& st, cudaStream_t stream) {
  if (Skv <= 16) return launch_small_mma_typed<kBf16, kD, 1>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
  if (Skv <= 32) return launch_small_mma_typed<kBf16, kD, 2>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
  return launch_small_mma_typed<kBf16, kD, 4>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
}

template <bool kBf16>
int launch_small_mma(const void* q, const void* k, const void* v, void* out, bool causal, int BH, int H, int Sq,
                     int Skv, int D, float sl, const GeneralStrides& st, cudaStream_t stream) {
  switch (D) {
    case 16: return launch_small_mma_keys<kBf16, 16>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
    case 32: return launch_small_mma_keys<kBf16, 32>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
    case 64: return launch_small_mma_keys<kBf16, 64>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
    default: return launch_small_mma_keys<kBf16, 128>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
  }
}

// ---------------------------------------------------------------------------
// Mid-length sequences on warp-level tensor cores (fp16/bf16, D in {16, 32,
// 64, 128}, any Skv; the dispatcher uses it for D = 16 / 32 and for short
// D = 64 problems): FlashAttention-2-style.  A CTA of 4 warps takes 64
// query rows of one (batch, head) slice, one m16 tile per warp; K and V stream
// through shared memory in 64-key chunks, double-buffered with cp.async
// (16-byte copies, zero-filled past Skv), rows padded by 16 bytes for
// conflict-free ldmatrix.  Per chunk each warp computes S = Q K^T with
// mma.sync m16n8k16 (fp32 accumulate), moves its running row max, rescales O
// and the row sums, and adds P V with P taken straight from the S fragments.
// ---------------------------------------------------------------------------
constexpr int kMidWarps = 4;  // 64 query rows per CTA


template <bool kBf16, int kD>
__global__ void __launch_bounds__(kMidWarps * 32) attn_mid_mma_kernel(const uint16_t* __restrict__ q,
                                                                      const uint16_t* __restrict__ k,
                                                                      const uint16_t* __restrict__ v,
                                                                      uint16_t* __restrict__ o, bool causal, int H,
                                                                      int Sq, int Skv, float scale_log2,
                                                                      const GeneralStrides st) {
  constexpr int kRow = kD + 8;
  constexpr int kChunks = kD / 8;
  constexpr int kThreads = kMidWarps * 32;
  extern __shared__ __align__(16) unsigned char mid_smem[];
  uint16_t* sQ = reinterpret_cast<uint16_t*>(mid_smem);  // [64][kRow]
  uint16_t* sKV = sQ + 64 * kRow;                         // [2 buffers][K, V][64][kRow]
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3, mi = lane >> 3, ri = lane & 7;
  const int mblocks = (Sq + 63) / 64;
  const int bh = static_cast<int>(blockIdx.x) / mblocks;
  const int row0 = (static_cast<int>(blockIdx.x) - bh * mblocks) * 64;
  const long long b = bh / H, h = bh - b * H;
  const uint16_t* qp = q + b * st.q[0] + h * st.q[1];
  const uint16_t* kp = k + b * st.k[0] + h * st.k[1];
  const uint16_t* vp = v + b * st.v[0] + h * st.v[1];
  const int key_end = causal ? min(Skv, min(Sq, row0 + 64)) : Skv;  // keys this CTA's rows can see
  const int nchunks = (key_end + 63) / 64;

  auto load_chunk = [&](int c, int buf) {
    uint16_t* dK = sKV + buf * 2 * 64 * kRow;
    uint16_t* dV = dK + 64 * kRow;
    for (int e = threadIdx.x; e < 64 * kChunks; e += kThreads) {
      const int r = e / kChunks, col = (e - r * kChunks) * 8;
      const int key = c * 64 + r;
      const bool in = key < Skv;
      const long long kr = in ? key : 0;
      cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dK + r * kRow + col)), kp + kr * st.k[2] + col, in);
      cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dV + r * kRow + col)), vp + kr * st.v[2] + col, in);
    }
  };
  for (int e = threadIdx.x; e < 64 * kChunks; e += kThreads) {
    const int r = e / kChunks, col = (e - r * kChunks) * 8;
    const bool in = row0 + r < Sq;
    const long long qr = in ? row0 + r : 0;
    cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(sQ + r * kRow + col)), qp + qr * st.q[2] + col, in);
  }
  load_chunk(0, 0);
  cp_async_commit();

  const int rowA = row0 + warp * 16 + g, rowB = rowA + 8;  // this lane's two query rows
  uint32_t qa[kD / 16][4];
  float of[kD / 8][4];
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) of[n][0] = of[n][1] = of[n][2] = of[n][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const uint32_t q_base = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));

  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_chunk(c + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // chunk c (and Q) visible to every warp
    if (c == 0) {
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks)
        ldsm_x4(q_base + 2 * ((warp * 16 + (mi & 1) * 8 + ri) * kRow + ks * 16 + (mi >> 1) * 8), qa[ks]);
    }
    const uint32_t k_base = static_cast<uint32_t>(__cvta_generic_to_shared(sKV + buf * 2 * 64 * kRow));
    const uint32_t v_base = k_base + 2 * 64 * kRow;

    float sf[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sf[n][0] = sf[n][1] = sf[n][2] = sf[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks) {
#pragma unroll
      for (int nk = 0; nk < 4; ++nk) {
        uint32_t bk[4];
        ldsm_x4(k_base + 2 * ((nk * 16 + (mi >> 1) * 8 + ri) * kRow + ks * 16 + (mi & 1) * 8), bk);
        mma16816<kBf16>(sf[2 * nk], qa[ks], bk[0], bk[1]);
        mma16816<kBf16>(sf[2 * nk + 1], qa[ks], bk[2], bk[3]);
      }
    }
    float cA = -INFINITY, cB = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = c * 64 + 8 * n + 2 * t4 + (e & 1);
        const int row = e < 2 ? rowA : rowB;
        const bool masked = key >= Skv || (causal && key > row);
        sf[n][e] = masked ? -INFINITY : sf[n][e] * scale_log2;
      }
      cA = fmaxf(cA, fmaxf(sf[n][0], sf[n][1]));
      cB = fmaxf(cB, fmaxf(sf[n][2], sf[n][3]));
    }
    cA = fmaxf(cA, __shfl_xor_sync(0xffffffffu, cA, 1));
    cA = fmaxf(cA, __shfl_xor_sync(0xffffffffu, cA, 2));
    cB = fmaxf(cB, __shfl_xor_sync(0xffffffffu, cB, 1));
    cB = fmaxf(cB, __shfl_xor_sync(0xffffffffu, cB, 2));
    const float nA = fmaxf(mA, cA), nB = fmaxf(mB, cB);
    // A row with every key so far masked keeps m = -inf; its P is 0.
    const float rA = nA == -INFINITY ? 0.f : nA, rB = nB == -INFINITY ? 0.f : nB;
    const float aA = exp2f(mA - rA), aB = exp2f(mB - rB);  // m = -inf gives 0
    mA = nA;
    mB = nB;
    lA *= aA;
    lB *= aB;
#pragma unroll
    for (int n = 0; n < kD / 8; ++n) {
      of[n][0] *= aA;
      of[n][1] *= aA;
      of[n][2] *= aB;
      of[n][3] *= aB;
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      sf[n][0] = exp2f(sf[n][0] - rA);
      sf[n][1] = exp2f(sf[n][1] - rA);
      sf[n][2] = exp2f(sf[n][2] - rB);
      sf[n][3] = exp2f(sf[n][3] - rB);
      lA += sf[n][0] + sf[n][1];
      lB += sf[n][2] + sf[n][3];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pack16x2<kBf16>(sf[2 * kk][0], sf[2 * kk][1]),
                             pack16x2<kBf16>(sf[2 * kk][2], sf[2 * kk][3]),
                             pack16x2<kBf16>(sf[2 * kk + 1][0], sf[2 * kk + 1][1]),
                             pack16x2<kBf16>(sf[2 * kk + 1][2], sf[2 * kk + 1][3])};
#pragma unroll
      for (int dt = 0; dt < kD / 8; dt += 2) {
        uint32_t bv[4];
        ldsm_x4_trans(v_base + 2 * ((kk * 16 + (mi & 1) * 8 + ri) * kRow + (dt + (mi >> 1)) * 8), bv);
        mma16816<kBf16>(of[dt], a, bv[0], bv[1]);
        mma16816<kBf16>(of[dt + 1], a, bv[2], bv[3]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before chunk c + 2 overwrites it
  }

  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
  uint16_t* ob = o + static_cast<size_t>(bh) * Sq * kD;
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) {
    const int col = 8 * n + 2 * t4;
    if (rowA < Sq) *reinterpret_cast<uint32_t*>(ob + static_cast<size_t>(rowA) * kD + col) = pack16x2<kBf16>(of[n][0] * iA, of[n][1] * iA);
    if (rowB < Sq) *reinterpret_cast<uint32_t*>(ob + static_cast<size_t>(rowB) * kD + col) = pack16x2<kBf16>(of[n][2] * iB, of[n][3] * iB);
  }
}

template <bool kBf16, int kD>
int launch_mid_typed(const void* q, const void* k, const void* v, void* out, bool causal, int BH, int H, int Sq,
                     int Skv, float scale_log2, const GeneralStrides& st, cudaStream_t stream) {
  constexpr int smem = 5 * 64 * (kD + 8) * 2;  // Q + two buffers of K and V
  static_assert(smem <= kMaxDynamicSmem, "mid-length kernel above the shared-memory limit");
  auto kern = attn_mid_mma_kernel<kBf16, kD>;
  static SmemOptIn opt_in;
  if (!opt_in.ensure(kern, smem)) return -1;
  const long long grid = static_cast<long long>(BH) * ((Sq + 63) / 64);
  if (grid > 0x7fffffffLL) return -1;
  kern<<<static_cast<unsigned>(grid), kMidWarps * 32, smem, stream>>>(
      static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v),
      static_cast<uint16_t*>(out), causal, H, Sq, Skv, scale_log2, st);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <bool kBf16>
int launch_mid(const void* q, const void* k, const void* v, void* out, bool causal, int BH, int H, int Sq, int Skv,
               int D, float sl, const GeneralStrides& st, cudaStream_t stream) {
  switch (D) {
    case 16: return launch_mid_typed<kBf16, 16>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
    case 32: return launch_mid_typed<kBf16, 32>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
    case 64: return launch_mid_typed<kBf16, 64>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
    default: return launch_mid_typed<kBf16, 128>(q, k, v, out, causal, BH, H, Sq, Skv, sl, st, stream);
  }
}

}  // namespace

bool mid_kernel_takes(int Sq, int Skv, int D, int dtype) {
  if (dtype == 2 || Sq < 1 || Skv < 1) return false;
  // D = 16 / 32 have no tcgen05 path: this kernel at every length.  D = 64:
  // where the 128-row tcgen05 tiles are mostly padding (measured: 20-40 %
  // faster for 40-64 query rows with up to 93 keys, even at 256 keys; slower
  // from 128 query rows or 351 keys on).  D = 128: the tcgen05 kernel.
  if (D == 16 || D == 32) return true;
  if (D == 64) return Sq <= kMidMaxQueries && Skv <= kMidMaxKeys;
  return false;
}

int launch_attn_mid(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv, int D,
                    bool causal, float scale, int dtype, const GeneralStrides& st, cudaStream_t stream) {
  const long long BH = static_cast<long long>(B) * H;
  if (B <= 0 || H <= 0 || BH > 0x7fffffffLL || !mid_kernel_takes(Sq, Skv, D, dtype)) return -1;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  for (const long long* s3 : {st.q, st.k, st.v})
    for (int i = 0; i < 3; ++i)
      if ((s3[i] * 2) % 16 != 0) return -2;
  if (!a16(q) || !a16(k) || !a16(v) || !a16(out)) return -2;
  const float sl = scale * 1.4426950408889634f;
  return dtype == 1 ? launch_mid<true>(q, k, v, out, causal, static_cast<int>(BH), H, Sq, Skv, D, sl, st, stream)
                    : launch_mid<false>(q, k, v, out, causal, static_cast<int>(BH), H, Sq, Skv, D, sl, st, stream);
}

bool small_kernel_takes(int Sq, int Skv, int D, int dtype) {
  if (D != 16 && D != 32 && D != 64 && D != 128) return false;
  if (Sq < 1 || Skv < 1 || Skv > kSmallMaxKeys) return false;
  if (dtype != 2 && Sq <= 16) return true;  // warp-level tensor-core kernel: one m16 tile
  // SIMT kernel: one lane group per row, and the slice's K and V as fp32 in
  // shared memory.
  return Sq <= 32 / small_lanes_per_row(D) && small_simt_smem_bytes(D, small_simt_keys(Skv)) <= kMaxDynamicSmem;
}

int launch_attn_small(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv, int D,
                      bool causal, float scale, int dtype, const GeneralStrides& st, cudaStream_t stream) {
  const long long BH = static_cast<long long>(B) * H;
  if (B <= 0 || H <= 0 || BH > 0x7fffffffLL || dtype < 0 || dtype > 2 || !small_kernel_takes(Sq, Skv, D, dtype))
    return -1;
  // 16-byte chunks: the bases and the row/head/batch strides must keep every
  // row 16-byte aligned.
  const long long esize = dtype == 2 ? 4 : 2;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  for (const long long* s3 : {st.q, st.k, st.v})
    for (int i = 0; i < 3; ++i)
      if ((s3[i] * esize) % 16 != 0) return -2;
  if (!a16(q) || !a16(k) || !a16(v) || !a16(out)) return -2;
  const int bh = static_cast<int>(BH);
  const float sl = scale * 1.4426950408889634f;
  // fp16/bf16 slices of up to 16 rows: warp-level tensor cores.
  if (dtype != 2 && Sq <= 16) {
    return dtype == 1 ? launch_small_mma<true>(q, k, v, out, causal, bh, H, Sq, Skv, D, sl, st, stream)
                      : launch_small_mma<false>(q, k, v, out, causal, bh, H, Sq, Skv, D, sl, st, stream);
  }
  switch (D) {
    case 16: return launch_small_keys<16>(q, k, v, out, dtype, causal, bh, H, Sq, Skv, sl, st, stream);
    case 32: return launch_small_keys<32>(q, k, v, out, dtype, causal, bh, H, Sq, Skv, sl, st, stream);
    case 64: return launch_small_keys<64>(q, k, v, out, dtype, causal, bh, H, Sq, Skv, sl, st, stream);
    default: return launch_small_keys<128>(q, k, v, out, dtype, causal, bh, H, Sq, Skv, sl, st, stream);
  }
}

int small_mma_group_key(int Sq, int Skv, int D, int dtype) {
  if (dtype == 2 || Sq > 16 || !small_kernel_takes(Sq, Skv, D, dtype)) return 0;
  return Skv <= 16 ? 1 : Skv <= 32 ? 2 : 4;
}

int launch_attn_small_grouped(const SmallProblem* p, int n, int D, int dtype, cudaStream_t stream,
                              std::vector<int>* fallback) {
  if (n <= 0) return 0;
  const int nk = small_mma_group_key(p[0].Sq, p[0].Skv, D, dtype);
  if (nk == 0) return -1;
  SmallGroupArgs a{};
  auto flush = [&]() -> int {
    if (a.n == 0) return 0;
    const int r = dtype == 1 ? launch_small_mma_group<true>(a, D, nk, stream)
                             : launch_small_mma_group<false>(a, D, nk, stream);
    a.n = 0;
    return r;
  };
  auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  long long slices = 0;
  for (int i = 0; i < n; ++i) {
    const SmallProblem& q = p[i];
    const long long BH = static_cast<long long>(q.B) * q.H;
    bool rows16 = a16(q.q) && a16(q.k) && a16(q.v) && a16(q.out);
    for (const long long* s3 : {q.st.q, q.st.k, q.st.v})
      for (int j = 0; j < 3; ++j) rows16 = rows16 && (s3[j] * 2) % 16 == 0;
    if (small_mma_group_key(q.Sq, q.Skv, D, dtype) != nk || BH <= 0 || BH > 0x7fffffffLL || !rows16) {
      fallback->push_back(i);  // the caller runs it alone
      continue;
    }
    if (a.n == kSmallGroupMax) {
      if (flush() != 0) return -1;
      slices = 0;
    }
    slices += BH;
    a.p[a.n] = SmallSlot{static_cast<const uint16_t*>(q.q), static_cast<const uint16_t*>(q.k),
                         static_cast<const uint16_t*>(q.v), static_cast<uint16_t*>(q.out), q.st, slices, q.H, q.Sq,
                         q.Skv, q.causal ? 1 : 0, q.scale * 1.4426950408889634f};
    ++a.n;
  }
  return flush();
}

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
