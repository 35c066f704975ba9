// Host-side construction of TMA tensor maps for [batch, heads, seq, head_dim]
// 16-bit tensors.  The driver entry point is resolved through the runtime
// (cudaGetDriverEntryPoint), so the library does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace ra {

using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

// Returns nullptr when the driver does not provide the entry point.
inline EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// The TMA encoder is a driver call and needs a current context on the calling
// thread.  A host thread that has made no CUDA runtime call yet has none (the
// runtime binds the device's primary context lazily, on the first call that
// needs it), so this binds it there: only when no context is current, so a
// context the caller made current is never replaced.  Returns false if that
// fails.  Checked once per thread and device.
inline bool tensor_map_context_ready() {
  thread_local int ready_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (ready_dev == dev) return true;
  using GetCurrentFn = CUresult (*)(CUcontext*);
  static GetCurrentFn get_current = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<GetCurrentFn>(nullptr);
    return reinterpret_cast<GetCurrentFn>(p);
  }();
  CUcontext ctx = nullptr;
  if (!get_current || get_current(&ctx) != CUDA_SUCCESS) return false;
  if (ctx == nullptr && cudaSetDevice(dev) != cudaSuccess) return false;
  ready_dev = dev;
  return true;
}

// 4-D map over a [batch, heads, rows, inner] tensor of 16-bit elements whose
// innermost dimension is contiguous and whose other dimensions have the given
// element strides (any order in memory, e.g. the [B, L, H, D] layout viewed
// as [B, H, L, D]), loaded/stored in boxes of [1, 1, box_rows, box_inner]
// with 128-byte swizzle (box_inner * 2 must be 128).  TMA needs a 16-byte
// aligned base and strides that are positive multiples of 16 bytes below
// 2^40; returns -2 (nothing encoded) when they are not, so the caller can
// take another path, 0 on success, or a CUresult.
inline int make_tensor_map_4d(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t rows,
                              uint64_t heads, uint64_t batch, uint64_t row_stride, uint64_t head_stride,
                              uint64_t batch_stride, uint32_t box_inner, uint32_t box_rows) {
  const uint64_t sb[3] = {row_stride * 2, head_stride * 2, batch_stride * 2};
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return -2;
  for (uint64_t b : sb)
    if (b == 0 || (b & 15u) != 0 || b >= (uint64_t(1) << 40)) return -2;
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc || !tensor_map_context_ready()) return -1;
  cuuint64_t dims[4] = {inner, rows, heads, batch};
  cuuint64_t strides[3] = {sb[0], sb[1], sb[2]};
  cuuint32_t box[4] = {box_inner, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return static_cast<int>(r);
}

}  // namespace ra
