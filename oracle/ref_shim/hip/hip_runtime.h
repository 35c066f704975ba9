/*
 * TEST INFRASTRUCTURE.  Host-only stand-in for <hip/hip_runtime.h>, just
 * enough for the reference's native known-answer test
 * (src/tests/attn_test.cpp of JoursBleu/rocm_attn) to compile with g++ on a
 * machine without ROCm: "device" memory is host memory and the launcher it
 * calls is ref_launch_shim.cpp, which runs this repository's C oracle.
 */
#pragma once
#include <cstdlib>
#include <cstring>

typedef void* hipStream_t;
typedef int hipError_t;
enum hipMemcpyKind { hipMemcpyHostToDevice = 1, hipMemcpyDeviceToHost = 2 };

template <class T>
static inline hipError_t hipMalloc(T** p, size_t n) {
  *p = static_cast<T*>(std::malloc(n));
  return *p ? 0 : 2;
}
static inline hipError_t hipMemcpy(void* dst, const void* src, size_t n, hipMemcpyKind) {
  std::memcpy(dst, src, n);
  return 0;
}
static inline hipError_t hipFree(void* p) {
  std::free(p);
  return 0;
}
static inline hipError_t hipDeviceSynchronize() { return 0; }
