/*
 * C-ABI launch interface of the sm_100a attention-forward library
 * (librocm_attn.so).  Plain pointers and sizes only; no framework types.
 *
 * Replaces the reference's `launch_attn_forward` declared at
 * src/attn_kernel.h:18-20 of JoursBleu/rocm_attn (enum AttnDType at
 * src/attn_kernel.h:12-16), whose definitions live at
 * src/attn_kernel_torch.cu:625-689 and src/attn_kernel.hip.cpp:304-367.
 *
 * Differences from the reference signature, all deliberate:
 *   - returns an int status (the reference returns void and checks nothing);
 *   - takes an explicit softmax scale (the reference hard-wires rsqrt(D),
 *     src/attn_kernel_torch.cu:111); a value <= 0 or non-finite selects the
 *     reference default 1/sqrt(D);
 *   - the stream is a cudaStream_t (the reference takes a hipStream_t).
 * The argument order otherwise matches the reference.
 */
#ifndef ROCM_ATTN_B200_ATTN_KERNEL_H_
#define ROCM_ATTN_B200_ATTN_KERNEL_H_

#include <cuda_runtime.h>
#include <stdbool.h>

#if defined(__GNUC__)
#define ATTN_API __attribute__((visibility("default")))
#else
#define ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of q/k/v/out.  Values match the reference enum
 * (src/attn_kernel.h:12-16) so the ABI stays compatible. */
typedef enum AttnDType {
  ATTN_F16 = 0,
  ATTN_BF16 = 1,
  ATTN_F32 = 2,
} AttnDType;

/* Status codes returned by the entry points below. */
enum AttnStatus {
  ATTN_OK = 0,
  ATTN_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, overflow   */
  ATTN_ERR_UNSUPPORTED = 2,      /* unknown dtype or head_dim > 256         */
  ATTN_ERR_MISALIGNED = 3,       /* pointer not aligned to its element size */
  ATTN_ERR_TENSOR_MAP = 4,       /* TMA descriptor could not be encoded     */
  ATTN_ERR_LAUNCH = 5,           /* CUDA runtime error at launch            */
  ATTN_ERR_DEVICE = 6,           /* current device is not an sm_100 GPU     */
  ATTN_ERR_WATCHDOG = 7          /* a kernel wait timed out (see below)     */
};

/*
 * Scaled dot-product attention forward, O = softmax(scale * Q K^T [+ mask]) V.
 *   q   [B, H, Sq,  D]  contiguous, row-major
 *   k,v [B, H, Skv, D]  contiguous, row-major
 *   out [B, H, Sq,  D]  contiguous, row-major, fully overwritten
 * causal: key j is masked for query i when j > i (top-left aligned, the
 * reference's rule at src/attn_kernel_torch.cu:54,238,263).  Skv == 0 gives
 * an all-zero output, like the reference's empty-denominator rule
 * (src/attn_kernel_torch.cu:335-336).
 * Supported: dtype ATTN_F16 / ATTN_BF16 / ATTN_F32 and 1 <= D <= 256, every
 * pointer aligned to its element size.  fp16/bf16 with D in {64, 128} and
 * 16-byte aligned buffers run the tcgen05 tensor-core kernel; every other
 * supported call runs the general kernel (fp32 arithmetic), which covers the
 * reference's fp32 and D=16 routes (src/attn_kernel_torch.cu:625-689).
 * Asynchronous on `stream`; allocates nothing; re-entrant.
 * Returns ATTN_OK or an AttnStatus code; on error nothing was launched.
 */
ATTN_API int launch_attn_forward(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv,
                        int D, bool causal, float softmax_scale, AttnDType dtype, cudaStream_t stream);

/*
 * launch_attn_forward on strided q, k and v: each *_strides array holds the
 * element strides over (batch, head, row), the head dim being contiguous; a
 * null array means the contiguous layout.  For example the [B, L, H, D]
 * layout of flash-style callers viewed as [B, H, L, D] has strides
 * {L*H*D, D, H*D}.  out stays contiguous [B, H, Sq, D].  The tensor-core
 * kernel reads strided inputs directly through TMA when every stride is a
 * multiple of 16 bytes; otherwise the general kernel runs.  Strides must be
 * >= 0.  No counterpart in the reference, whose binding copies inputs to
 * contiguous tensors first (src/attn_torch.cpp:20-22).
 */
ATTN_API int launch_attn_forward_strided(const void* q, const void* k, const void* v, void* out, int B, int H,
                                         int Sq, int Skv, int D, bool causal, float softmax_scale, AttnDType dtype,
                                         const long long* q_strides, const long long* k_strides,
                                         const long long* v_strides, cudaStream_t stream);

/*
 * One problem of launch_attn_forward_batch: the arguments of
 * launch_attn_forward_strided for one call (null strides: contiguous).
 */
typedef struct AttnProblem {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int B, H, Sq, Skv, D;
  bool causal;
  float softmax_scale;
  const long long* q_strides;
  const long long* k_strides;
  const long long* v_strides;
} AttnProblem;

/*
 * Runs n independent problems of one dtype, as launch_attn_forward_strided
 * would one by one, with the same results bit for bit, in fewer launches:
 * the problems that run the tcgen05 tensor-core kernel with the same head
 * dim, masking and tile shape share one grid (up to 16 problems per grid),
 * whose work units are ordered longest first, so the short units of one
 * problem fill the last wave of another and no launch waits for the tail of
 * the previous one.  Short problems (fp16/bf16, at most 16 queries and 64
 * keys) with the same head dim and 16-key group count share one grid of the
 * warp-level tensor-core kernel the same way.  The others are launched one
 * by one.  Every problem is
 * checked before anything is launched; on an error nothing was launched.
 * The output buffers must not overlap any input or each other.  No
 * counterpart in the reference, whose benchmark launches one shape at a time
 * (benchmark/bench_attention.py:81-100,171-175).
 */
ATTN_API int launch_attn_forward_batch(const AttnProblem* problems, int n, AttnDType dtype, cudaStream_t stream);

/*
 * Reads and clears the device status word of the current device, after
 * synchronising `stream`.  *status receives ATTN_OK, or ATTN_ERR_WATCHDOG when a
 * kernel launched earlier gave up on a wait (its output is then invalid).
 * No counterpart in the reference, whose launcher has no error reporting.
 * Returns ATTN_OK, or ATTN_ERR_LAUNCH if the synchronisation itself failed.
 */
ATTN_API int attn_get_status(cudaStream_t stream, int* status);

/*
 * Sets the limit, in nanoseconds, of each pipeline wait inside the
 * tensor-core kernel for launches queued from now on (all devices); 0 restores
 * the default of 2 s.  The clock is checked each time the hardware's own
 * suspension of an mbarrier wait ends without the awaited arrival, so a
 * legitimate wait (microseconds) never expires whatever the limit, and a
 * lost arrival ends the wait after about the limit: the kernel then records
 * ATTN_ERR_WATCHDOG (read with attn_get_status), lets the copies and products
 * it already issued finish under the default limit, frees its tensor memory
 * and returns.  Returns the previous limit (0 = default).  No counterpart in
 * the reference, whose kernels have no bounded waits.
 */
ATTN_API unsigned long long attn_set_wait_limit_ns(unsigned long long ns);

/* Library version, major * 10000 + minor * 100 + patch.  No reference
 * counterpart; lets a binding check which build it loaded. */
ATTN_API int attn_library_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ROCM_ATTN_B200_ATTN_KERNEL_H_ */
