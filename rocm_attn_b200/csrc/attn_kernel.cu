// C-ABI entry points of the attention-forward library and their dispatcher.
//
// Replaces the reference's launcher (src/attn_kernel_torch.cu:625-689,
// src/attn_kernel.hip.cpp:304-367 of JoursBleu/rocm_attn), which picks one of
// its HIP kernels by head dim and shared-memory size.  Here `prepare` checks
// a call and picks its route without queueing anything, and `run` launches
// it: short sequences, mid-length sequences, fp32 and other head dims go to
// the kernels of attn_general.cu; fp16/bf16 at D = 64 / 128 with buffers TMA
// can describe go to the tcgen05 kernel of attn_fwd.cuh, one grid per call
// (here) or several problems per grid (attn_group.cu, for
// launch_attn_forward_batch).  Also: the watchdog's status word and limit,
// and, in the watchdog test build only, the hook that loses one arrival.

#include "attn_fwd.cuh"
#include "attn_general.h"

#include <atomic>
#include <vector>

namespace ra {

// Pipeline wait limit for launches from now on (attn_set_wait_limit_ns);
// 0 selects kWaitTimeoutNs.
static std::atomic<unsigned long long> g_wait_limit_ns{0};
unsigned long long wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }
#ifdef RA_WATCHDOG_TEST
static std::atomic<int> g_drop_arrival{0};
int drop_arrival_requested() { return g_drop_arrival.load(std::memory_order_relaxed); }
#else
int drop_arrival_requested() { return 0; }
#endif

// One problem, one launch.
template <bool kBf16, int kD, bool kCausal, int kTiles, int kBlockKeys>
static int launch_impl(const FwdProblem& d, cudaStream_t stream) {
  FwdArgs<1> a;
  const int e = encode_problem<kBf16, kD, kTiles, kBlockKeys, 1>(d, a, 0);
  if (e != 0) return e;
  const long long units = problem_units<kD, kTiles, kBlockKeys>(d);
  if (units > 0x7fffffffLL) return ATTN_ERR_INVALID_ARGUMENT;
  a.unit_end[0] = static_cast<int>(units);
  a.n = 1;
  return launch_fwd<kBf16, kD, kCausal, kTiles, kBlockKeys, 1>(a, stream);
}

// Multiprocessor count of the current device, cached per device (0 if it
// cannot be read).
static int sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// D=64 problems for 64-key blocks: four 64-key CTAs per SM hide the fixed
// cost of a CTA (set-up, first block, epilogue) and each other's softmax
// latency better than two 128-key ones whenever the grid fills the SMs at
// least twice over (measured: 2-11 % faster up to 2048 keys, equal from 2560
// to 8192); on smaller grids the 128-key CTAs are 8-16 % faster.
static bool d64_use_64_key_blocks(long long ctas) { return ctas >= 2LL * sm_count(); }

// Compute capability 10.x check, cached per device.
static int check_device() {
  static std::atomic<int> cached[64];  // 0 unknown, 1 ok, 2 not sm_100
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ATTN_ERR_DEVICE;
  int state = cached[dev].load(std::memory_order_relaxed);
  if (state == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return ATTN_ERR_DEVICE;
    state = (major == 10 && minor == 0) ? 1 : 2;
    cached[dev].store(state, std::memory_order_relaxed);
  }
  return state == 1 ? ATTN_OK : ATTN_ERR_DEVICE;
}

}  // namespace ra

namespace ra {

// Which kernel runs a call, decided from its sizes, dtype and buffers.
enum class Route { kEmpty, kZeroFill, kSmall, kMid, kGeneral, kTensorCore };

// A validated call: its problem, route and, for the tensor-core route, the
// kernel instantiation.
struct Call {
  FwdProblem prob;
  int D;
  bool causal;
  AttnDType dtype;
  GeneralStrides gs;
  Route route;
  TcKey key;
};

// Checks the arguments and picks the route; no CUDA work is queued.  Returns
// ATTN_OK or the status the entry point reports.
static int prepare(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq, int Skv, int D,
                   bool causal, float softmax_scale, AttnDType dtype, const long long* q_strides,
                   const long long* k_strides, const long long* v_strides, Call* c) {
  if (B < 0 || H < 0 || Sq < 0 || Skv < 0 || D <= 0) return ATTN_ERR_INVALID_ARGUMENT;
  if (dtype != ATTN_F16 && dtype != ATTN_BF16 && dtype != ATTN_F32) return ATTN_ERR_UNSUPPORTED;
  if (D > kGeneralMaxHeadDim) return ATTN_ERR_UNSUPPORTED;
  const long long BH = static_cast<long long>(B) * H;
  c->route = Route::kEmpty;
  if (BH == 0 || Sq == 0) return ATTN_OK;  // empty output, nothing to do
  if (BH > 0x7fffffffLL) return ATTN_ERR_INVALID_ARGUMENT;
  if (!q || !out || (Skv > 0 && (!k || !v))) return ATTN_ERR_INVALID_ARGUMENT;
  // Strides over (batch, head, row) in elements; null means contiguous.
  auto strides_of = [&](const long long* st, int L, Strides* o) {
    if (!st) {
      *o = Strides{static_cast<long long>(H) * L * D, static_cast<long long>(L) * D, D};
      return true;
    }
    *o = Strides{st[0], st[1], st[2]};
    return o->b >= 0 && o->h >= 0 && o->l >= 0;
  };
  Strides sq, sk, sv;
  if (!strides_of(q_strides, Sq, &sq) || !strides_of(k_strides, Skv, &sk) || !strides_of(v_strides, Skv, &sv))
    return ATTN_ERR_INVALID_ARGUMENT;
  const size_t elem = dtype == ATTN_F32 ? 4 : 2;
  auto aligned = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; };
  if (!aligned(q, elem) || !aligned(out, elem) || (Skv > 0 && (!aligned(k, elem) || !aligned(v, elem))))
    return ATTN_ERR_MISALIGNED;
  const int dev_ok = check_device();
  if (dev_ok != ATTN_OK) return dev_ok;
  float scale = softmax_scale;
  if (!(scale > 0.f) || !isfinite(scale)) scale = 1.0f / sqrtf(static_cast<float>(D));
  c->prob = FwdProblem{q, k, v, out, B, H, Sq, Skv, sq, sk, sv, scale};
  c->D = D;
  c->causal = causal;
  c->dtype = dtype;
  c->gs = GeneralStrides{{sq.b, sq.h, sq.l}, {sk.b, sk.h, sk.l}, {sv.b, sv.h, sv.l}};
  const int dt = static_cast<int>(dtype);
  if (Skv == 0) {
    c->route = Route::kZeroFill;
  } else if (small_kernel_takes(Sq, Skv, D, dt)) {
    // Short sequences (a few dozen rows per head): one warp per (batch,
    // head) slice instead of a mostly empty 128- or 256-row tcgen05 unit.
    c->route = Route::kSmall;
  } else if (mid_kernel_takes(Sq, Skv, D, dt) &&
             !(D == 64 && Skv > 64 && d64_use_64_key_blocks(BH * ((Sq + 127) / 128)))) {
    // D = 16 / 32 at any length, and D = 64 with at most 64 queries and 256
    // keys: 64-row warp-level tensor-core tiles instead of 128-row tcgen05
    // tiles.  At D = 64 only where the tcgen05 kernel would not run four
    // 64-key CTAs per SM or the keys fit one 64-key chunk: with more keys on
    // such grids the tcgen05 kernel measured 15-28 % faster (e.g. 64x16x48x256,
    // 32x16x56x200), with 64 keys or fewer 15-25 % slower.
    c->route = Route::kMid;
  } else if (dtype == ATTN_F32 || (D != 64 && D != 128) || !aligned(out, 16)) {
    // The tensor-core kernel takes fp16/bf16 with D in {64, 128} and
    // buffers TMA can describe (16-byte aligned base and strides); every
    // other call runs the general kernel.
    c->route = Route::kGeneral;
  } else {
    c->route = Route::kTensorCore;
    // D=128: two-tile CTAs.  D=64: one-tile CTAs with 128-key blocks (two
    // per SM), or with 64-key blocks (four per SM) on grids of at least two
    // CTAs per SM.
    c->key = TcKey{dtype == ATTN_BF16, D, causal,
                   (D == 64 && d64_use_64_key_blocks(BH * ((Sq + 127) / 128))) ? 64 : 128};
  }
  return ATTN_OK;
}

static int run_general(const Call& c, cudaStream_t stream) {
  const FwdProblem& d = c.prob;
  return launch_attn_general(d.q, d.k, d.v, d.out, d.B, d.H, d.Sq, d.Skv, c.D, c.causal, d.scale,
                             static_cast<int>(c.dtype), c.gs, stream) == 0
             ? ATTN_OK
             : ATTN_ERR_LAUNCH;
}

// Launches one prepared call on its route.  A short or mid-length launcher
// that returns non-zero launched nothing (-2: rows not 16-byte aligned; -1:
// it could not be configured), and the general kernel, which takes every
// problem, runs instead; so does a tensor-core call whose buffers TMA cannot
// describe.
static int run(const Call& c, cudaStream_t stream) {
  const FwdProblem& d = c.prob;
  const int dt = static_cast<int>(c.dtype);
  switch (c.route) {
    case Route::kEmpty:
      return ATTN_OK;
    case Route::kZeroFill:
      // No keys: every row's softmax denominator is empty; the reference
      // writes zeros in that case.
      return cudaMemsetAsync(d.out, 0, static_cast<size_t>(d.B) * d.H * d.Sq * c.D * (dt == 2 ? 4 : 2), stream) ==
                     cudaSuccess
                 ? ATTN_OK
                 : ATTN_ERR_LAUNCH;
    case Route::kSmall:
      if (launch_attn_small(d.q, d.k, d.v, d.out, d.B, d.H, d.Sq, d.Skv, c.D, c.causal, d.scale, dt, c.gs, stream) ==
          0)
        return ATTN_OK;
      if (mid_kernel_takes(d.Sq, d.Skv, c.D, dt) &&
          launch_attn_mid(d.q, d.k, d.v, d.out, d.B, d.H, d.Sq, d.Skv, c.D, c.causal, d.scale, dt, c.gs, stream) == 0)
        return ATTN_OK;
      return run_general(c, stream);
    case Route::kMid:
      if (launch_attn_mid(d.q, d.k, d.v, d.out, d.B, d.H, d.Sq, d.Skv, c.D, c.causal, d.scale, dt, c.gs, stream) == 0)
        return ATTN_OK;
      return run_general(c, stream);
    case Route::kGeneral:
      return run_general(c, stream);
    case Route::kTensorCore: {
      const int st = launch_tc_single(c.key, c.prob, stream);
      return st == kNoTensorMap ? run_general(c, stream) : st;
    }
  }
  return ATTN_ERR_UNSUPPORTED;
}

// One tensor-core problem per launch (kMaxProblems = 1).
int launch_tc_single(const TcKey& key, const FwdProblem& d, cudaStream_t stream) {
  int st = ATTN_ERR_UNSUPPORTED;
#define RA_DISPATCH(BF, DD, CA, TILES, KEYS)                                         \
  if (key.bf16 == BF && key.D == DD && key.causal == CA && key.keys == KEYS)         \
    st = launch_impl<BF, DD, CA, TILES, KEYS>(d, stream);                            \
  else
  RA_DISPATCH(false, 128, false, 2, 128)
  RA_DISPATCH(false, 128, true, 2, 128)
  RA_DISPATCH(false, 64, false, 1, 128)
  RA_DISPATCH(false, 64, true, 1, 128)
  RA_DISPATCH(false, 64, false, 1, 64)
  RA_DISPATCH(false, 64, true, 1, 64)
  RA_DISPATCH(true, 128, false, 2, 128)
  RA_DISPATCH(true, 128, true, 2, 128)
  RA_DISPATCH(true, 64, false, 1, 128)
  RA_DISPATCH(true, 64, true, 1, 128)
  RA_DISPATCH(true, 64, false, 1, 64)
  RA_DISPATCH(true, 64, true, 1, 64) {}
#undef RA_DISPATCH
  return st;
}

}  // namespace ra

extern "C" int launch_attn_forward_strided(const void* q, const void* k, const void* v, void* out, int B, int H,
                                           int Sq, int Skv, int D, bool causal, float softmax_scale, AttnDType dtype,
                                           const long long* q_strides, const long long* k_strides,
                                           const long long* v_strides, cudaStream_t stream) {
  ra::Call c;
  const int st = ra::prepare(q, k, v, out, B, H, Sq, Skv, D, causal, softmax_scale, dtype, q_strides, k_strides,
                             v_strides, &c);
  if (st != ATTN_OK) return st;
  return ra::run(c, stream);
}

extern "C" int launch_attn_forward_batch(const AttnProblem* problems, int n, AttnDType dtype, cudaStream_t stream) {
  using namespace ra;
  if (n < 0 || (n > 0 && !problems)) return ATTN_ERR_INVALID_ARGUMENT;
  // Every problem is checked before anything is launched.
  std::vector<Call> calls(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) {
    const AttnProblem& p = problems[i];
    const int st = prepare(p.q, p.k, p.v, p.out, p.B, p.H, p.Sq, p.Skv, p.D, p.causal, p.softmax_scale, dtype,
                           p.q_strides, p.k_strides, p.v_strides, &calls[static_cast<size_t>(i)]);
    if (st != ATTN_OK) return st;
  }
  // Problems of the tensor-core route that share an instantiation run as one
  // grid (launch_tc_grouped), and so do short problems of the warp-level
  // tensor-core kernel with the same head dim and key-group count
  // (launch_attn_small_grouped); the others launch one by one.
  const int dt = static_cast<int>(dtype);
  std::vector<bool> done(static_cast<size_t>(n), false);
  for (int i = 0; i < n; ++i) {
    if (done[static_cast<size_t>(i)]) continue;
    const Call& c = calls[static_cast<size_t>(i)];
    const int nk = c.route == Route::kSmall ? small_mma_group_key(c.prob.Sq, c.prob.Skv, c.D, dt) : 0;
    if (nk > 0) {
      std::vector<SmallProblem> group;
      std::vector<int> members;
      for (int j = i; j < n; ++j) {
        const Call& o = calls[static_cast<size_t>(j)];
        if (!done[static_cast<size_t>(j)] && o.route == Route::kSmall && o.D == c.D &&
            small_mma_group_key(o.prob.Sq, o.prob.Skv, o.D, dt) == nk) {
          const FwdProblem& d = o.prob;
          group.push_back(SmallProblem{d.q, d.k, d.v, d.out, d.B, d.H, d.Sq, d.Skv, o.causal, d.scale, o.gs});
          members.push_back(j);
          done[static_cast<size_t>(j)] = true;
        }
      }
      std::vector<int> fallback;
      if (launch_attn_small_grouped(group.data(), static_cast<int>(group.size()), c.D, dt, stream, &fallback) != 0)
        return ATTN_ERR_LAUNCH;
      for (int f : fallback) {  // rows not 16-byte aligned: the single-call route and its fallbacks
        const int g = run(calls[static_cast<size_t>(members[static_cast<size_t>(f)])], stream);
        if (g != ATTN_OK) return g;
      }
      continue;
    }
    if (c.route != Route::kTensorCore) {
      const int st = run(c, stream);
      if (st != ATTN_OK) return st;
      done[static_cast<size_t>(i)] = true;
      continue;
    }
    std::vector<FwdProblem> group;
    std::vector<int> members;
    for (int j = i; j < n; ++j) {
      const Call& o = calls[static_cast<size_t>(j)];
      if (!done[static_cast<size_t>(j)] && o.route == Route::kTensorCore && o.key == c.key) {
        group.push_back(o.prob);
        members.push_back(j);
        done[static_cast<size_t>(j)] = true;
      }
    }
    std::vector<int> fallback;
    const int st = launch_tc_grouped(c.key, group.data(), static_cast<int>(group.size()), stream, &fallback);
    if (st != ATTN_OK) return st;
    for (int f : fallback) {  // buffers TMA cannot describe: the general kernel
      const int g = run_general(calls[static_cast<size_t>(members[static_cast<size_t>(f)])], stream);
      if (g != ATTN_OK) return g;
    }
  }
  return ATTN_OK;
}

extern "C" int launch_attn_forward(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq,
                                   int Skv, int D, bool causal, float softmax_scale, AttnDType dtype,
                                   cudaStream_t stream) {
  return launch_attn_forward_strided(q, k, v, out, B, H, Sq, Skv, D, causal, softmax_scale, dtype, nullptr, nullptr,
                                     nullptr, stream);
}

namespace ra {
// Queues a copy of this translation unit's status word into *host and a
// reset of the word on `stream`.
int status_word_read_clear_single(cudaStream_t stream, int* host) {
  static const int zero = 0;
  return cudaMemcpyFromSymbolAsync(host, g_attn_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) ==
                     cudaSuccess &&
                 cudaMemcpyToSymbolAsync(g_attn_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream) ==
                     cudaSuccess
             ? 0
             : -1;
}
}  // namespace ra

extern "C" int attn_get_status(cudaStream_t stream, int* status) {
  if (!status) return ATTN_ERR_INVALID_ARGUMENT;
  int single = 0, grouped = 0;
  if (ra::status_word_read_clear_single(stream, &single) != 0 ||
      ra::status_word_read_clear_grouped(stream, &grouped) != 0 || cudaStreamSynchronize(stream) != cudaSuccess)
    return ATTN_ERR_LAUNCH;
  *status = (single == 0 && grouped == 0) ? ATTN_OK : ATTN_ERR_WATCHDOG;
  return ATTN_OK;
}

extern "C" unsigned long long attn_set_wait_limit_ns(unsigned long long ns) {
  return ra::g_wait_limit_ns.exchange(ns);
}

extern "C" int attn_library_version(void) { return 200; }

#ifdef RA_WATCHDOG_TEST
// Watchdog test build only (librocm_attn_wdtest.so, never the product
// library): with `on` set, every later tensor-core launch loses one P arrival
// in CTA 0, so that its wait can only end by the watchdog.
extern "C" ATTN_API void attn_test_drop_arrival(int on) { ra::g_drop_arrival.store(on); }
#endif

#ifdef RA_TRACE
// Trace builds only: selects the traced CTA and copies the timeline out.
extern "C" ATTN_API int attn_trace_read(int next_cta, unsigned long long* host, int n) {
  if (cudaDeviceSynchronize() != cudaSuccess) return ATTN_ERR_LAUNCH;
  if (host && n > 0 &&
      cudaMemcpyFromSymbol(host, ra::g_attn_trace, sizeof(unsigned long long) * (n < ra::kTraceSlots ? n : ra::kTraceSlots)) !=
          cudaSuccess)
    return ATTN_ERR_LAUNCH;
  static unsigned long long zeros[ra::kTraceSlots];
  if (cudaMemcpyToSymbol(ra::g_attn_trace, zeros, sizeof(zeros)) != cudaSuccess ||
      cudaMemcpyToSymbol(ra::g_attn_trace_cta, &next_cta, sizeof(int)) != cudaSuccess)
    return ATTN_ERR_LAUNCH;
  return ATTN_OK;
}
#endif
