// Grouped launches of the tcgen05 attention-forward kernel: several
// independent problems (shapes) that run the same instantiation share one
// grid, for launch_attn_forward_batch (attn_kernel.cu).
//
// The reference's benchmark runs a sequence of shapes one launch after the
// other (benchmark/bench_attention.py:81-100,171-175; the UnifoLM preset
// list benchmark/attn_shapes_unifolm_infer.txt has 17 of them).  Launched
// one by one, every shape pays a launch and a last wave in which SMs idle
// while its final units finish.  In one grid the CTAs of all problems are
// ordered longest unit first, so the short units of the later problems fill
// the SMs the long ones leave idle, and there is one launch.
//
// Each CTA finds its problem from the per-problem unit ranges in the kernel
// arguments (FwdArgs<kGroupMax>: tensor maps and parameters of up to 16
// problems, about 9 KB, passed as a __grid_constant__ block) and then runs
// exactly the code of a single-problem launch on it, so every problem's
// output is identical to that of its own launch.

#include "attn_fwd.cuh"

#include <algorithm>
#include <numeric>

namespace ra {

constexpr int kGroupMax = 16;

int status_word_read_clear_grouped(cudaStream_t stream, int* host) {
  static const int zero = 0;
  return cudaMemcpyFromSymbolAsync(host, g_attn_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) ==
                     cudaSuccess &&
                 cudaMemcpyToSymbolAsync(g_attn_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream) ==
                     cudaSuccess
             ? 0
             : -1;
}

namespace {

// Key blocks of the longest work unit of problem d (a unit's duration is
// about proportional to it).
long long unit_cost(const TcKey& key, const FwdProblem& d) {
  const long long blocks = (d.Skv + key.keys - 1) / key.keys;
  if (!key.causal) return blocks;
  return std::min<long long>(blocks, (d.Sq - 1) / key.keys + 1);  // the unit holding the last query row
}

template <bool kBf16, int kD, bool kCausal, int kTiles, int kBlockKeys>
int launch_group(const FwdProblem* d, const std::vector<int>& order, cudaStream_t stream,
                 std::vector<int>* fallback) {
  FwdArgs<kGroupMax> a;
  int m = 0;
  long long end = 0;
  auto flush = [&]() -> int {
    if (m == 0) return ATTN_OK;
    a.n = m;
    const int st = launch_fwd<kBf16, kD, kCausal, kTiles, kBlockKeys, kGroupMax>(a, stream);
    m = 0;
    end = 0;
    return st;
  };
  for (int idx : order) {
    const FwdProblem& p = d[idx];
    const int e = encode_problem<kBf16, kD, kTiles, kBlockKeys, kGroupMax>(p, a, m);
    if (e == kNoTensorMap) {
      fallback->push_back(idx);
      continue;
    }
    if (e != 0) return e;
    end += problem_units<kD, kTiles, kBlockKeys>(p);
    if (end > 0x7fffffffLL) return ATTN_ERR_INVALID_ARGUMENT;
    a.unit_end[m++] = static_cast<int>(end);
    if (m == kGroupMax) {
      const int st = flush();
      if (st != ATTN_OK) return st;
    }
  }
  return flush();
}

}  // namespace

int launch_tc_grouped(const TcKey& key, const FwdProblem* d, int n, cudaStream_t stream,
                      std::vector<int>* fallback) {
  if (n <= 0) return ATTN_OK;
  if (n == 1) {  // a single problem takes the smaller argument block
    const int st = launch_tc_single(key, d[0], stream);
    if (st == kNoTensorMap) {
      fallback->push_back(0);
      return ATTN_OK;
    }
    return st;
  }
  // Longest units first across the problems (a stable order keeps equal
  // problems in the caller's order).
  std::vector<int> order(static_cast<size_t>(n));
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int x, int y) { return unit_cost(key, d[x]) > unit_cost(key, d[y]); });
  int st = ATTN_ERR_UNSUPPORTED;
#define RA_DISPATCH(BF, DD, CA, TILES, KEYS)                                     \
  if (key.bf16 == BF && key.D == DD && key.causal == CA && key.keys == KEYS)     \
    st = launch_group<BF, DD, CA, TILES, KEYS>(d, order, stream, fallback);      \
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
