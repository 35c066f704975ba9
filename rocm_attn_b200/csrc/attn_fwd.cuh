// The tcgen05 attention-forward kernel (device code) and the host helpers
// that encode its problems and launch it, shared by the single-problem entry
// points (attn_kernel.cu) and the grouped launch of several problems
// (attn_group.cu).
//
// Replaces the reference's HIP kernels and their launcher
// (src/attn_kernel_torch.cu:36-689, src/attn_kernel.hip.cpp:36-367 of
// JoursBleu/rocm_attn).  The math is the reference's: per query row,
// s_j = (q . k_j) * scale, masked when causal and j > i
// (src/attn_kernel_torch.cu:54,238,263), softmax in the exp2 domain with a
// running fp32 max and sum (src/attn_kernel_torch.cu:269-298), O = P V / sum
// (src/attn_kernel_torch.cu:333-354).
//
// CTA work unit.  D=128: 256 query rows of one (batch, head) as two 128-row
// Q tiles, one CTA per SM.  D=64: one 128-row tile, two CTAs per SM with
// 128-key blocks, four with 64-key blocks (grids of two or more CTAs per SM).
// Warp roles (320 threads with two tiles, 192 with one):
//   warps 0-3  softmax of Q tile 0 (thread <-> TMEM lane <-> query row)
//   warps 4-7  softmax of Q tile 1 (two-tile CTAs)
//   next warp  UMMA issue (one elected lane) and TMEM allocation
//   last warp  TMA producer for K/V blocks 1.. of 128 or 64 keys (thread 0 starts
//              the Q tiles and block 0 during setup)
// Tensor memory (128 lanes x 32 bit; 512 columns for two tiles, 256 or 128
// for one):
//   D=128: S0 [0,128) S1 [128,256) fp32 scores of the current key block;
//          P0 = S0 cols [0,64), P1 = S1 cols [0,64) (16-bit, aliasing S);
//          O0 [256,384) O1 [384,512) fp32 output accumulators
//   D=64:  S [0,128), P [128,192) apart from S, O [192,256); with 64-key
//          blocks S [0,64), P aliasing S cols [0,32), O [64,128)
// UMMA issue order per key block j at D=128 (tcgen05.mma executes in issue
// order):
//   S0(j)=Q0 K_j^T, O1+=P1(j-1) V_{j-1}, S1(j)=Q1 K_j^T, O0+=P0(j) V_j
// so each softmax warpgroup works while the tensor core runs the other tile;
// at D=64 with 128-key blocks, S(j+1) is issued as soon as the softmax has
// read S(j), and the other CTAs on the SM keep the tensor core busy meanwhile.
// The running max is only moved (and O rescaled) when it grows by more than
// 2^8 in the exp2 domain; P values stay <= 256, exact in fp16/bf16 range, and
// the final division by the matching running sum makes the result identical
// in exact arithmetic.

#pragma once

#include "sm100_ptx.cuh"
#include "tensor_map.h"
#include "attn_kernel.h"

#include <math.h>

#include <mutex>
#include <vector>

namespace ra {

// Sticky per-device status word written by the kernel's watchdog (one per
// translation unit that includes this header; attn_get_status reads them all).
static __device__ int g_attn_status = 0;

// Optional device-side timeline of one CTA (build with -DRA_TRACE): lane 0 of
// each role writes %clock64 at fixed points of every key block into
// g_attn_trace, read back with attn_trace_read().  Compiled out by default.
#ifdef RA_TRACE
constexpr int kTraceSlots = 8192;
static __device__ unsigned long long g_attn_trace[kTraceSlots];
static __device__ int g_attn_trace_cta = 0;
#define RA_MARK(idx)                                                                      \
  do {                                                                                    \
    if ((threadIdx.x & 31) == 0 && ra_traced &&                                           \
        (idx) < kTraceSlots)                                                              \
      g_attn_trace[(idx)] = clock64();                                                    \
  } while (0)
#else
#define RA_MARK(idx) \
  do {               \
  } while (0)
#endif

enum : int { kWatchQ = 0x10, kWatchK = 0x20, kWatchV = 0x30, kWatchS = 0x40, kWatchP = 0x50, kWatchO = 0x60,
             kWatchDrain = 0x70 };

struct AttnParams {
  int Lq;           // query rows per (batch, head)
  int Lk;           // key rows per (batch, head)
  int BH;           // batch * heads
  int H;            // heads (TMA coordinates are (d, row, head, batch))
  int num_qblocks;  // ceil(Lq / query rows per CTA)
  int head_group;   // causal: heads per scheduling group (their K/V fit in L2)
  float scale_log2; // softmax scale * log2(e)
  void* out;        // O, contiguous [B, H, Lq, D] (16-byte aligned: its tensor map was encoded)
  unsigned long long wait_ns;  // limit of every pipeline wait (the watchdog)
  int drop_arrival;            // watchdog test build only: lose one P arrival of CTA 0
};

// Compile-time shape of the pipeline for head dimension kD, kTiles 128-row
// Q tiles per CTA and kBlockKeys keys per K/V block.
template <int kD, int kTiles, int kBlockKeys>
struct Cfg {
  static_assert(kTiles == 1 || kTiles == 2, "one or two Q tiles per CTA");
  static_assert(kBlockKeys == 128 || (kBlockKeys == 64 && kD == 64 && kTiles == 1),
                "64-key blocks only for one-tile D=64 CTAs");
  static constexpr int kBM = 128;                       // rows per Q tile
  static constexpr int kBN = kBlockKeys;                // keys per block
  static constexpr int kRows = kBM * kTiles;            // query rows per CTA
  // K / V ring depths.  One-tile CTAs run two (four with 64-key blocks) per
  // SM, so each keeps to its share of the SM's shared memory: four 64-key
  // CTAs with two-stage rings measured 6-11 % faster than three with
  // three-stage rings on short key ranges.
  static constexpr int kStagesK = (kD == 64 && kTiles == 2) ? 3 : 2;
  static constexpr int kStagesV = kStagesK;
  static constexpr uint32_t kTileBytes = 128u * kD * 2; // one 128 x D Q tile
  static constexpr uint32_t kBlockBytes = 128u * 128;   // one 64-column block of a Q tile
  static constexpr uint32_t kKVBytes = kBN * kD * 2u;   // one K or V block
  static constexpr uint32_t kKVBlockBytes = kBN * 128u; // one 64-column block of a K or V block
  static constexpr uint32_t kSmemBytes = 1024 + kTiles * kTileBytes + (kStagesK + kStagesV) * kKVBytes;
  // D=64 with 128-key blocks leaves TMEM room for P apart from S: the scores
  // of block j+1 can then be computed while the softmax of block j is still
  // running.  Otherwise P aliases the first half of S.
  static constexpr bool kSepP = kD == 64 && kBN == 128;
  static constexpr uint32_t kTmemCols = kTiles == 2 ? 512 : (kBN == 64 ? 128 : 256);
  static constexpr uint32_t kColP = kBN * kTiles;                            // P per tile (64 columns) when kSepP
  static constexpr uint32_t kColO = kSepP ? kColP + 64 * kTiles : kBN * kTiles;  // O per tile (kD columns)
  static constexpr int kMmaWarp = 4 * kTiles;            // after the softmax warpgroups
  static constexpr int kTmaWarp = 4 * kTiles + 1;
  static constexpr int kThreads = 128 * kTiles + 64;
  static constexpr int kMinBlocksPerSm = kTiles == 2 ? 1 : (kBN == 64 ? 4 : 2);  // one-tile CTAs share an SM
};

// Fraction of the softmax exponentials evaluated by the FMA-pipe polynomial
// (exp2_poly2) instead of the MUFU: pairs i with (i % kPolyDen) < kPolyNum.
#ifndef RA_POLY_NUM
#define RA_POLY_NUM 1
#endif
#ifndef RA_POLY_DEN
#define RA_POLY_DEN 4
#endif
constexpr int kPolyNum = RA_POLY_NUM;
constexpr int kPolyDen = RA_POLY_DEN;

struct __align__(8) SharedCtl {
  uint64_t q_full[2];     // [tile]: Q tile loaded
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[3], v_empty[3];
  uint64_t s_full[2];     // [tile]: S(j) computed
  uint64_t s_free[2];     // [tile]: softmax done reading S(j) (128 arrivals; separate-P layout)
  uint64_t p_free[2];     // [tile]: one phase per retired P*V product (separate-P layout)
  uint64_t p_full[2][2];  // [tile][64-key half]: P(j) half stored (128 arrivals)
  uint64_t o_full[2];     // [tile]: the last P*V product retired
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

// Number of bn-key blocks Q tile `t` of the CTA starting at row q0 needs.
__device__ __forceinline__ int tile_key_blocks(int q0, int t, int Lq, int Lk, bool causal, int bn) {
  const int first = q0 + t * 128;
  if (first >= Lq) return 0;
  const int all = (Lk + bn - 1) / bn;
  if (!causal) return all;
  const int last = min(first + 127, Lq - 1);
  return min(all, last / bn + 1);
}

// exp2 of 32 consecutive scores (relative to the reference point -nmc2/c2),
// packed to 16-bit pairs; returns the fp32 sum of the exponentials in `sum2`.
template <bool kBf16, int kSrc, int kDst, int kN>
__device__ __forceinline__ void exp_pack32(const float (&s)[kN], uint64_t c2, uint64_t nmc2, uint32_t (&pk)[32],
                                           uint64_t& sum2) {
  static_assert(kSrc + 32 <= kN && kDst + 16 <= 32, "source or destination out of range");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t x = f2_fma(f2(s[kSrc + 2 * i], s[kSrc + 2 * i + 1]), c2, nmc2);
    float x0, x1, a, b;
    f2_split(x, x0, x1);
    if ((i % kPolyDen) < kPolyNum) {
      exp2_poly2(x0, x1, a, b);  // FMA pipe
    } else {
      a = ex2_approx(x0);        // MUFU
      b = ex2_approx(x1);
    }
    sum2 = f2_add(sum2, f2(a, b));
    pk[kDst + i] = pack2<kBf16>(a, b);
  }
}

// Kernel arguments: up to kMaxProblems independent attention problems of the
// same dtype, head dim, masking and tile shape; CTA indices
// [unit_end[i-1], unit_end[i]) are the work units of problem i.  Single calls
// use kMaxProblems = 1; the grouped launch of several shapes uses more, and
// lists its problems longest units first.
template <int kMaxProblems>
struct FwdArgs {
  CUtensorMap map[kMaxProblems][4];  // q, k, v, o of each problem
  AttnParams prm[kMaxProblems];
  int unit_end[kMaxProblems];
  int n;
};

template <bool kBf16, int kD, bool kCausal, int kTiles, int kBlockKeys, int kMaxProblems>
__global__ void __launch_bounds__(Cfg<kD, kTiles, kBlockKeys>::kThreads, Cfg<kD, kTiles, kBlockKeys>::kMinBlocksPerSm)
    attn_fwd_kernel(const __grid_constant__ FwdArgs<kMaxProblems> args) {
  using C = Cfg<kD, kTiles, kBlockKeys>;
  // This CTA's problem and its work unit within it.
  int pi = 0;
  if constexpr (kMaxProblems > 1) {
    while (pi + 1 < args.n && static_cast<int>(blockIdx.x) >= args.unit_end[pi]) ++pi;
  }
  const int unit = static_cast<int>(blockIdx.x) - (pi > 0 ? args.unit_end[pi - 1] : 0);
  const AttnParams p = args.prm[pi];
  const CUtensorMap* map_q = &args.map[pi][0];
  const CUtensorMap* map_k = &args.map[pi][1];
  const CUtensorMap* map_v = &args.map[pi][2];
  const CUtensorMap* map_o = &args.map[pi][3];
  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                    // kTiles tiles
  uint8_t* sK = smem + kTiles * C::kTileBytes;           // kStagesK blocks
  uint8_t* sV = sK + C::kStagesK * C::kKVBytes;         // kStagesV blocks
  volatile int* abort_flag = &ctl.abort_flag;
  int* status = &g_attn_status;
  const uint64_t wait_ns = p.wait_ns;

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x) / 32, 0);
  const int lane = threadIdx.x & 31;
#ifdef RA_TRACE
  const bool ra_traced = static_cast<int>(blockIdx.x) == g_attn_trace_cta;  // read once, not per mark
#endif

  // Work unit (bh, qb).  Non-causal: every unit costs the same; the query
  // blocks of a head are adjacent so its K/V stay hot in L2.  Causal: unit
  // cost grows with qb, so all heads' longest query blocks go first (longest
  // processing time first keeps the last wave short).
  int bh, qb;
  if (kCausal) {
    // Groups of head_group heads in sequence; inside a group, all query
    // blocks of its heads in longest-first order.
    const int per_group = p.head_group * p.num_qblocks;
    const int g = unit / per_group;
    const int r = unit - g * per_group;
    const int heads = min(p.head_group, p.BH - g * p.head_group);
    qb = p.num_qblocks - 1 - r / heads;
    bh = g * p.head_group + r % heads;
  } else {
    bh = unit / p.num_qblocks;
    qb = p.num_qblocks - 1 - unit % p.num_qblocks;
  }
  const int hh = bh % p.H, bb = bh / p.H;  // TMA coordinates of the (batch, head) slice
  const int q0 = qb * C::kRows;
  const int n0 = tile_key_blocks(q0, 0, p.Lq, p.Lk, kCausal, C::kBN);
  const int n1 = kTiles > 1 ? tile_key_blocks(q0, 1, p.Lq, p.Lk, kCausal, C::kBN) : 0;
  const int nkb = max(n0, n1);

  if (threadIdx.x == 0) {
    ctl.abort_flag = 0;
    mbar_init(&ctl.q_full[0], 1);
    mbar_init(&ctl.q_full[1], 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&ctl.k_full[s], 1);
      mbar_init(&ctl.k_empty[s], 1);
      mbar_init(&ctl.v_full[s], 1);
      mbar_init(&ctl.v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&ctl.s_full[t], 1);
      mbar_init(&ctl.s_free[t], 128);
      mbar_init(&ctl.p_free[t], 1);
      mbar_init(&ctl.p_full[t][0], 128);
      mbar_init(&ctl.p_full[t][1], 128);
      mbar_init(&ctl.o_full[t], 1);
    }
    mbar_init(&ctl.mma_done, 1);
    fence_mbar_init();
    // Start the first copies before the CTA synchronises and allocates
    // tensor memory, in the order the first products need them (Q tile 0
    // and K block 0 for S0(0), then Q tile 1, then V block 0); the producer
    // warp issues every later block.
    const uint64_t pol_stream = l2_policy_evict_first();
    const uint64_t pol_keep = l2_policy_evict_last();
    auto load_q = [&](int t) {
      mbar_arrive_expect_tx(&ctl.q_full[t], C::kTileBytes);
      for (int cb = 0; cb < kD / 64; ++cb)
        tma_load_4d(smem_addr(sQ + t * C::kTileBytes + cb * C::kBlockBytes), map_q, &ctl.q_full[t], cb * 64,
                    q0 + t * 128, hh, bb, pol_stream);
    };
    load_q(0);
    mbar_arrive_expect_tx(&ctl.k_full[0], C::kKVBytes);
    for (int cb = 0; cb < kD / 64; ++cb)
      tma_load_4d(smem_addr(sK + cb * C::kKVBlockBytes), map_k, &ctl.k_full[0], cb * 64, 0, hh, bb, pol_keep);
    if (n1 > 0) load_q(1);
    mbar_arrive_expect_tx(&ctl.v_full[0], C::kKVBytes);
    for (int cb = 0; cb < kD / 64; ++cb)
      tma_load_4d(smem_addr(sV + cb * C::kKVBlockBytes), map_v, &ctl.v_full[0], cb * 64, 0, hh, bb, pol_keep);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(smem_addr(&ctl.tmem_base), C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == C::kTmaWarp && lane == 0) {
    tma_prefetch_desc(map_q);
    tma_prefetch_desc(map_k);
    tma_prefetch_desc(map_v);
    tma_prefetch_desc(map_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  RA_MARK(8190 - warp);
  // The last block loaded into each K / V stage (TMA warp; block 0 was issued
  // during setup), for the drain of an aborted CTA.
  int last_k[3] = {0, -1, -1}, last_v[3] = {0, -1, -1};
  if (warp == C::kTmaWarp) {
    // ------------------------------------------------------------------ TMA
    const uint64_t pol_keep = l2_policy_evict_last();
    const bool leader = elect_one();
    bool ok = true;
    for (int j = 1; j < nkb && ok; ++j) {
      const int sk = j % C::kStagesK;
      RA_MARK(6144 + j * 4 + 0);
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&ctl.k_empty[sk], ((j / C::kStagesK) & 1) ^ 1, abort_flag, status, kWatchK + 1, wait_ns));
      if (!ok) break;
      if (leader) {
        mbar_arrive_expect_tx(&ctl.k_full[sk], C::kKVBytes);
        for (int cb = 0; cb < kD / 64; ++cb)
          tma_load_4d(smem_addr(sK + sk * C::kKVBytes + cb * C::kKVBlockBytes), map_k, &ctl.k_full[sk], cb * 64,
                      j * C::kBN, hh, bb, pol_keep);
      }
      last_k[sk] = j;
      RA_MARK(6144 + j * 4 + 1);
      const int sv = j % C::kStagesV;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&ctl.v_empty[sv], ((j / C::kStagesV) & 1) ^ 1, abort_flag, status, kWatchV + 1, wait_ns));
      if (!ok) break;
      if (leader) {
        mbar_arrive_expect_tx(&ctl.v_full[sv], C::kKVBytes);
        for (int cb = 0; cb < kD / 64; ++cb)
          tma_load_4d(smem_addr(sV + sv * C::kKVBytes + cb * C::kKVBlockBytes), map_v, &ctl.v_full[sv], cb * 64,
                      j * C::kBN, hh, bb, pol_keep);
      }
      last_v[sv] = j;
      RA_MARK(6144 + j * 4 + 2);
    }
  } else if (warp == C::kMmaWarp) {
    // ------------------------------------------------------------------ UMMA
    const uint32_t idesc_s = umma_idesc_f16(kBf16, 128, C::kBN, false);
    const uint32_t idesc_o = umma_idesc_f16(kBf16, 128, kD, true);
    const bool leader = elect_one();
    const uint32_t tS0 = tmem + 0, tS1 = tmem + C::kBN;
    const uint32_t tO0 = tmem + C::kColO, tO1 = tmem + C::kColO + kD;
    const uint32_t q_addr0 = smem_addr(sQ), q_addr1 = smem_addr(sQ + C::kTileBytes);

    // S = Q K^T over D in steps of 16 (K-major operands, 128-byte swizzle).
    // Each step's descriptors are the operand's base descriptor with the
    // step's offset added to the address field (sw128_desc_step).
    auto issue_s = [&](uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr) {
      const uint64_t qd = sw128_desc(q_addr, 16, 1024), kd = sw128_desc(k_addr, 16, 1024);
#pragma unroll
      for (int k = 0; k < kD / 16; ++k) {
        const uint32_t q_off = (k / 4) * C::kBlockBytes + (k % 4) * 32;
        const uint32_t k_off = (k / 4) * C::kKVBlockBytes + (k % 4) * 32;
        umma_ss(d_tmem, sw128_desc_step(qd, q_off), sw128_desc_step(kd, k_off), idesc_s, k > 0 ? 1u : 0u);
      }
    };
    // O (+)= P V over 128 keys in steps of 16 (P from TMEM, V MN-major).  The
    // two 64-key halves wait for their own half of P, so the first half of
    // the product overlaps the softmax of the second half.
    auto issue_pv = [&](int t, uint32_t v_addr, bool acc, uint32_t parity, int code) -> bool {
      const uint32_t d_tmem = t == 0 ? tO0 : tO1;
      const uint32_t p_tmem = C::kSepP ? tmem + C::kColP + t * 64 : (t == 0 ? tS0 : tS1);
      const uint64_t vd = sw128_desc(v_addr, C::kKVBlockBytes, 1024);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!__all_sync(0xffffffffu, mbar_wait(&ctl.p_full[t][h], parity, abort_flag, status, code + h, wait_ns)))
          return false;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int k = h * (C::kBN / 32); k < (h + 1) * (C::kBN / 32); ++k)
            umma_ts(d_tmem, p_tmem + k * 8, sw128_desc_step(vd, k * 2048), idesc_o, (acc || k > 0) ? 1u : 0u);
        }
        __syncwarp();
      }
      return true;
    };

    bool ok = __all_sync(0xffffffffu, mbar_wait(&ctl.q_full[0], 0, abort_flag, status, kWatchQ + 2, wait_ns));
    if constexpr (C::kSepP) {
      // Issue order: S0(0) S1(0) | per block j: S0(j+1) O0+=P0(j)V(j) S1(j+1) O1+=P1(j)V(j).
      // S(j+1) only waits for the softmax to have read S(j) (s_free), so the
      // scores of the next block are ready when the softmax finishes.
      const int nt[2] = {n0, n1};
      if (ok && n1 > 0) ok = __all_sync(0xffffffffu, mbar_wait(&ctl.q_full[1], 0, abort_flag, status, kWatchQ + 3, wait_ns));
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(&ctl.k_full[0], 0, abort_flag, status, kWatchK + 2, wait_ns));
        if (ok) {
          tc_fence_after();
          if (leader) {
            if (n0 > 0) { issue_s(tS0, q_addr0, smem_addr(sK)); umma_commit(&ctl.s_full[0]); }
            if (n1 > 0) { issue_s(tS1, q_addr1, smem_addr(sK)); umma_commit(&ctl.s_full[1]); }
            umma_commit(&ctl.k_empty[0]);
          }
          __syncwarp();
        }
      }
      for (int j = 0; j < nkb && ok; ++j) {
        RA_MARK(4096 + j * 8 + 0);
        const int sk1 = (j + 1) % C::kStagesK, sv = j % C::kStagesV;
        if (j + 1 < nkb) {
          ok = __all_sync(0xffffffffu, mbar_wait(&ctl.k_full[sk1], ((j + 1) / C::kStagesK) & 1, abort_flag,
                                                 status, kWatchK + 3));
          if (!ok) break;
        }
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&ctl.v_full[sv], (j / C::kStagesV) & 1, abort_flag, status, kWatchV + 2, wait_ns));
        if (!ok) break;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j + 1 < nt[t]) {
            ok = __all_sync(0xffffffffu, mbar_wait(&ctl.s_free[t], j & 1, abort_flag, status, kWatchS + 5 + t, wait_ns));
            if (!ok) break;
            tc_fence_after();
            if (leader) {
              issue_s(t == 0 ? tS0 : tS1, t == 0 ? q_addr0 : q_addr1, smem_addr(sK + sk1 * C::kKVBytes));
              umma_commit(&ctl.s_full[t]);
            }
            __syncwarp();
          }
          if (j < nt[t]) {
            ok = issue_pv(t, smem_addr(sV + sv * C::kKVBytes), j > 0, j & 1, kWatchP + 2 * t);
            if (!ok) break;
            if (leader) {
              umma_commit(&ctl.p_free[t]);
              if (j == nt[t] - 1) umma_commit(&ctl.o_full[t]);
            }
            __syncwarp();
          }
        }
        if (!ok) break;
        if (leader) {
          if (j + 1 < nkb) umma_commit(&ctl.k_empty[sk1]);
          umma_commit(&ctl.v_empty[sv]);
        }
        __syncwarp();
        RA_MARK(4096 + j * 8 + 1);
      }
    } else {
    // Issue order per key block j: S0(j), O1 += P1(j-1) V(j-1), S1(j), O0 += P0(j) V(j).
    for (int j = 0; j < nkb && ok; ++j) {
      const int sk = j % C::kStagesK, sv = j % C::kStagesV;
      const uint32_t k_addr = smem_addr(sK + sk * C::kKVBytes);
      RA_MARK(4096 + j * 8 + 0);
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&ctl.k_full[sk], (j / C::kStagesK) & 1, abort_flag, status, kWatchK + 2, wait_ns));
      if (!ok) break;
      tc_fence_after();
      if (leader && j < n0) {
        issue_s(tS0, q_addr0, k_addr);
        umma_commit(&ctl.s_full[0]);
      }
      __syncwarp();
      RA_MARK(4096 + j * 8 + 1);
      if (j >= 1 && j - 1 < n1) {
        const int pv = (j - 1) % C::kStagesV;
        ok = issue_pv(1, smem_addr(sV + pv * C::kKVBytes), j - 1 > 0, (j - 1) & 1, kWatchP + 2);
        if (!ok) break;
        if (leader) umma_commit(&ctl.v_empty[pv]);
        __syncwarp();
      }
      RA_MARK(4096 + j * 8 + 2);
      if (j == 0 && n1 > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&ctl.q_full[1], 0, abort_flag, status, kWatchQ + 3, wait_ns));
        if (!ok) break;
        tc_fence_after();
      }
      if (leader) {
        if (j < n1) {
          issue_s(tS1, q_addr1, k_addr);
          umma_commit(&ctl.s_full[1]);
        }
        umma_commit(&ctl.k_empty[sk]);
      }
      __syncwarp();
      RA_MARK(4096 + j * 8 + 3);
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&ctl.v_full[sv], (j / C::kStagesV) & 1, abort_flag, status, kWatchV + 2, wait_ns));
      if (!ok) break;
      if (j < n0) {
        ok = issue_pv(0, smem_addr(sV + sv * C::kKVBytes), j > 0, j & 1, kWatchP + 0);
        if (!ok) break;
        if (leader && j == n0 - 1) umma_commit(&ctl.o_full[0]);
        __syncwarp();
      }
      RA_MARK(4096 + j * 8 + 4);
      if (leader && j >= n1) umma_commit(&ctl.v_empty[sv]);
      __syncwarp();
    }
    if (ok && n1 > 0 && n1 == nkb) {
      const int pv = (nkb - 1) % C::kStagesV;
      ok = issue_pv(1, smem_addr(sV + pv * C::kKVBytes), nkb - 1 > 0, (nkb - 1) & 1, kWatchP + 4);
      if (ok && leader) {
        umma_commit(&ctl.v_empty[pv]);
        umma_commit(&ctl.o_full[1]);
      }
      __syncwarp();
    }
    }
    // Every UMMA this warp issued has retired before TMEM is released.
    if (leader) umma_commit(&ctl.mma_done);
    __syncwarp();
    volatile int no_abort = 0;
    mbar_wait(&ctl.mma_done, 0, &no_abort, status, kWatchDrain + 1);
  } else {
    // --------------------------------------------------------------- softmax
    const int t = warp >> 2;                       // Q tile of this warpgroup
    const int row_in_tile = (warp & 3) * 32 + lane; // == TMEM lane
    const int row_abs = q0 + t * 128 + row_in_tile;
    const int n_t = t == 0 ? n0 : n1;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * C::kBN;
    const uint32_t tP = C::kSepP ? tmem + lane_off + C::kColP + t * 64 : tS;
    const uint32_t tO = tmem + lane_off + C::kColO + t * kD;
    const float c = p.scale_log2;
    const uint64_t c2 = f2(c, c);
    float m = -INFINITY;  // running max of raw scores (exp2 reference point)
    float l = 0.f;        // running sum of probabilities relative to m
    bool ok = true;

    constexpr int kBN = C::kBN;
    // Stores half h of the block's P (keys [h*kBN/2, (h+1)*kBN/2), packed
    // 16-bit pairs in P columns [h*kBN/4, (h+1)*kBN/4)) and signals it.
    // With 128-key blocks pk holds the half; with 64-key blocks pk holds both
    // halves, half h in pk[16h, 16h+16).
    auto store_half = [&](int h, const uint32_t (&pk)[32]) {
      if constexpr (kBN == 128) {
        tmem_st32(tP + 32 * h, pk);
      } else {
        uint32_t q[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) q[i] = pk[16 * h + i];
        tmem_st16(tP + 16 * h, q);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&ctl.p_full[t][h]);
    };
#ifdef RA_WATCHDOG_TEST
    // Watchdog test build: when the launch asks for it, CTA 0's tile 0 loses
    // its first P arrival (half 0 of block 0).  Nothing else ever completes
    // that phase, so the MMA warp's wait for it can only end by the watchdog.
    const bool drop_first = p.drop_arrival != 0 && blockIdx.x == 0 && t == 0;
#endif

    // Loads the block's kBN fp32 scores of this thread's row and masks keys
    // past Lk and, when causal, keys after the query.
    auto load_scores = [&](int j, float (&s)[kBN]) {
      uint32_t u[kBN / 32][32];
#pragma unroll
      for (int cb = 0; cb < kBN / 32; ++cb) tmem_ld32(tS + 32 * cb, u[cb]);
      tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < kBN / 32; ++cb)
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 * cb + i] = __uint_as_float(u[cb][i]);
      const int kbase = j * kBN;
      if ((kbase + kBN > p.Lk) || (kCausal && kbase + kBN - 1 > q0 + t * 128)) {
        int limit = p.Lk - 1 - kbase;
        if (kCausal) limit = min(limit, row_abs - kbase);
#pragma unroll
        for (int i = 0; i < kBN; ++i)
          if (i > limit) s[i] = -INFINITY;
      }
    };
    // Exponentials of the first half of the block's keys against the
    // reference -nmc2/c2 (pk half 0 and its sums).
    auto exp_half0 = [&](const float (&s)[kBN], uint64_t nmc2, uint32_t (&pk)[32], uint64_t& sum0,
                         uint64_t& sum1) {
      if constexpr (kBN == 128) {
        exp_pack32<kBf16, 0, 0>(s, c2, nmc2, pk, sum0);
        exp_pack32<kBf16, 32, 16>(s, c2, nmc2, pk, sum1);
      } else {
        exp_pack32<kBf16, 0, 0>(s, c2, nmc2, pk, sum0);
      }
    };

    for (int j = 0; j < n_t; ++j) {
      RA_MARK(t * 2048 + j * 16 + 0);
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl.s_full[t], j & 1, abort_flag, status, kWatchS + 1 + t, wait_ns));
      if (!ok) break;
      tc_fence_after();
      RA_MARK(t * 2048 + j * 16 + 1);
      float s[kBN];
      load_scores(j, s);
      RA_MARK(t * 2048 + j * 16 + 2);
      // Row max of the block: four independent chains of 3-input max.
      float mx[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int i = 4; i < kBN - 4; i += 8) {
        mx[0] = fmax3(mx[0], s[i + 0], s[i + 4]);
        mx[1] = fmax3(mx[1], s[i + 1], s[i + 5]);
        mx[2] = fmax3(mx[2], s[i + 2], s[i + 6]);
        mx[3] = fmax3(mx[3], s[i + 3], s[i + 7]);
      }
      const float mb = fmax3(fmax3(mx[0], mx[1], s[kBN - 4]), fmax3(mx[2], mx[3], s[kBN - 3]),
                             fmaxf(s[kBN - 2], s[kBN - 1]));

      // Exponentials of the first half against the running max, computed
      // while the block max is still being reduced: after the first blocks
      // the max almost never moves by more than 2^8, and then these values
      // are final.  The first block takes its own max as the running max
      // (l and O are still zero), so it needs no second pass.
      if (j == 0) m = mb;
      uint64_t sum0 = f2(0.f, 0.f), sum1 = f2(0.f, 0.f);
      uint32_t pk[32];
      {
        const float mc = (m == -INFINITY) ? 0.f : m * c;
        exp_half0(s, f2(-mc, -mc), pk, sum0, sum1);
      }
      RA_MARK(t * 2048 + j * 16 + 3);
      const bool grow = (fmaxf(m, mb) - m) * c > 8.0f;
      if (__any_sync(0xffffffffu, grow)) {
        // The running max moves for some row of this warp (always on the first
        // block).  Rows that grow take the block max; O and l are rescaled
        // (S(j) retired, so every P*V product up to block j-1 has too) and
        // the first half is recomputed from the scores, still intact in TMEM.
        float alpha = 1.f;
        if (grow) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - mb) * c);
          l *= alpha;
          m = mb;
        }
        if (C::kSepP && j > 0) {
          // Separate-P layout: S(j) may retire before the product of block
          // j-1, so wait for that product before touching O.
          ok = __all_sync(0xffffffffu, mbar_wait(&ctl.p_free[t], (j - 1) & 1, abort_flag, status, kWatchO + 5 + t, wait_ns));
          if (!ok) break;
          tc_fence_after();
        }
        if (j > 0) {
#pragma unroll 1
          for (int cc = 0; cc < kD; cc += 32) {
            uint32_t o[32];
            tmem_ld32(tO + cc, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + cc, o);
          }
        }
        load_scores(j, s);
        const float mc = m * c;
        sum0 = f2(0.f, 0.f);
        sum1 = f2(0.f, 0.f);
        exp_half0(s, f2(-mc, -mc), pk, sum0, sum1);
      }
      RA_MARK(t * 2048 + j * 16 + 4);
      if constexpr (C::kSepP) {
        // Every score of this block is in registers now (the first half
        // already as packed P): let the next block's S*K^T overwrite S, and
        // store P only once the previous block's product has read it.
        tc_fence_before();
        mbar_arrive(&ctl.s_free[t]);
        if (j > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(&ctl.p_free[t], (j - 1) & 1, abort_flag, status, kWatchO + 5 + t, wait_ns));
          if (!ok) break;
          tc_fence_after();
        }
      }
#ifdef RA_WATCHDOG_TEST
      if (!(drop_first && j == 0))  // lost: neither stored nor signalled
#endif
      store_half(0, pk);
      RA_MARK(t * 2048 + j * 16 + 5);
      {
        const float mc = m * c;
        const uint64_t nmc2 = f2(-mc, -mc);
        if constexpr (kBN == 128) {
          exp_pack32<kBf16, 64, 0>(s, c2, nmc2, pk, sum0);
          exp_pack32<kBf16, 96, 16>(s, c2, nmc2, pk, sum1);
        } else {
          exp_pack32<kBf16, 32, 16>(s, c2, nmc2, pk, sum1);
        }
      }
      RA_MARK(t * 2048 + j * 16 + 6);
      store_half(1, pk);
      RA_MARK(t * 2048 + j * 16 + 7);
      {
        float a0, a1, b0, b1;
        f2_split(sum0, a0, a1);
        f2_split(sum1, b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
    }

    // ------------------------------------------------------------- epilogue
    bool store = ok && n_t > 0;
    if (store) {
      store = __all_sync(0xffffffffu, mbar_wait(&ctl.o_full[t], 0, abort_flag, status, kWatchO + 1 + t, wait_ns));
    }
    uint8_t* stage = sQ + t * C::kTileBytes;  // Q tile t is dead once O_t is final
    // How the staged tile reaches O.  One-tile CTAs with 128-key blocks (two
    // per SM) copy it with their own warpgroup in coalesced 16-byte stores,
    // so nothing remains in flight when the CTA exits (measured 2 % faster at
    // D=64).  The others hand it to the TMA engine, which stores it while the
    // SM keeps working: a copy by the warps measured 1-3 % slower for both
    // tiles of two-tile CTAs and with several 64-key-block CTAs per SM.
    constexpr bool kCoopCopy = kTiles == 1 && kBN == 128;
    if (store) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      // The whole O row at once (one wait for all loads; the scores are dead).
      uint32_t o[kD / 32][32];
#pragma unroll
      for (int cq = 0; cq < kD / 32; ++cq) tmem_ld32(tO + 32 * cq, o[cq]);
      tmem_wait_ld();
#pragma unroll
      for (int cq = 0; cq < kD / 32; ++cq) {
        const int cb = cq / 2;
        const int chunk0 = (cq % 2) * 4;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint32_t* w = &o[cq][8 * q4];
          uint4 v;
          v.x = pack2<kBf16>(__uint_as_float(w[0]) * inv_l, __uint_as_float(w[1]) * inv_l);
          v.y = pack2<kBf16>(__uint_as_float(w[2]) * inv_l, __uint_as_float(w[3]) * inv_l);
          v.z = pack2<kBf16>(__uint_as_float(w[4]) * inv_l, __uint_as_float(w[5]) * inv_l);
          v.w = pack2<kBf16>(__uint_as_float(w[6]) * inv_l, __uint_as_float(w[7]) * inv_l);
          const int chunk = chunk0 + q4;
          const uint32_t off = cb * C::kBlockBytes + row_in_tile * 128 + ((chunk ^ (row_in_tile & 7)) << 4);
          *reinterpret_cast<uint4*>(stage + off) = v;
        }
      }
      if constexpr (!kCoopCopy) fence_proxy_async_smem();
    }
    // All four warps of the group pass this barrier exactly once.
    named_barrier_sync(1 + t, 128);
    if (store && !kCoopCopy && (threadIdx.x & 127) == 0) {
      for (int cb = 0; cb < kD / 64; ++cb)
        tma_store_4d(map_o, smem_addr(stage + cb * C::kBlockBytes), cb * 64, q0 + t * 128, hh, bb);
      tma_store_commit();
      tma_store_wait_smem_read();
    }
    if (store && kCoopCopy) {
      // The group copies the staged tile to O (contiguous [B, H, Lq, D]) in
      // 16-byte chunks taken in row-major order, so each warp instruction
      // writes whole rows, 512 contiguous bytes; rows past Lq are skipped.
      // Nothing is left in flight that the CTA must wait for before it exits.
      constexpr int kChunks = kD / 8;  // 16-byte chunks per row
      const int tid = threadIdx.x & 127;
      const int rows = min(128, p.Lq - (q0 + t * 128));
      uint8_t* const orow0 =
          static_cast<uint8_t*>(p.out) + (static_cast<long long>(bh) * p.Lq + q0 + t * 128) * (kD * 2);
      const uint64_t pol = l2_policy_evict_first();
#pragma unroll
      for (int k = 0; k < kChunks; ++k) {
        const int lin = k * 128 + tid;
        const int r = lin / kChunks, c = lin % kChunks;
        if (r < rows) {
          const uint32_t off = (c / 8) * C::kBlockBytes + r * 128 + (((c % 8) ^ (r & 7)) << 4);
          st_global_v4_hint(orow0 + static_cast<long long>(r) * (kD * 2) + c * 16,
                            *reinterpret_cast<const uint4*>(stage + off), pol);
        }
      }
    }
  }

  RA_MARK(8180 - warp);
  tc_fence_before();
  __syncthreads();
  if (warp == C::kTmaWarp && *abort_flag) {
    // Some role gave up on a wait (every role has finished by now, so the flag
    // is final): let every copy already issued land before the CTA exits,
    // also when this warp itself had issued all its blocks.  Without an abort
    // every issued block was consumed, so there is nothing to wait for.
    volatile int no_abort = 0;
    mbar_wait(&ctl.q_full[0], 0, &no_abort, status, kWatchDrain);
    if (n1 > 0) mbar_wait(&ctl.q_full[1], 0, &no_abort, status, kWatchDrain);
    for (int s = 0; s < 3; ++s) {
      if (last_k[s] >= 0) mbar_wait(&ctl.k_full[s], (last_k[s] / C::kStagesK) & 1, &no_abort, status, kWatchDrain);
      if (last_v[s] >= 0) mbar_wait(&ctl.v_full[s], (last_v[s] / C::kStagesV) & 1, &no_abort, status, kWatchDrain);
    }
  }
  if (warp == C::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------

// Element strides of one input over (batch, head, row); the head dim is
// contiguous.
struct Strides {
  long long b, h, l;
};


// Returned by launch_impl when a buffer or stride cannot be described to TMA
// (the caller then runs the general kernel).
constexpr int kNoTensorMap = -2;

// Causal scheduling groups hold about this many bytes of K+V (three
// quarters of L2): with fewer, the last group's longest units start late and
// leave a tail when a launch has only 8-32 heads (measured 6-14 % slower).
#ifndef RA_HEAD_GROUP_BYTES
#define RA_HEAD_GROUP_BYTES 96.0e6
#endif

// One problem of a launch: buffers, sizes, element strides, softmax scale.
struct FwdProblem {
  const void *q, *k, *v;
  void* out;
  int B, H, Sq, Skv;
  Strides sq, sk, sv;
  float scale;
};

// Pipeline wait limit for launches from now on (attn_set_wait_limit_ns);
// 0 selects kWaitTimeoutNs.  Defined in attn_kernel.cu.
unsigned long long wait_limit_ns();
// Watchdog test builds: whether launches drop one arrival (attn_kernel.cu).
int drop_arrival_requested();

// Work units (CTAs) of one problem.
template <int kD, int kTiles, int kBlockKeys>
inline long long problem_units(const FwdProblem& d) {
  using C = Cfg<kD, kTiles, kBlockKeys>;
  return static_cast<long long>((d.Sq + C::kRows - 1) / C::kRows) * d.B * d.H;
}

// Encodes problem d's tensor maps and parameters into slot i of `a`.
// Returns 0, kNoTensorMap (a buffer or stride TMA cannot describe: the caller
// runs the general kernel instead) or ATTN_ERR_TENSOR_MAP.
template <bool kBf16, int kD, int kTiles, int kBlockKeys, int kMaxProblems>
int encode_problem(const FwdProblem& d, FwdArgs<kMaxProblems>& a, int i) {
  using C = Cfg<kD, kTiles, kBlockKeys>;
  const uint64_t D = kD;
  CUtensorMap* m = a.map[i];
  const int r[4] = {
      make_tensor_map_4d(&m[0], d.q, kBf16, D, d.Sq, d.H, d.B, d.sq.l, d.sq.h, d.sq.b, 64, 128),
      make_tensor_map_4d(&m[1], d.k, kBf16, D, d.Skv, d.H, d.B, d.sk.l, d.sk.h, d.sk.b, 64, C::kBN),
      make_tensor_map_4d(&m[2], d.v, kBf16, D, d.Skv, d.H, d.B, d.sv.l, d.sv.h, d.sv.b, 64, C::kBN),
      make_tensor_map_4d(&m[3], d.out, kBf16, D, d.Sq, d.H, d.B, D, static_cast<uint64_t>(d.Sq) * D,
                         static_cast<uint64_t>(d.H) * d.Sq * D, 64, 128)};
  for (int e : r)
    if (e == kNoTensorMap) return kNoTensorMap;
  for (int e : r)
    if (e != 0) return ATTN_ERR_TENSOR_MAP;
  AttnParams& prm = a.prm[i];
  prm.Lq = d.Sq;
  prm.Lk = d.Skv;
  const int BH = d.B * d.H;
  prm.BH = BH;
  prm.H = d.H;
  prm.num_qblocks = (d.Sq + C::kRows - 1) / C::kRows;
  // K+V bytes of one head; about RA_HEAD_GROUP_BYTES of them per group.
  const double kv_bytes = 2.0 * d.Skv * kD * 2;
  prm.head_group = static_cast<int>(fmax(1.0, fmin(static_cast<double>(BH), RA_HEAD_GROUP_BYTES / kv_bytes)));
  prm.scale_log2 = d.scale * 1.4426950408889634f;
  prm.out = d.out;
  const unsigned long long limit = wait_limit_ns();
  prm.wait_ns = limit != 0 ? limit : kWaitTimeoutNs;
  prm.drop_arrival = drop_arrival_requested();
  return 0;
}

// Instantiation of the tensor-core kernel a problem runs on.
struct TcKey {
  bool bf16;
  int D;
  bool causal;
  int keys;  // keys per K/V block
  bool operator==(const TcKey& o) const { return bf16 == o.bf16 && D == o.D && causal == o.causal && keys == o.keys; }
};

// One problem, one grid (attn_kernel.cu).  Returns an AttnStatus, or
// kNoTensorMap when the buffers cannot be described to TMA.
int launch_tc_single(const TcKey& key, const FwdProblem& d, cudaStream_t stream);

// The n problems, all on instantiation `key`, as few grids as the argument
// block allows, longest units first (attn_group.cu).  Problems whose buffers
// TMA cannot describe are not launched; their indices go to *fallback.
int launch_tc_grouped(const TcKey& key, const FwdProblem* d, int n, cudaStream_t stream, std::vector<int>* fallback);

// Queue a read of one translation unit's watchdog status word into *host and
// its reset on `stream` (attn_kernel.cu and attn_group.cu each hold one).
int status_word_read_clear_single(cudaStream_t stream, int* host);
int status_word_read_clear_grouped(cudaStream_t stream, int* host);

// Launches the problems in `a` (a.n of them, unit_end filled in) as one grid.
template <bool kBf16, int kD, bool kCausal, int kTiles, int kBlockKeys, int kMaxProblems>
int launch_fwd(const FwdArgs<kMaxProblems>& a, cudaStream_t stream) {
  using C = Cfg<kD, kTiles, kBlockKeys>;
  auto kern = attn_fwd_kernel<kBf16, kD, kCausal, kTiles, kBlockKeys, kMaxProblems>;
  // Opt in to the large dynamic shared-memory carve-out once per device
  // (under the mutex: launches may come from several host threads).
  static bool configured[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ATTN_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> g(mu);
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(C::kSmemBytes)) != cudaSuccess)
        return ATTN_ERR_LAUNCH;
      // One-tile CTAs: ask for the largest shared-memory carve-out so two
      // of them fit on an SM.
      if (kTiles == 1 && cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                              static_cast<int>(cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
        return ATTN_ERR_LAUNCH;
      configured[dev] = true;
    }
  }
  const long long grid = a.unit_end[a.n - 1];
  if (grid <= 0) return ATTN_OK;
  if (grid > 0x7fffffffLL) return ATTN_ERR_INVALID_ARGUMENT;
  kern<<<static_cast<unsigned>(grid), C::kThreads, C::kSmemBytes, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? ATTN_OK : ATTN_ERR_LAUNCH;
}

}  // namespace ra
