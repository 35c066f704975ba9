// Fused attention forward for NVIDIA B200 (sm_100a): TMA -> shared memory ->
// tcgen05 UMMA with accumulators in tensor memory, online softmax in base 2.
//
// Replaces the reference's three HIP kernels and their launcher
// (src/attn_kernel_torch.cu:36-689, src/attn_kernel.hip.cpp:36-367 of
// JoursBleu/rocm_attn).  The math is the reference's: per query row,
// s_j = (q . k_j) * scale, masked when causal and j > i
// (src/attn_kernel_torch.cu:54,238,263), softmax in the exp2 domain with a
// running fp32 max and sum (src/attn_kernel_torch.cu:269-298), O = P V / sum
// (src/attn_kernel_torch.cu:333-354).
//
// CTA work unit: 256 query rows of one (batch, head) as two 128-row Q tiles.
// Warp roles (320 threads):
//   warps 0-3  softmax of Q tile 0 (thread <-> TMEM lane <-> query row)
//   warps 4-7  softmax of Q tile 1
//   warp  8    UMMA issue (one elected lane) and TMEM allocation
//   warp  9    TMA producer (Q once, then K/V blocks of 128 keys)
// Tensor memory (512 columns x 128 lanes x 32 bit):
//   S0 [0,128)  S1 [128,256)   fp32 scores of the current key block
//   P0 = S0 cols [0,64), P1 = S1 cols [0,64)   16-bit probabilities (aliases S)
//   O0 [256,256+D)  O1 [256+D,256+2D)          fp32 output accumulators
// UMMA issue order per key block j (tcgen05.mma executes in issue order):
//   S0(j)=Q0 K_j^T, O1+=P1(j-1) V_{j-1}, S1(j)=Q1 K_j^T, O0+=P0(j) V_j
// so each softmax warpgroup works while the tensor core runs the other tile.
// The running max is only moved (and O rescaled) when it grows by more than
// 2^8 in the exp2 domain; P values stay <= 256, exact in fp16/bf16 range, and
// the final division by the matching running sum makes the result identical
// in exact arithmetic.

#include "sm100_ptx.cuh"
#include "tensor_map.h"
#include "attn_kernel.h"

#include <math.h>
#include <mutex>

namespace ra {

// Sticky per-device status word written by the kernel's watchdog.
__device__ int g_attn_status = 0;

enum : int { kWatchQ = 0x10, kWatchK = 0x20, kWatchV = 0x30, kWatchS = 0x40, kWatchP = 0x50, kWatchO = 0x60,
             kWatchDrain = 0x70 };

struct AttnParams {
  int Lq;           // query rows per (batch, head)
  int Lk;           // key rows per (batch, head)
  int BH;           // batch * heads
  int num_qblocks;  // ceil(Lq / 256)
  float scale_log2; // softmax scale * log2(e)
};

template <int kD>
struct Cfg {
  static constexpr int kBM = 128;                       // rows per Q tile
  static constexpr int kBN = 128;                       // keys per block
  static constexpr int kStagesK = kD == 128 ? 2 : 3;    // K ring depth
  static constexpr int kStagesV = kD == 128 ? 2 : 3;    // V ring depth
  static constexpr uint32_t kTileBytes = 128u * kD * 2; // one 128 x D tile
  static constexpr uint32_t kSmemBytes = 1024 + 2 * kTileBytes + (kStagesK + kStagesV) * kTileBytes;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColO = 256;
  static constexpr int kThreads = 320;
};

struct __align__(8) SharedCtl {
  uint64_t q_full;
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[3], v_empty[3];
  uint64_t s_full[2], p_full[2], o_full[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

// Number of 128-key blocks Q tile `t` of the CTA starting at row q0 needs.
__device__ __forceinline__ int tile_key_blocks(int q0, int t, int Lq, int Lk, bool causal) {
  const int first = q0 + t * 128;
  if (first >= Lq) return 0;
  const int all = (Lk + 127) / 128;
  if (!causal) return all;
  const int last = min(first + 127, Lq - 1);
  return min(all, last / 128 + 1);
}

template <bool kBf16, int kD, bool kCausal>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                    const AttnParams p) {
  using C = Cfg<kD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                    // 2 tiles
  uint8_t* sK = smem + 2 * C::kTileBytes;                // kStagesK tiles
  uint8_t* sV = sK + C::kStagesK * C::kTileBytes;        // kStagesV tiles
  volatile int* abort_flag = &ctl.abort_flag;
  int* status = &g_attn_status;

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x) / 32, 0);
  const int lane = threadIdx.x & 31;

  // Work unit: heads in order, the longest (last) query blocks of a head first.
  const int bh = blockIdx.x / p.num_qblocks;
  const int qb = p.num_qblocks - 1 - static_cast<int>(blockIdx.x % p.num_qblocks);
  const int q0 = qb * 256;
  const int n0 = tile_key_blocks(q0, 0, p.Lq, p.Lk, kCausal);
  const int n1 = tile_key_blocks(q0, 1, p.Lq, p.Lk, kCausal);
  const int nkb = max(n0, n1);

  if (threadIdx.x == 0) {
    ctl.abort_flag = 0;
    mbar_init(&ctl.q_full, 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&ctl.k_full[s], 1);
      mbar_init(&ctl.k_empty[s], 1);
      mbar_init(&ctl.v_full[s], 1);
      mbar_init(&ctl.v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&ctl.s_full[t], 1);
      mbar_init(&ctl.p_full[t], 128);
      mbar_init(&ctl.o_full[t], 1);
    }
    mbar_init(&ctl.mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(smem_addr(&ctl.tmem_base), C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 9 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
    tma_prefetch_desc(&map_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  if (warp == 9) {
    // ------------------------------------------------------------------ TMA
    const uint64_t pol_stream = l2_policy_evict_first();
    const uint64_t pol_keep = l2_policy_evict_last();
    const bool leader = elect_one();
    int last_k[3] = {-1, -1, -1}, last_v[3] = {-1, -1, -1};
    if (leader) {
      mbar_arrive_expect_tx(&ctl.q_full, (n1 > 0 ? 2u : 1u) * C::kTileBytes);
      for (int t = 0; t < (n1 > 0 ? 2 : 1); ++t)
        for (int cb = 0; cb < kD / 64; ++cb)
          tma_load_3d(smem_addr(sQ + t * C::kTileBytes + cb * 16384), &map_q, &ctl.q_full, cb * 64,
                      q0 + t * 128, bh, pol_stream);
    }
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int sk = j % C::kStagesK;
      ok = mbar_wait(&ctl.k_empty[sk], ((j / C::kStagesK) & 1) ^ 1, abort_flag, status, kWatchK + 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (leader) {
        mbar_arrive_expect_tx(&ctl.k_full[sk], C::kTileBytes);
        for (int cb = 0; cb < kD / 64; ++cb)
          tma_load_3d(smem_addr(sK + sk * C::kTileBytes + cb * 16384), &map_k, &ctl.k_full[sk], cb * 64,
                      j * 128, bh, pol_keep);
      }
      last_k[sk] = j;
      const int sv = j % C::kStagesV;
      ok = mbar_wait(&ctl.v_empty[sv], ((j / C::kStagesV) & 1) ^ 1, abort_flag, status, kWatchV + 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (leader) {
        mbar_arrive_expect_tx(&ctl.v_full[sv], C::kTileBytes);
        for (int cb = 0; cb < kD / 64; ++cb)
          tma_load_3d(smem_addr(sV + sv * C::kTileBytes + cb * 16384), &map_v, &ctl.v_full[sv], cb * 64,
                      j * 128, bh, pol_keep);
      }
      last_v[sv] = j;
    }
    if (!ok) {
      // Aborted: let every copy already issued land before the CTA exits.
      volatile int no_abort = 0;
      mbar_wait(&ctl.q_full, 0, &no_abort, status, kWatchDrain);
      for (int s = 0; s < 3; ++s) {
        if (last_k[s] >= 0) mbar_wait(&ctl.k_full[s], (last_k[s] / C::kStagesK) & 1, &no_abort, status, kWatchDrain);
        if (last_v[s] >= 0) mbar_wait(&ctl.v_full[s], (last_v[s] / C::kStagesV) & 1, &no_abort, status, kWatchDrain);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ UMMA
    const uint32_t idesc_s = umma_idesc_f16(kBf16, 128, 128, false);
    const uint32_t idesc_o = umma_idesc_f16(kBf16, 128, kD, true);
    const bool leader = elect_one();
    const uint32_t tS0 = tmem + 0, tS1 = tmem + 128;
    const uint32_t tO0 = tmem + C::kColO, tO1 = tmem + C::kColO + kD;
    const uint32_t q_addr0 = smem_addr(sQ), q_addr1 = smem_addr(sQ + C::kTileBytes);

    // S = Q K^T over D in steps of 16 (K-major operands, 128-byte swizzle).
    auto issue_s = [&](uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr) {
#pragma unroll
      for (int k = 0; k < kD / 16; ++k) {
        const uint32_t off = (k / 4) * 16384 + (k % 4) * 32;
        umma_ss(d_tmem, sw128_desc(q_addr + off, 16, 1024), sw128_desc(k_addr + off, 16, 1024), idesc_s,
                k > 0 ? 1u : 0u);
      }
    };
    // O (+)= P V over 128 keys in steps of 16 (P from TMEM, V MN-major).
    auto issue_o = [&](uint32_t d_tmem, uint32_t p_tmem, uint32_t v_addr, bool acc) {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        umma_ts(d_tmem, p_tmem + k * 8, sw128_desc(v_addr + k * 2048, 16384, 1024), idesc_o,
                (acc || k > 0) ? 1u : 0u);
    };

    bool ok = mbar_wait(&ctl.q_full, 0, abort_flag, status, kWatchQ + 2);
    ok = __all_sync(0xffffffffu, ok);
    for (int j = 0; j < nkb && ok; ++j) {
      const int sk = j % C::kStagesK, sv = j % C::kStagesV;
      const uint32_t k_addr = smem_addr(sK + sk * C::kTileBytes);
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl.k_full[sk], (j / C::kStagesK) & 1, abort_flag, status, kWatchK + 2));
      if (!ok) break;
      tc_fence_after();
      if (leader && j < n0) {
        issue_s(tS0, q_addr0, k_addr);
        umma_commit(&ctl.s_full[0]);
      }
      __syncwarp();
      if (j >= 1 && j - 1 < n1) {
        ok = __all_sync(0xffffffffu, mbar_wait(&ctl.p_full[1], (j - 1) & 1, abort_flag, status, kWatchP + 2));
        if (!ok) break;
        tc_fence_after();
        const int pv = (j - 1) % C::kStagesV;
        if (leader) {
          issue_o(tO1, tS1, smem_addr(sV + pv * C::kTileBytes), j - 1 > 0);
          umma_commit(&ctl.v_empty[pv]);
        }
        __syncwarp();
      }
      if (leader) {
        if (j < n1) {
          issue_s(tS1, q_addr1, k_addr);
          umma_commit(&ctl.s_full[1]);
        }
        umma_commit(&ctl.k_empty[sk]);
      }
      __syncwarp();
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl.v_full[sv], (j / C::kStagesV) & 1, abort_flag, status, kWatchV + 2));
      if (!ok) break;
      if (j < n0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&ctl.p_full[0], j & 1, abort_flag, status, kWatchP + 1));
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          issue_o(tO0, tS0, smem_addr(sV + sv * C::kTileBytes), j > 0);
          if (j == n0 - 1) umma_commit(&ctl.o_full[0]);
        }
        __syncwarp();
      }
      if (leader && j >= n1) umma_commit(&ctl.v_empty[sv]);
      __syncwarp();
    }
    if (ok && n1 > 0 && n1 == nkb) {
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl.p_full[1], (nkb - 1) & 1, abort_flag, status, kWatchP + 3));
      if (ok) {
        tc_fence_after();
        const int pv = (nkb - 1) % C::kStagesV;
        if (leader) {
          issue_o(tO1, tS1, smem_addr(sV + pv * C::kTileBytes), nkb - 1 > 0);
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
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + C::kColO + t * kD;
    const float c = p.scale_log2;
    float m = -INFINITY;  // running max of raw scores (exp2 reference point)
    float l = 0.f;        // running sum of probabilities relative to m
    bool ok = true;

    for (int j = 0; j < n_t; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl.s_full[t], j & 1, abort_flag, status, kWatchS + 1 + t));
      if (!ok) break;
      tc_fence_after();
      float s[128];
      {
        uint32_t u0[32], u1[32], u2[32], u3[32];
        tmem_ld32(tS + 0, u0);
        tmem_ld32(tS + 32, u1);
        tmem_ld32(tS + 64, u2);
        tmem_ld32(tS + 96, u3);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(u0[i]);
          s[32 + i] = __uint_as_float(u1[i]);
          s[64 + i] = __uint_as_float(u2[i]);
          s[96 + i] = __uint_as_float(u3[i]);
        }
      }
      const int kbase = j * 128;
      const bool need_mask = (kbase + 128 > p.Lk) || (kCausal && kbase + 127 > q0 + t * 128);
      if (need_mask) {
        int limit = p.Lk - 1 - kbase;
        if (kCausal) limit = min(limit, row_abs - kbase);
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > limit) s[i] = -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = s[i];
#pragma unroll
      for (int i = 8; i < 128; ++i) mx[i & 7] = fmaxf(mx[i & 7], s[i]);
      const float mb = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      const float m_new = fmaxf(m, mb);
      const bool grow = (m_new - m) * c > 8.0f;
      float alpha = 1.f;
      if (grow) {
        alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - m_new) * c);
        l *= alpha;
        m = m_new;
      }
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // Rare: bring O (all PV of earlier blocks have retired) onto the new max.
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
      const float mc = (m == -INFINITY) ? 0.f : m * c;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = ex2_approx(fmaf(s[64 * h + 2 * i], c, -mc));
          const float b = ex2_approx(fmaf(s[64 * h + 2 * i + 1], c, -mc));
          ls[i & 3] += a + b;
          pk[i] = pack2<kBf16>(a, b);
        }
        tmem_st32(tS + 32 * h, pk);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&ctl.p_full[t]);
    }

    // ------------------------------------------------------------- epilogue
    bool store = ok && n_t > 0;
    if (store) {
      store = __all_sync(0xffffffffu, mbar_wait(&ctl.o_full[t], 0, abort_flag, status, kWatchO + 1 + t));
    }
    uint8_t* stage = sQ + t * C::kTileBytes;  // Q tile t is dead once O_t is final
    if (store) {
      tc_fence_after();
      const float inv_l = 1.f / l;
#pragma unroll 1
      for (int cc = 0; cc < kD; cc += 32) {
        uint32_t o[32];
        tmem_ld32(tO + cc, o);
        tmem_wait_ld();
        const int cb = cc / 64;
        const int chunk0 = (cc % 64) / 8;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 v;
          v.x = pack2<kBf16>(__uint_as_float(o[8 * q4 + 0]) * inv_l, __uint_as_float(o[8 * q4 + 1]) * inv_l);
          v.y = pack2<kBf16>(__uint_as_float(o[8 * q4 + 2]) * inv_l, __uint_as_float(o[8 * q4 + 3]) * inv_l);
          v.z = pack2<kBf16>(__uint_as_float(o[8 * q4 + 4]) * inv_l, __uint_as_float(o[8 * q4 + 5]) * inv_l);
          v.w = pack2<kBf16>(__uint_as_float(o[8 * q4 + 6]) * inv_l, __uint_as_float(o[8 * q4 + 7]) * inv_l);
          const int chunk = chunk0 + q4;
          const uint32_t off = cb * 16384 + row_in_tile * 128 + ((chunk ^ (row_in_tile & 7)) << 4);
          *reinterpret_cast<uint4*>(stage + off) = v;
        }
      }
      fence_proxy_async_smem();
    }
    // All four warps of the group pass this barrier exactly once.
    named_barrier_sync(1 + t, 128);
    if (store && (threadIdx.x & 127) == 0) {
      for (int cb = 0; cb < kD / 64; ++cb)
        tma_store_3d(&map_o, smem_addr(stage + cb * 16384), cb * 64, q0 + t * 128, bh);
      tma_store_commit();
      tma_store_wait_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------

template <bool kBf16, int kD, bool kCausal>
static int launch_impl(const void* q, const void* k, const void* v, void* out, int BH, int Sq, int Skv,
                       float scale, cudaStream_t stream) {
  using C = Cfg<kD>;
  CUtensorMap mq, mk, mv, mo;
  const uint64_t D = kD;
  if (make_tensor_map_3d(&mq, q, kBf16, D, Sq, BH, D, static_cast<uint64_t>(Sq) * D, 64, 128) ||
      make_tensor_map_3d(&mk, k, kBf16, D, Skv, BH, D, static_cast<uint64_t>(Skv) * D, 64, 128) ||
      make_tensor_map_3d(&mv, v, kBf16, D, Skv, BH, D, static_cast<uint64_t>(Skv) * D, 64, 128) ||
      make_tensor_map_3d(&mo, out, kBf16, D, Sq, BH, D, static_cast<uint64_t>(Sq) * D, 64, 128))
    return ATTN_ERR_TENSOR_MAP;

  auto kern = attn_fwd_kernel<kBf16, kD, kCausal>;
  // Opt in to the large dynamic shared-memory carve-out once per device.
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
      configured[dev] = true;
    }
  }
  AttnParams prm;
  prm.Lq = Sq;
  prm.Lk = Skv;
  prm.BH = BH;
  prm.num_qblocks = (Sq + 255) / 256;
  prm.scale_log2 = scale * 1.4426950408889634f;
  const long long grid = static_cast<long long>(prm.num_qblocks) * BH;
  if (grid > 0x7fffffffLL) return ATTN_ERR_INVALID_ARGUMENT;
  kern<<<static_cast<unsigned>(grid), C::kThreads, C::kSmemBytes, stream>>>(mq, mk, mv, mo, prm);
  return cudaGetLastError() == cudaSuccess ? ATTN_OK : ATTN_ERR_LAUNCH;
}

// Compute capability 10.x check, cached per device.
static int check_device() {
  static int cached[64] = {};  // 0 unknown, 1 ok, 2 not sm_100
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ATTN_ERR_DEVICE;
  if (cached[dev] == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return ATTN_ERR_DEVICE;
    cached[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return cached[dev] == 1 ? ATTN_OK : ATTN_ERR_DEVICE;
}

}  // namespace ra

extern "C" int launch_attn_forward(const void* q, const void* k, const void* v, void* out, int B, int H, int Sq,
                                   int Skv, int D, bool causal, float softmax_scale, AttnDType dtype,
                                   cudaStream_t stream) {
  using namespace ra;
  if (B < 0 || H < 0 || Sq < 0 || Skv < 0 || D <= 0) return ATTN_ERR_INVALID_ARGUMENT;
  if (dtype != ATTN_F16 && dtype != ATTN_BF16) return ATTN_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return ATTN_ERR_UNSUPPORTED;
  const long long BH = static_cast<long long>(B) * H;
  if (BH == 0 || Sq == 0) return ATTN_OK;  // empty output, nothing to do
  if (BH > 0x7fffffffLL) return ATTN_ERR_INVALID_ARGUMENT;
  if (!q || !out || (Skv > 0 && (!k || !v))) return ATTN_ERR_INVALID_ARGUMENT;
  auto misaligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; };
  if (misaligned(q) || misaligned(out) || (Skv > 0 && (misaligned(k) || misaligned(v))))
    return ATTN_ERR_MISALIGNED;
  const int dev_ok = check_device();
  if (dev_ok != ATTN_OK) return dev_ok;
  if (Skv == 0) {
    // No keys: every row's softmax denominator is empty; the reference
    // writes zeros in that case.
    const size_t bytes = static_cast<size_t>(BH) * Sq * D * 2;
    return cudaMemsetAsync(out, 0, bytes, stream) == cudaSuccess ? ATTN_OK : ATTN_ERR_LAUNCH;
  }
  float scale = softmax_scale;
  if (!(scale > 0.f) || !isfinite(scale)) scale = 1.0f / sqrtf(static_cast<float>(D));
  const bool bf16 = dtype == ATTN_BF16;
  const int bh = static_cast<int>(BH);
#define RA_DISPATCH(BF, DD, CA) \
  if (bf16 == BF && D == DD && causal == CA) return launch_impl<BF, DD, CA>(q, k, v, out, bh, Sq, Skv, scale, stream);
  RA_DISPATCH(false, 128, false)
  RA_DISPATCH(false, 128, true)
  RA_DISPATCH(false, 64, false)
  RA_DISPATCH(false, 64, true)
  RA_DISPATCH(true, 128, false)
  RA_DISPATCH(true, 128, true)
  RA_DISPATCH(true, 64, false)
  RA_DISPATCH(true, 64, true)
#undef RA_DISPATCH
  return ATTN_ERR_UNSUPPORTED;
}

extern "C" int attn_get_status(cudaStream_t stream, int* status) {
  if (!status) return ATTN_ERR_INVALID_ARGUMENT;
  int host = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(&host, ra::g_attn_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaMemcpyToSymbolAsync(ra::g_attn_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return ATTN_ERR_LAUNCH;
  *status = host == 0 ? ATTN_OK : ATTN_ERR_WATCHDOG;
  return ATTN_OK;
}

extern "C" int attn_library_version(void) { return 100; }
