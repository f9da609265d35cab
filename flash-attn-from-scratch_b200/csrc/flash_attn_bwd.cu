// flash_attn_bwd.cu — flash-attention backward on sm_100a: tcgen05 MMAs into tensor memory,
// TMA tile streaming, no atomics.
//
// Restates the backward of the reference (kernels/flash_attn/flash_attn_bwd.py:127-237, the
// FlashAttention-2 recurrences it cites), with the forward's log-sum-exp L (:118-119) and
// Delta_m = sum_d dO[m,d] O[m,d] (:293):
//     P  = exp(scale * Q K^T - L)          recomputed per tile, never stored
//     dV = P^T dO                          dP = dO V^T
//     dS = P * (dP - Delta)                dQ = scale * dS K,   dK = scale * dS^T Q
// The reference accumulates dQ with atomics from the key-tile loop (:217-220); here dQ has its
// own pass over key tiles, so every sum is formed in a fixed order and repeated calls give
// identical bits.  (The reference's kernels cannot run as written: the head dimension D they
// use at :85 and :190 is never defined.)
//
// Three kernels, all on the launching stream:
//   fa_bwd_prep_kernel   Delta[b,h,m] = sum_d O * dO in fp32 (HBM-bound: reads O and dO once).
//   fa_bwd_dkdv_kernel   CTA = one (b, h) and 128 keys; loops over the query blocks that see
//                        them.  Tensor memory: S^T = K Q^T [0,128), dP^T = V dO^T [128,256),
//                        dV [256, 256+D), dK [256+D, 256+2D) (fp32).  P^T and dS^T (input
//                        dtype, two per column) overwrite S^T / dP^T and feed dV += P^T dO and
//                        dK += dS^T Q as the A operand from tensor memory.
//   fa_bwd_dq_kernel     CTA = one (b, h) and 128 queries; loops over the visible key blocks.
//                        S = Q K^T [0,128), dP = dO V^T [128,256), dQ [256, 256+D); dS
//                        overwrites S and feeds dQ += dS K.
// Roles (10 warps, one CTA per SM): warps 0-7 compute (thread = one TMEM lane = one row; warp
// w handles lane quadrant w % 4 and column half w / 4), warp 8 TMA producer, warp 9 TMEM owner
// and MMA issuer (the whole warp runs the loop, one elected lane issues).  All MMAs are M128 N128 (or N=D) K16 kind::f16, with the
// operand forms of the forward kernel: K-major A and B from shared memory for the score-like
// products, A from tensor memory and an MN-major B for the accumulations.  Every mbarrier wait
// is bounded; teardown drains copies and MMAs before tensor memory is freed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "fa_common.cuh"
#include "lk_abi.h"
#include "lk_sm100.cuh"

namespace lk {
namespace fab {

using fa::ex2;
using fa::f2;
using fa::fma2;
using fa::pack2;
using fa::uf2;

constexpr int kThreads = 320;
constexpr int kTile = 128;  // rows of every Q / K / V / dO tile
constexpr float kLog2e = 1.4426950408889634f;

enum Site : int {
  kSiteLoad = 301,
  kSiteMmaIn = 302,
  kSiteMmaP = 303,
  kSiteMmaDs = 304,
  kSiteSoftS = 305,
  kSiteSoftDp = 306,
  kSiteAcc = 307,
  kSiteTeardown = 308,
};

struct Params {
  int B, H, M, N;
  int H_kv, kv_group;  // K/V heads, query heads per K/V head (grouped-query attention)
  int causal;
  float scale;       // softmax scale (also the dQ / dK multiplier)
  float scale_log2;  // scale * log2(e)
  int num_qtiles, num_ktiles;
  int group_heads;  // heads per scheduling group
  // lse and delta: fp32 [B*H][lse_ld], rows padded to whole 128-row tiles (lse_ld % 4 == 0)
  const float* lse;
  const float* delta;
  int64_t lse_ld;
  void* out0;  // dkdv: dV, dq: dQ
  void* out1;  // dkdv: dK
  int64_t s0[3], s1[3];  // element strides (b, h, row) of out0 / out1; the d stride is 1
};

template <int D>
struct Cfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr int kBudget = 232448 - 1024 - 512;  // opt-in smem - align slack - barriers
  // dK/dV: K, V resident; a ring of (Q, dO, 128 lse, 128 delta) stages.
  static constexpr int kDkdvStage = 2 * kTileBytes + 1024;
  static constexpr int kDkdvFit = (kBudget - 2 * kTileBytes) / kDkdvStage;
  static constexpr int kDkdvStages = kDkdvFit > 4 ? 4 : kDkdvFit;
  static constexpr int kDkdvSmem = 2 * kTileBytes + kDkdvStages * kDkdvStage + 1024 + 512;
  // dQ: Q, dO resident; a ring of (K, V) stages.
  static constexpr int kDqStage = 2 * kTileBytes;
  static constexpr int kDqFit = (kBudget - 2 * kTileBytes) / kDqStage;
  static constexpr int kDqStages = kDqFit > 4 ? 4 : kDqFit;
  static constexpr int kDqSmem = 2 * kTileBytes + kDqStages * kDqStage + 1024 + 512;
  static_assert(kDkdvStages >= 2 && kDqStages >= 2, "rings need two stages");
};

// Tensor-memory column of the A operand for K step ks (16 elements) of a 128-long K dimension
// whose packed halves sit at columns [base, base+32) (elements 0-63) and [base+64, base+96)
// (elements 64-127): each column-half warp packs its 64 values into the first half of the 64
// columns it read them from, so no warp overwrites columns another warp still reads.
__device__ __forceinline__ uint32_t packed_col(int ks) { return (uint32_t)((ks >> 2) * 64 + (ks & 3) * 8); }

// Scheduling over B * heads (query heads for dQ, K/V heads for dK/dV): heads in groups of
// p.group_heads, inside a group the tile index `t` of every head in turn, so the CTAs resident
// at a time share a few heads' operands in L2.
__device__ __forceinline__ void cta_coords(const Params& p, int heads, int ntiles, int& bh, int& t) {
  const int BH = p.B * heads;
  const int per_group = p.group_heads * ntiles;
  const int grp = (int)(blockIdx.x / per_group);
  const int gbase = grp * p.group_heads;
  const int gsz = min(p.group_heads, BH - gbase);
  const int rem = (int)(blockIdx.x - (unsigned)grp * per_group);
  t = rem / gsz;
  bh = gbase + rem % gsz;
}

// Stores 32 fp32 values (times mul) of one row as 16-bit values, 16-byte stores.
template <bool kBf16>
__device__ __forceinline__ void store_row32(void* dst, const uint32_t (&r)[32], float mul) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack2<kBf16>(__uint_as_float(r[8 * q + 0]) * mul, __uint_as_float(r[8 * q + 1]) * mul);
    w.y = pack2<kBf16>(__uint_as_float(r[8 * q + 2]) * mul, __uint_as_float(r[8 * q + 3]) * mul);
    w.z = pack2<kBf16>(__uint_as_float(r[8 * q + 4]) * mul, __uint_as_float(r[8 * q + 5]) * mul);
    w.w = pack2<kBf16>(__uint_as_float(r[8 * q + 6]) * mul, __uint_as_float(r[8 * q + 7]) * mul);
    d[q] = w;
  }
}

template <int D>
__device__ __forceinline__ void store_zero_row(void* dst) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < D / 8; ++q) d[q] = make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------------------------------------
// Delta[b,h,m] = sum_d O[b,h,m,d] * dO[b,h,m,d].  Each lane takes one 16-byte vector of a row,
// D / 8 lanes per row (two rows per warp at D = 128, four at D = 64), reduced by shuffles.
// ---------------------------------------------------------------------------------------------
template <int D, bool kBf16>
__global__ void __launch_bounds__(256) fa_bwd_prep_kernel(const void* __restrict__ o, const void* __restrict__ dout,
                                                          Params p, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                                          int64_t d_sb, int64_t d_sh, int64_t d_sm,
                                                          float* __restrict__ delta) {
  constexpr int kVec = D / 8;
  constexpr int kRowsPerWarp = 32 / kVec;
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * kRowsPerWarp + lane / kVec;
  const int v = lane % kVec;
  const int64_t rows = (int64_t)p.B * p.H * p.M;
  const bool live = row < rows;
  const int m = live ? (int)(row % p.M) : 0;
  const int bh = live ? (int)(row / p.M) : 0;
  const int b = bh / p.H, h = bh % p.H;
  float acc = 0.f;
  if (live) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(o) + b * o_sb + h * o_sh +
                                                         (int64_t)m * o_sm) + v);
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(dout) + b * d_sb + h * d_sh +
                                                         (int64_t)m * d_sm) + v);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a0, a1, c0, c1;
      if constexpr (kBf16) {
        a0 = __uint_as_float(aw[j] << 16), a1 = __uint_as_float(aw[j] & 0xFFFF0000u);
        c0 = __uint_as_float(cw[j] << 16), c1 = __uint_as_float(cw[j] & 0xFFFF0000u);
      } else {
        a0 = __half2float(__ushort_as_half((unsigned short)(aw[j] & 0xFFFFu)));
        a1 = __half2float(__ushort_as_half((unsigned short)(aw[j] >> 16)));
        c0 = __half2float(__ushort_as_half((unsigned short)(cw[j] & 0xFFFFu)));
        c1 = __half2float(__ushort_as_half((unsigned short)(cw[j] >> 16)));
      }
      acc = fmaf(a0, c0, acc);
      acc = fmaf(a1, c1, acc);
    }
  }
#pragma unroll
  for (int off = kVec / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && v == 0) delta[(int64_t)bh * p.lse_ld + m] = acc;
}

// ---------------------------------------------------------------------------------------------
// dK, dV for 128 keys of one (b, h).
// ---------------------------------------------------------------------------------------------
template <int D, bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const Params p) {
  using C = Cfg<D>;
  constexpr int S = C::kDkdvStages;
  constexpr int T = C::kTileBytes;
  constexpr uint32_t kIdescS = make_idesc(1, kBf16 ? 1 : 0, kBf16 ? 1 : 0, 0, 0, kTile, kTile);
  constexpr uint32_t kIdescAcc = make_idesc(1, kBf16 ? 1 : 0, kBf16 ? 1 : 0, 0, 1, kTile, D);
  constexpr uint32_t kColS = 0, kColDp = 128, kColDv = 256, kColDk = 256 + D;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + T;
  uint8_t* sRing = smem + 2 * T;  // stage: Q [T], dO [T], lse [128 f32], delta [128 f32]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + S * C::kDkdvStage);
  uint64_t* kv_full = bars;           // [1]
  uint64_t* q_full = bars + 1;        // [S]  TMA -> MMA and compute
  uint64_t* q_empty = q_full + S;     // [S]  MMA commit -> TMA
  uint64_t* s_full = q_empty + S;     // [1]  S^T complete
  uint64_t* dp_full = s_full + 1;     // [1]  dP^T complete
  uint64_t* p_ready = dp_full + 1;    // [1]  P^T in tensor memory (8 warp arrivals)
  uint64_t* ds_ready = p_ready + 1;   // [1]  dS^T in tensor memory (8 warp arrivals)
  uint64_t* acc_full = ds_ready + 1;  // [1]  dV, dK complete
  uint64_t* drain = acc_full + 1;     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  int bhk, kt;
  cta_coords(p, p.H_kv, p.num_ktiles, bhk, kt);  // kt ascending = heaviest first when causal
  const int b = bhk / p.H_kv, hk = bhk % p.H_kv;  // this CTA's K/V head
  const int n0 = kt * kTile;
  const int i0 = p.causal ? kt : 0;  // first query tile that sees a key of this tile (n <= m)
  const int nq = p.num_qtiles > i0 ? p.num_qtiles - i0 : 0;
  // Blocks j = g * nq + (i - i0): query head hk * kv_group + g, query tile i.  The query heads
  // sharing this K/V head all accumulate into the same dK, dV.
  const int nblk = nq * p.kv_group;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(ds_ready, 8);
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && nq > 0) {
      mbar_arrive_expect_tx(kv_full, 2 * T);
      for (int x = 0; x < C::kBoxes; ++x) {
        tma_load_4d(sK + x * (kTile * 128), &tmK, kv_full, 64 * x, n0, hk, b);
        tma_load_4d(sV + x * (kTile * 128), &tmV, kv_full, 64 * x, n0, hk, b);
      }
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int st = j % S;
        if (!mbar_wait(&q_empty[st], ((j / S) & 1) ^ 1u, kSiteLoad)) break;
        const int qh = hk * p.kv_group + j / nq;
        const int m0 = (i0 + j % nq) * kTile;
        uint8_t* stage = sRing + st * C::kDkdvStage;
        mbar_arrive_expect_tx(&q_full[st], 2 * T + 1024);
        for (int x = 0; x < C::kBoxes; ++x) {
          tma_load_4d(stage + x * (kTile * 128), &tmQ, &q_full[st], 64 * x, m0, qh, b);
          tma_load_4d(stage + T + x * (kTile * 128), &tmDO, &q_full[st], 64 * x, m0, qh, b);
        }
        const int64_t row = (int64_t)(b * p.H + qh) * p.lse_ld + m0;
        bulk_load(stage + 2 * T, p.lse + row, 512, &q_full[st]);
        bulk_load(stage + 2 * T + 512, p.delta + row, 512, &q_full[st]);
        issued = j + 1;
      }
      // Teardown: every copy issued lands before the CTA can exit.
      mbar_wait_drain(kv_full, 0, kSiteTeardown);
      for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
        mbar_wait_drain(&q_full[j % S], (j / S) & 1, kSiteTeardown);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the issue loop (voted waits) and one elected lane issues each MMA
    // and commit: 10% faster than a loop of lane 0 alone for these 64-cycle N=128 MMAs.
    if (nq > 0) {
      bool ok = mbar_wait_warp(kv_full, 0, kSiteMmaIn);
      const uint64_t k_desc = sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t v_desc = sdesc_sw128(smem_u32(sV), 16, 1024);
      for (int j = 0; j < nblk && ok; ++j) {
        const int st = j % S;
        if (!(ok = mbar_wait_warp(&q_full[st], (j / S) & 1, kSiteMmaIn))) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sRing + st * C::kDkdvStage);
        const uint32_t do_addr = q_addr + T;
        const uint64_t q_kmaj = sdesc_sw128(q_addr, 16, 1024);
        const uint64_t do_kmaj = sdesc_sw128(do_addr, 16, 1024);
        const uint64_t q_mn = sdesc_sw128(q_addr, kTile * 128, 1024);
        const uint64_t do_mn = sdesc_sw128(do_addr, kTile * 128, 1024);
        // S^T = K Q^T and dP^T = V dO^T: K = D in steps of 16.
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kTile * 128) + (ks & 3) * 32;
          mma_f16_ss_warp(tmem + kColS, sdesc_add(k_desc, off), sdesc_add(q_kmaj, off), kIdescS, ks > 0);
        }
        tc_commit_warp(s_full);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kTile * 128) + (ks & 3) * 32;
          mma_f16_ss_warp(tmem + kColDp, sdesc_add(v_desc, off), sdesc_add(do_kmaj, off), kIdescS, ks > 0);
        }
        tc_commit_warp(dp_full);
        // dV += P^T dO: K = the 128 queries of the tile, 16 per step.
        if (!(ok = mbar_wait_warp(p_ready, j & 1, kSiteMmaP))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks)
          mma_f16_ts_warp(tmem + kColDv, tmem + kColS + packed_col(ks), sdesc_add(do_mn, ks * 16 * 128), kIdescAcc,
                     (j > 0 || ks > 0) ? 1u : 0u);
        // dK += dS^T Q (scaled in the epilogue).
        if (!(ok = mbar_wait_warp(ds_ready, j & 1, kSiteMmaDs))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks)
          mma_f16_ts_warp(tmem + kColDk, tmem + kColDp + packed_col(ks), sdesc_add(q_mn, ks * 16 * 128), kIdescAcc,
                     (j > 0 || ks > 0) ? 1u : 0u);
        tc_commit_warp(&q_empty[st]);  // the stage (Q, dO, lse, delta) is free once these are done
      }
      if (ok) tc_commit_warp(acc_full);
      tc_commit_warp(drain);
      mbar_wait_drain(drain, 0, kSiteTeardown);
    }
  } else {
    // ---------------------------------------------------------------- compute (warps 0-7)
    const int qd = warp & 3;
    const int hf = warp >> 2;  // column half: queries [64 hf, 64 hf + 64) of each tile
    const int r = qd * 32 + lane;
    const int n = n0 + r;  // this thread's key
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      const int st = j % S;
      const int m0 = (i0 + j % nq) * kTile;
      const float* s_lse = reinterpret_cast<const float*>(sRing + st * C::kDkdvStage + 2 * T) + hf * 64;
      const float* s_delta = s_lse + 128;
      if (!(ok = mbar_wait_warp(&q_full[st], (j / S) & 1, kSiteSoftS))) break;  // lse / delta visible
      if (!(ok = mbar_wait_warp(s_full, j & 1, kSiteSoftS))) break;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(tmem + lane_off + kColS + hf * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(tmem + lane_off + kColS + hf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_wait_ld();
      // Columns to zero: queries past M, and (causal) queries before this key.
      const bool masked_tile = (m0 + kTile > p.M) || (p.causal && n0 + kTile - 1 > m0);
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
      float pv[64];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float2 l2 = *reinterpret_cast<const float2*>(s_lse + c);
        const uint64_t x2 = fma2(f2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2,
                                 f2(-l2.x * kLog2e, -l2.y * kLog2e));
        float x0, x1;
        uf2(x2, x0, x1);
        pv[c] = ex2(x0);
        pv[c + 1] = ex2(x1);
      }
      if (masked_tile) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int m = m0 + hf * 64 + c;
          if (m >= p.M || (p.causal && n > m)) pv[c] = 0.f;
        }
      }
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) pk[c] = pack2<kBf16>(pv[2 * c], pv[2 * c + 1]);
      tmem_st32(tmem + lane_off + kColS + hf * 64, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      // dS^T = P^T * (dP^T - Delta), 32 columns at a time.
      if (!(ok = mbar_wait_warp(dp_full, j & 1, kSiteSoftDp))) break;
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint32_t dp[32];
        tmem_ld32(tmem + lane_off + kColDp + hf * 64 + ch * 32, dp);
        tmem_wait_ld();
        uint32_t dk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float2 d2 = *reinterpret_cast<const float2*>(s_delta + ch * 32 + c);
          float a = pv[ch * 32 + c] * (__uint_as_float(dp[c]) - d2.x);
          float bb = pv[ch * 32 + c + 1] * (__uint_as_float(dp[c + 1]) - d2.y);
          if (masked_tile) {  // Delta past M is not data: keep masked columns exactly zero
            const int m = m0 + hf * 64 + ch * 32 + c;
            if (m >= p.M || (p.causal && n > m)) a = 0.f;
            if (m + 1 >= p.M || (p.causal && n > m + 1)) bb = 0.f;
          }
          dk[c / 2] = pack2<kBf16>(a, bb);
        }
        tmem_st16(tmem + lane_off + kColDp + hf * 64 + ch * 16, dk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
    }
    // Epilogue: warps of half 0 write dV, of half 1 dK (times the softmax scale).  The tensor
    // memory loads are warp-wide; only the stores depend on the row.
    void* out = hf == 0 ? p.out0 : p.out1;
    const int64_t* so = hf == 0 ? p.s0 : p.s1;
    uint16_t* row = static_cast<uint16_t*>(out) + b * so[0] + hk * so[1] + (int64_t)n * so[2];
    if (nq == 0) {
      if (n < p.N) store_zero_row<D>(row);  // no query sees these keys
    } else if (ok && mbar_wait_warp(acc_full, 0, kSiteAcc)) {
      tc_fence_after();
      const uint32_t col = hf == 0 ? kColDv : kColDk;
      const float mul = hf == 0 ? 1.f : p.scale;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + col + c * 32, v);
        tmem_wait_ld();
        if (n < p.N) store_row32<kBf16>(row + c * 32, v, mul);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------------------
// dQ for 128 queries of one (b, h).
// ---------------------------------------------------------------------------------------------
template <int D, bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                     const Params p) {
  using C = Cfg<D>;
  constexpr int S = C::kDqStages;
  constexpr int T = C::kTileBytes;
  constexpr uint32_t kIdescS = make_idesc(1, kBf16 ? 1 : 0, kBf16 ? 1 : 0, 0, 0, kTile, kTile);
  constexpr uint32_t kIdescAcc = make_idesc(1, kBf16 ? 1 : 0, kBf16 ? 1 : 0, 0, 1, kTile, D);
  constexpr uint32_t kColS = 0, kColDp = 128, kColDq = 256;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = smem + T;
  uint8_t* sRing = smem + 2 * T;  // stage: K [T], V [T]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + S * C::kDqStage);
  uint64_t* q_full = bars;            // [1]
  uint64_t* kv_full = bars + 1;       // [S]
  uint64_t* kv_empty = kv_full + S;   // [S]
  uint64_t* s_full = kv_empty + S;    // [1]
  uint64_t* dp_full = s_full + 1;     // [1]
  uint64_t* ds_ready = dp_full + 1;   // [1]  (8 warp arrivals)
  uint64_t* acc_full = ds_ready + 1;  // [1]
  uint64_t* drain = acc_full + 1;     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  int bh, t;
  cta_coords(p, p.H, p.num_qtiles, bh, t);
  const int qt = p.causal ? p.num_qtiles - 1 - t : t;  // causal: the longest key loops first
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / p.kv_group;  // K/V head of query head h
  const int m0 = qt * kTile;
  const int nk = p.causal ? min(p.num_ktiles, qt + 1) : p.num_ktiles;  // key n visible iff n <= m

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(ds_ready, 8);
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * T);
      for (int x = 0; x < C::kBoxes; ++x) {
        tma_load_4d(sQ + x * (kTile * 128), &tmQ, q_full, 64 * x, m0, h, b);
        tma_load_4d(sDO + x * (kTile * 128), &tmDO, q_full, 64 * x, m0, h, b);
      }
      int issued = 0;
      for (int j = 0; j < nk; ++j) {
        const int st = j % S;
        if (!mbar_wait(&kv_empty[st], ((j / S) & 1) ^ 1u, kSiteLoad)) break;
        uint8_t* stage = sRing + st * C::kDqStage;
        mbar_arrive_expect_tx(&kv_full[st], 2 * T);
        for (int x = 0; x < C::kBoxes; ++x) {
          tma_load_4d(stage + x * (kTile * 128), &tmK, &kv_full[st], 64 * x, j * kTile, hk, b);
          tma_load_4d(stage + T + x * (kTile * 128), &tmV, &kv_full[st], 64 * x, j * kTile, hk, b);
        }
        issued = j + 1;
      }
      mbar_wait_drain(q_full, 0, kSiteTeardown);
      for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
        mbar_wait_drain(&kv_full[j % S], (j / S) & 1, kSiteTeardown);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the issue loop (voted waits); one elected lane issues.
    {
      bool ok = mbar_wait_warp(q_full, 0, kSiteMmaIn);
      const uint64_t q_desc = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t do_desc = sdesc_sw128(smem_u32(sDO), 16, 1024);
      for (int j = 0; j < nk && ok; ++j) {
        const int st = j % S;
        if (!(ok = mbar_wait_warp(&kv_full[st], (j / S) & 1, kSiteMmaIn))) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sRing + st * C::kDqStage);
        const uint64_t k_kmaj = sdesc_sw128(k_addr, 16, 1024);
        const uint64_t v_kmaj = sdesc_sw128(k_addr + T, 16, 1024);
        const uint64_t k_mn = sdesc_sw128(k_addr, kTile * 128, 1024);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kTile * 128) + (ks & 3) * 32;
          mma_f16_ss_warp(tmem + kColS, sdesc_add(q_desc, off), sdesc_add(k_kmaj, off), kIdescS, ks > 0);
        }
        tc_commit_warp(s_full);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kTile * 128) + (ks & 3) * 32;
          mma_f16_ss_warp(tmem + kColDp, sdesc_add(do_desc, off), sdesc_add(v_kmaj, off), kIdescS, ks > 0);
        }
        tc_commit_warp(dp_full);
        // dQ += dS K (scaled in the epilogue): K = the 128 keys of the block, 16 per step.
        if (!(ok = mbar_wait_warp(ds_ready, j & 1, kSiteMmaDs))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks)
          mma_f16_ts_warp(tmem + kColDq, tmem + kColS + packed_col(ks), sdesc_add(k_mn, ks * 16 * 128), kIdescAcc,
                     (j > 0 || ks > 0) ? 1u : 0u);
        tc_commit_warp(&kv_empty[st]);
      }
      if (ok) tc_commit_warp(acc_full);
      tc_commit_warp(drain);
      mbar_wait_drain(drain, 0, kSiteTeardown);
    }
  } else {
    // ---------------------------------------------------------------- compute (warps 0-7)
    const int qd = warp & 3;
    const int hf = warp >> 2;  // column half: keys [64 hf, 64 hf + 64) of each block
    const int r = qd * 32 + lane;
    const int m = m0 + r;  // this thread's query
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const bool row_ok = m < p.M;
    const float nlse = row_ok ? -p.lse[(int64_t)bh * p.lse_ld + m] * kLog2e : 0.f;
    const float dlt = row_ok ? p.delta[(int64_t)bh * p.lse_ld + m] : 0.f;
    bool ok = true;
    for (int j = 0; j < nk && ok; ++j) {
      const int n0 = j * kTile;
      if (!(ok = mbar_wait_warp(s_full, j & 1, kSiteSoftS))) break;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(tmem + lane_off + kColS + hf * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(tmem + lane_off + kColS + hf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_wait_ld();
      const bool masked_tile = (n0 + kTile > p.N) || (p.causal && n0 + kTile - 1 > m0);
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
      const uint64_t nl2 = f2(nlse, nlse);
      float pv[64];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const uint64_t x2 = fma2(f2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, nl2);
        float x0, x1;
        uf2(x2, x0, x1);
        pv[c] = ex2(x0);
        pv[c + 1] = ex2(x1);
      }
      if (masked_tile) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int n = n0 + hf * 64 + c;
          if (n >= p.N || (p.causal && n > m)) pv[c] = 0.f;
        }
      }
      if (!(ok = mbar_wait_warp(dp_full, j & 1, kSiteSoftDp))) break;
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint32_t dp[32];
        tmem_ld32(tmem + lane_off + kColDp + hf * 64 + ch * 32, dp);
        tmem_wait_ld();
        uint32_t dk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2)
          dk[c / 2] = pack2<kBf16>(pv[ch * 32 + c] * (__uint_as_float(dp[c]) - dlt),
                                   pv[ch * 32 + c + 1] * (__uint_as_float(dp[c + 1]) - dlt));
        // dS packed into the first half of the S columns this warp read (no other warp reads them).
        tmem_st16(tmem + lane_off + kColS + hf * 64 + ch * 16, dk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
    }
    // Epilogue: each warp writes D/2 columns of dQ (times the softmax scale) for its 32 rows.
    if (ok && mbar_wait_warp(acc_full, 0, kSiteAcc)) {
      tc_fence_after();
      uint16_t* row = static_cast<uint16_t*>(p.out0) + b * p.s0[0] + h * p.s0[1] + (int64_t)m * p.s0[2];
#pragma unroll 1
      for (int c = hf * (D / 64); c < (hf + 1) * (D / 64); ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + kColDq + c * 32, v);
        tmem_wait_ld();
        if (row_ok) store_row32<kBf16>(row + c * 32, v, p.scale);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// Opts `Kern` into `bytes` of dynamic shared memory on the current device, once per device (the
// flag lives in this instantiation, i.e. per kernel).
template <auto Kern>
int set_smem(int bytes) {
  static std::atomic<uint64_t> configured{0};
  auto kern = Kern;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return cuda_status(e);
    configured.fetch_or(bit);
  }
  return LK_OK;
}

int group_heads(int64_t BH, int64_t ntiles, int waves) {
  const int64_t g = (int64_t)waves * sm_count() / (ntiles > 0 ? ntiles : 1);
  return (int)(g < 1 ? 1 : (g > BH ? BH : g));
}

template <int D, bool kBf16>
int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
           const void* o, const int64_t* o_st, const void* dout, const int64_t* do_st, float* delta, Params p,
           void* dq, const int64_t* dq_st, void* dk, const int64_t* dk_st, void* dv, const int64_t* dv_st,
           cudaStream_t s) {
  using C = Cfg<D>;
  const int64_t BH = (int64_t)p.B * p.H;
  // 1) Delta
  {
    const int64_t rows = BH * p.M;
    const int64_t rows_per_cta = 8 * (32 / (D / 8));
    fa_bwd_prep_kernel<D, kBf16><<<(unsigned)((rows + rows_per_cta - 1) / rows_per_cta), 256, 0, s>>>(
        o, dout, p, o_st[0], o_st[1], o_st[2], do_st[0], do_st[1], do_st[2], delta);
    if (int st = check_launch()) return st;
  }
  p.delta = delta;
  // 2) dK, dV
  {
    auto kern = fa_bwd_dkdv_kernel<D, kBf16>;
    if (int st = set_smem<fa_bwd_dkdv_kernel<D, kBf16>>(C::kDkdvSmem)) return st;
    Params q = p;
    q.out0 = dv;
    q.out1 = dk;
    for (int i = 0; i < 3; ++i) {
      q.s0[i] = dv_st[i];
      q.s1[i] = dk_st[i];
    }
    const int64_t BHk = (int64_t)p.B * p.H_kv;
    q.group_heads = group_heads(BHk, p.num_ktiles, p.causal ? 3 : 1);
    kern<<<(unsigned)(BHk * p.num_ktiles), kThreads, C::kDkdvSmem, s>>>(tq, tk, tv, tdo, q);
    if (int st = check_launch()) return st;
  }
  // 3) dQ
  {
    auto kern = fa_bwd_dq_kernel<D, kBf16>;
    if (int st = set_smem<fa_bwd_dq_kernel<D, kBf16>>(C::kDqSmem)) return st;
    Params q = p;
    q.out0 = dq;
    for (int i = 0; i < 3; ++i) q.s0[i] = dq_st[i];
    q.group_heads = group_heads(BH, p.num_qtiles, p.causal ? 3 : 1);
    kern<<<(unsigned)(BH * p.num_qtiles), kThreads, C::kDqSmem, s>>>(tq, tk, tv, tdo, q);
    return check_launch();
  }
}

}  // namespace fab
}  // namespace lk

extern "C" int lk_flash_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                 const float* lse, int64_t lse_ld, void* dq, void* dk, void* dv, float* delta,
                                 int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t M, int64_t N, int64_t D,
                                 const int64_t* strides, int causal, float softmax_scale, void* stream) {
  using namespace lk;
  if (B < 0 || H < 0 || M < 0 || N < 0) return LK_ERR_INVALID_ARG;
  if (H > 0 && (H_kv <= 0 || H % H_kv != 0)) return LK_ERR_INVALID_ARG;
  if (B == 0 || H == 0 || (M == 0 && N == 0)) return LK_OK;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || !delta || !strides) return LK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return LK_ERR_INVALID_ARG;  // gradients of an empty softmax are undefined
  if (dtype != LK_BF16 && dtype != LK_F16) return LK_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return LK_ERR_UNSUPPORTED;
  if (M > (1 << 30) || N > (1 << 30) || B * H > (1 << 24)) return LK_ERR_INVALID_ARG;
  const int64_t num_qtiles = (M + fab::kTile - 1) / fab::kTile;
  const int64_t num_ktiles = (N + fab::kTile - 1) / fab::kTile;
  if (lse_ld < num_qtiles * fab::kTile || lse_ld % 4) return LK_ERR_INVALID_ARG;
  if (((uintptr_t)lse & 15) || ((uintptr_t)delta & 15)) return LK_ERR_ALIGNMENT;
  if (B * H * num_ktiles > 0x7FFFFFFF || B * H * num_qtiles > 0x7FFFFFFF) return LK_ERR_INVALID_ARG;
  // strides: 8 tensors x (b, h, row, d) in the order q, k, v, o, dout, dq, dk, dv.
  const int64_t* sq = strides;
  const int64_t* sk = strides + 4;
  const int64_t* sv = strides + 8;
  const int64_t* so = strides + 12;
  const int64_t* sdo = strides + 16;
  const int64_t* sdq = strides + 20;
  const int64_t* sdk = strides + 24;
  const int64_t* sdv = strides + 28;
  // O, dO are read with 16-byte loads and dQ, dK, dV written with 16-byte stores.
  const void* vec_ptrs[5] = {o, dout, dq, dk, dv};
  const int64_t* vec_st[5] = {so, sdo, sdq, sdk, sdv};
  for (int i = 0; i < 5; ++i) {
    if (vec_st[i][3] != 1 || ((uintptr_t)vec_ptrs[i] & 15)) return LK_ERR_ALIGNMENT;
    for (int j = 0; j < 3; ++j)
      if (vec_st[i][j] % 8) return LK_ERR_ALIGNMENT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = bind_stream(s)) return st;
  const bool bf16 = dtype == LK_BF16;
  CUtensorMap tq, tk, tv, tdo;
  if (int st = fa::make_map(&tq, bf16, q, B, H, M, D, sq)) return st;
  if (int st = fa::make_map(&tk, bf16, k, B, H_kv, N, D, sk)) return st;
  if (int st = fa::make_map(&tv, bf16, v, B, H_kv, N, D, sv)) return st;
  if (int st = fa::make_map(&tdo, bf16, dout, B, H, M, D, sdo)) return st;
  fab::Params p{};
  p.B = (int)B;
  p.H = (int)H;
  p.M = (int)M;
  p.N = (int)N;
  p.H_kv = (int)H_kv;
  p.kv_group = (int)(H / H_kv);
  p.causal = causal ? 1 : 0;
  p.scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = p.scale * fab::kLog2e;
  p.num_qtiles = (int)num_qtiles;
  p.num_ktiles = (int)num_ktiles;
  p.lse = lse;
  p.lse_ld = lse_ld;
  if (D == 128)
    return bf16 ? fab::launch<128, true>(tq, tk, tv, tdo, o, so, dout, sdo, delta, p, dq, sdq, dk, sdk, dv, sdv, s)
                : fab::launch<128, false>(tq, tk, tv, tdo, o, so, dout, sdo, delta, p, dq, sdq, dk, sdk, dv, sdv, s);
  return bf16 ? fab::launch<64, true>(tq, tk, tv, tdo, o, so, dout, sdo, delta, p, dq, sdq, dk, sdk, dv, sdv, s)
              : fab::launch<64, false>(tq, tk, tv, tdo, o, so, dout, sdo, delta, p, dq, sdq, dk, sdk, dv, sdv, s);
}
