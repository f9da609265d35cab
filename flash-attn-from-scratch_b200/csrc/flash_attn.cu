// flash_attn.cu — flash-attention forward on sm_100a: tcgen05 MMAs into tensor memory, TMA
// K/V streaming, online softmax in registers.
//
// Restates the reference's online-softmax forward (kernels/flash_attn/flash_attn_fwd.py:47-64
// non-causal, :108-128 causal):  for each key block, S = Q K^T * scale, running row max m and
// row sum l, O = alpha * O + P V with P cast to the input dtype (:61), final O / l (:63).
// Causal masking keeps key n for query m iff n <= m (top-left, :118) and skips key blocks
// entirely above the diagonal (:112).
//
// CTA = one (batch, head) and 256 query rows held as two 128-row tiles (t = 0, 1).  10 warps:
//   warps 0-3  softmax for tile 0 (thread = one query row = one TMEM lane)
//   warps 4-7  softmax for tile 1
//   warp  8    TMA producer: Q0/Q1 once, then K_0, V_0, K_1, V_1, ... (consumption order)
//              through a ring of 128-row stages (128B swizzle)
//   warp  9    TMEM owner + MMA issuer (the whole warp; one elected lane issues)
// Tensor memory (512 columns): S_t = cols [128t, 128t+128) fp32, O_t = cols
// [256 + D*t, 256 + D*(t+1)) fp32.  P_t (the input dtype, two per column) overwrites the first
// 64 columns of S_t once the softmax has S_t(j) in registers, and the PV product takes its A
// operand from tensor memory (an M128 N128 K16 MMA costs the same 64 cycles with A in TMEM or
// in shared memory), so shared memory holds only Q and a deep K/V ring.
// Per tile the MMA warp issues PV_t(j) and then S_t(j+1) as soon as P_t(j) is ready: the
// tensor pipe executes a thread's MMAs in order, so S_t(j+1) overwrites P_t(j) only after
// PV_t(j) has read it, and when S_t(j+1) is complete PV_t(j) is too -- the softmax of block
// j+1 may then rescale O_t in place with no further wait.  The two tiles interleave, so the
// tensor core multiplies one tile while the other tile's softmax runs.
// Rescaling is lazy: the running max used for exp2 only moves when the block max exceeds it
// by more than 8 (log2 units), so P <= 256 and O is rarely touched.
// Every mbarrier wait is bounded; on failure all roles unwind and TMEM is freed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "fa_common.cuh"
#include "lk_abi.h"
#include "lk_sm100.cuh"

namespace lk {
namespace fa {

constexpr int kThreads = 320;
constexpr int kTileM = 128;   // query rows per tile
constexpr int kBlockN = 128;  // keys per block
constexpr float kRescaleThreshold = 8.0f;  // log2 units
#ifndef LK_FA_GROUP_HEADS
#define LK_FA_GROUP_HEADS 1  // 0: one global heavy-first order over all heads
#endif
// The two tiles take turns on the exp phase: measured faster at D = 128 (where the exp phase
// is on each tile's critical chain), slower at D = 64.  -1 = per head dim, 0/1 = off/on.
#ifndef LK_FA_EXP_TURNS
#define LK_FA_EXP_TURNS -1
#endif
template <int D>
__host__ __device__ constexpr bool exp_turns() {
  return LK_FA_EXP_TURNS < 0 ? (D == 128) : (LK_FA_EXP_TURNS != 0);
}

enum Site : int {
  kSiteLoadQ = 201,
  kSiteLoadEmpty = 202,
  kSiteMmaQ = 203,
  kSiteMmaKV = 204,
  kSiteMmaP = 205,
  kSiteSoftS = 206,
  kSiteSoftO = 207,
  kSiteTeardown = 208,
};

struct Params {
  int B, H, M, N;
  int num_qblocks;  // ceil(M / 256)
  int kv_group;     // query heads per K/V head (grouped-query attention; 1 = one K/V head each)
  int group_heads;  // heads per scheduling group (>= 1)
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  void* o;
  int64_t o_sb, o_sh, o_sm;  // element strides of O (d stride is 1)
  // Optional log-sum-exp output (nullptr: none): lse[(b*H + h) * lse_ld + m] =
  // ln(sum_n exp(scale * q_m . k_n)) over the visible keys.
  float* lse;
  int64_t lse_ld;
  // Test hook (lk_debug_inject): CTA drop_block's producer skips ring item drop_item (no copy,
  // no arrive).  drop_block = -1: none.
  int drop_block, drop_item;
};

template <int D>
struct Cfg {
  static constexpr int kQBoxes = D / 64;               // 64-element (128 B) boxes per row
  static constexpr int kTileBytes = kTileM * D * 2;    // one 128-row tile of Q, K or V
  static constexpr int kFixedBytes = 2 * kTileBytes;   // Q_0, Q_1
  static constexpr int kBudget = 232448 - 1024 - 512;  // opt-in smem - align slack - barriers
  static constexpr int kFit = (kBudget - kFixedBytes) / kTileBytes;
  static constexpr int kStages = kFit > 10 ? 10 : kFit;  // 5 (D=128) / 10 (D=64)
  static constexpr int kSmemBytes = kFixedBytes + kStages * kTileBytes + 1024 + 512;
  static constexpr int kOCol0 = 256;
  static_assert(kStages >= 4, "K/V ring needs four stages");
};

// Max of n fp32 values (bit patterns): four chains of three-input max over sr[4 .. n-4), the
// first and last four values opening and closing the chains.
template <int n>
__device__ __forceinline__ float row_max(const uint32_t (&sr)[n]) {
  static_assert(n % 8 == 0, "row length");
  float mx4[4] = {__uint_as_float(sr[0]), __uint_as_float(sr[1]), __uint_as_float(sr[2]), __uint_as_float(sr[3])};
#pragma unroll
  for (int c = 4; c < n - 4; c += 8) {
    mx4[0] = max3(mx4[0], __uint_as_float(sr[c + 0]), __uint_as_float(sr[c + 1]));
    mx4[1] = max3(mx4[1], __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
    mx4[2] = max3(mx4[2], __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
    mx4[3] = max3(mx4[3], __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
  }
  mx4[0] = max3(mx4[0], __uint_as_float(sr[n - 4]), __uint_as_float(sr[n - 3]));
  mx4[1] = max3(mx4[1], __uint_as_float(sr[n - 2]), __uint_as_float(sr[n - 1]));
  return fmaxf(max3(mx4[0], mx4[1], mx4[2]), mx4[3]);
}

template <int D, bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const Params p) {
  using C = Cfg<D>;
  constexpr int S = C::kStages;
  constexpr bool kExpTurns = exp_turns<D>();
  constexpr uint32_t kIdescS = make_idesc(1, kBf16 ? 1 : 0, kBf16 ? 1 : 0, 0, 0, kTileM, kBlockN);
  constexpr uint32_t kIdescO = make_idesc(1, kBf16 ? 1 : 0, kBf16 ? 1 : 0, 0, 1, kTileM, D);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                          // [2][kTileBytes]
  uint8_t* sRing = smem + 2 * C::kTileBytes;   // [S][kTileBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + S * C::kTileBytes);
  uint64_t* q_full = bars;             // [1]
  uint64_t* kv_full = bars + 1;        // [S]   TMA -> MMA
  uint64_t* kv_empty = kv_full + S;    // [S]   MMA -> TMA (tcgen05.commit)
  uint64_t* s_full = kv_empty + S;     // [2]   S_t(j) in TMEM, PV_t(j-1) complete (tcgen05.commit)
  uint64_t* p_full = s_full + 2;       // [2]   P_t(j) in TMEM, O_t rescaled (4 warp arrivals)
  uint64_t* o_full = p_full + 2;       // [2]   last PV_t complete (tcgen05.commit)
  uint64_t* exp_tok = o_full + 2;      // [2]   exp_tok[t]: the other tile finished an exp phase
  uint64_t* p_half = exp_tok + 2;      // [2]   keys 0-63 of P_t(j) in TMEM, O_t rescaled (4 warp arrivals)
  uint64_t* drain = p_half + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;

  // CTA order: heads are taken in groups of p.group_heads (about one wave of CTAs per group)
  // so the CTAs resident at any time share a few heads' K/V in L2; inside a group the
  // heaviest (last, when causal) q-blocks of every head go first.
  const int BH = p.B * p.H;
  const int per_group = p.group_heads * p.num_qblocks;
  const int grp = (int)(blockIdx.x / per_group);
  const int gbase = grp * p.group_heads;
  const int gsz = min(p.group_heads, BH - gbase);
  const int rem = (int)(blockIdx.x - (unsigned)grp * per_group);
  const int qb = p.num_qblocks - 1 - rem / gsz;
  const int bh = gbase + rem % gsz;
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / p.kv_group;  // K/V head of query head h
  const int q0 = qb * 2 * kTileM;
  const int nkb = (p.N + kBlockN - 1) / kBlockN;
  int nb[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = q0 + t * kTileM;
    if (qs >= p.M) {
      nb[t] = 0;
    } else if (p.causal) {
      const int last = (qs + kTileM - 1) / kBlockN;  // diagonal block (qs is a multiple of 128)
      nb[t] = min(nkb, last + 1);
    } else {
      nb[t] = nkb;
    }
  }
  const int J = max(nb[0], nb[1]);  // key blocks loaded (tile 0 always has rows: nb[0] >= 1)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&p_half[t], 4);
      mbar_init(&o_full[t], 1);
      mbar_init(&exp_tok[t], 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
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
      bool ok = true;
      const int ntiles = nb[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, ntiles * C::kTileBytes);
      for (int t = 0; t < ntiles; ++t)
        for (int x = 0; x < C::kQBoxes; ++x)
          tma_load_4d(sQ + t * C::kTileBytes + x * (kTileM * 128), &tmQ, q_full, 64 * x, q0 + t * kTileM, h, b);
      // Ring order = MMA consumption order: item 2j = K_j, item 2j+1 = V_j.
      const int drop = (p.drop_block == (int)blockIdx.x) ? p.drop_item : -1;
      int issued = 0;
      for (int i = 0; i < 2 * J && ok; ++i) {
        const int slot = i % S;
        const uint32_t par = ((i / S) & 1) ^ 1u;
        if (!mbar_wait(&kv_empty[slot], par, kSiteLoadEmpty)) {
          ok = false;
          break;
        }
        if (i == drop) {  // test hook: this item never arrives, its consumer's wait runs out
          issued = i + 1;
          continue;
        }
        mbar_arrive_expect_tx(&kv_full[slot], C::kTileBytes);
        const CUtensorMap* tm = (i & 1) ? &tmV : &tmK;
        const int row = (i >> 1) * kBlockN;
        uint8_t* dst = sRing + slot * C::kTileBytes;
        for (int x = 0; x < C::kQBoxes; ++x) tma_load_4d(dst + x * (kTileM * 128), tm, &kv_full[slot], 64 * x, row, hk, b);
        issued = i + 1;
      }
      // Teardown: every copy issued must land before the CTA can exit -- also after a failure,
      // so these waits do not give up early when the status word is set.  A ring slot holds at
      // most one unconsumed item, the last S items cover them all.
      mbar_wait_drain(q_full, 0, kSiteTeardown);
      for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
        if (i != drop) mbar_wait_drain(&kv_full[i % S], (i / S) & 1, kSiteTeardown);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs this loop (waits voted, operands warp-uniform) and one elected lane
    // issues each MMA and commit.  With the softmax reduced to bare arrivals, this kernel's MMA
    // sequence ran ~20% faster than as a loop of lane 0 alone, whose issue of 64-cycle MMAs
    // fell behind the tensor pipe.
    {
      bool ok = mbar_wait_warp(q_full, 0, kSiteMmaQ);
      // Descriptors are built once and advanced with sdesc_add inside the issue loops, so an
      // MMA costs the issuing warp a few instructions.
      const uint64_t q_desc[2] = {sdesc_sw128(smem_u32(sQ), 16, 1024), sdesc_sw128(smem_u32(sQ + C::kTileBytes), 16, 1024)};
      const uint64_t ring_k_desc = sdesc_sw128(smem_u32(sRing), 16, 1024);
      const uint64_t ring_v_desc = sdesc_sw128(smem_u32(sRing), kTileM * 128, 1024);
      auto wait_item = [&](int i) { return mbar_wait_warp(&kv_full[i % S], (i / S) & 1, kSiteMmaKV); };
      auto release_item = [&](int i) { tc_commit_warp(&kv_empty[i % S]); };
      // S_t = Q_t K^T : K-major A (Q) and B (K), K = D in steps of 16.
      auto issue_s = [&](int t, int blk) {
        const uint64_t kd = sdesc_add(ring_k_desc, ((2 * blk) % S) * C::kTileBytes);
        const uint32_t d_tmem = tmem + t * kBlockN;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * (kTileM * 128) + (ks & 3) * 32;
          mma_f16_ss_warp(d_tmem, sdesc_add(q_desc[t], off), sdesc_add(kd, off), kIdescS, ks > 0);
        }
        tc_commit_warp(&s_full[t]);
      };
      // O_t (+)= P_t V : A = P_t from TMEM (columns [128t, 128t+64), two keys per column),
      // B = V MN-major from shared memory.
      // Issued in two key halves: keys 0-63 as soon as that half of P is in TMEM.
      auto issue_pv = [&](int t, int blk, int ks0, int ks1) {
        const uint64_t vd = sdesc_add(ring_v_desc, ((2 * blk + 1) % S) * C::kTileBytes);
        const uint32_t o_tmem = tmem + C::kOCol0 + t * D;
        const uint32_t p_tmem = tmem + t * kBlockN;
#pragma unroll
        for (int ks = ks0; ks < ks1; ++ks)
          mma_f16_ts_warp(o_tmem, p_tmem + ks * 8, sdesc_add(vd, ks * 16 * 128), kIdescO, (blk > 0 || ks > 0) ? 1u : 0u);
      };
      // Prologue: S_t(0) for both tiles.
      if (ok && (ok = wait_item(0))) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (nb[t] > 0) issue_s(t, 0);
        release_item(0);
      }
      for (int j = 0; j < J && ok; ++j) {
        if (!wait_item(2 * j + 1)) {  // V_j
          ok = false;
          break;
        }
        tc_fence_after();
        bool k_next = false;  // K_{j+1} is in (and used by this iteration)
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= nb[t]) continue;
          if (!mbar_wait_warp(&p_half[t], j & 1, kSiteMmaP)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, j, 0, kBlockN / 32);
          if (!mbar_wait_warp(&p_full[t], j & 1, kSiteMmaP)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, j, kBlockN / 32, kBlockN / 16);
          if (j + 1 < nb[t]) {
            // In issue order after PV_t(j): overwrites P_t(j) only once PV_t(j) has read it.
            if (!k_next) {
              if (!wait_item(2 * j + 2)) {
                ok = false;
                break;
              }
              tc_fence_after();
              k_next = true;
            }
            issue_s(t, j + 1);
          } else {
            tc_commit_warp(&o_full[t]);
          }
        }
        if (!ok) break;
        release_item(2 * j + 1);
        if (k_next) release_item(2 * j + 2);
      }
      // Every MMA issued must be complete before tensor memory is freed.
      tc_commit_warp(drain);
      mbar_wait_drain(drain, 0, kSiteTeardown);
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 0-7)
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // row inside the tile == TMEM lane
    const int m = q0 + t * kTileM + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_tmem = tmem + lane_off + t * kBlockN;
    const uint32_t o_tmem = tmem + lane_off + C::kOCol0 + t * D;
    const int lim = p.causal ? min(m, p.N - 1) : (p.N - 1);  // last visible key of this row
    float m_used = -INFINITY;  // running max actually used for exp2 (log2-scaled units)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb[t]; ++j) {
      // S_t(j) complete -- and with it PV_t(j-1), issued before it.
      if (!mbar_wait_warp(&s_full[t], j & 1, kSiteSoftS)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[kBlockN];
      const int n0 = j * kBlockN;
      // Tile-uniform: does any row of this tile see a masked key in block j?
      const bool masked_block = (n0 + kBlockN > p.N) || (p.causal && n0 + kBlockN - 1 > q0 + t * kTileM);
#pragma unroll
      for (int c = 0; c < kBlockN / 32; ++c) tmem_ld32(s_tmem + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_wait_ld();
      if (masked_block && n0 + kBlockN - 1 > lim) {
#pragma unroll
        for (int c = 0; c < kBlockN; ++c)
          if (n0 + c > lim) sr[c] = __float_as_uint(-INFINITY);
      }
      const float mx = row_max<kBlockN>(sr);
      const float m_new = mx * p.scale_log2;
      const bool need = m_new > m_used + kRescaleThreshold;
      const bool warp_rescale = __any_sync(0xffffffffu, need) && j > 0;
      float alpha = 1.f;
      if (need) {
        alpha = ex2(m_used - m_new);  // 0 on the first block (m_used = -inf)
        m_used = m_new;
      }
      l *= alpha;
      // The two tiles take turns on the exp phase (tile 0 block j, tile 1 block j, tile 0
      // block j+1, ...): the MUFU pipe runs one tile's exponentials at full rate.  Tile 0
      // block j waits for tile 1's block j-1, tile 1 block j for tile 0's block j (skipped
      // where the other tile has no such block); each tile's turns complete in order, so
      // parities stay one phase apart.
      if (kExpTurns && (t == 0 ? (j >= 1 && j - 1 < nb[1]) : (j < nb[0]))) {
        // Every lane polls the token in lockstep (no vote here: one costs registers in this
        // loop); the waits whose outcome gates tensor-memory access are voted.
        if (!mbar_wait(&exp_tok[t], (t == 0 ? j - 1 : j) & 1, kSiteSoftS)) {
          ok = false;
          break;
        }
      }
      // p = 2^(s * scale * log2e - m_used), packed two per 32-bit word in the input dtype.
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
      const uint64_t ng2 = f2(-m_used, -m_used);
      uint64_t rs2 = f2(0.f, 0.f);
      uint32_t pk[kBlockN / 2];
#pragma unroll
      for (int e = 0; e < kBlockN / 2; ++e) {
        const uint64_t x2 = fma2(f2(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1])), sc2, ng2);
        float x0, x1;
        uf2(x2, x0, x1);
        // One key pair in eight takes its exponentials on the FMA pipe (exp2_poly_pair): with
        // the MMA warp converged this measured 1.5-2.5% faster; larger shares were slower.
        float p0, p1;
        if ((e & 7) == 0) {
          exp2_poly_pair(x0, x1, p0, p1);
        } else {
          p0 = ex2(x0);
          p1 = ex2(x1);
        }
        rs2 = add2(rs2, f2(p0, p1));
        pk[e] = pack2<kBf16>(p0, p1);
        if (e == kBlockN / 4 - 1) {
          // Keys 0-63 of P_t(j) -> columns 0-31 of S_t (this thread's row, two keys per column);
          // the MMA warp starts PV_t(j) on them while the rest are computed.
          tmem_st32(s_tmem, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
          if (warp_rescale) {
            // O_t holds exactly PV_t(0..j-1) (complete since S_t(j) is): rescale it before the
            // first half of PV_t(j) accumulates -- here, where half of S is no longer live.
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t ov[32];
              tmem_ld32(o_tmem + c * 32, ov);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
              tmem_st32(o_tmem + c * 32, ov);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_half[t]);
        }
      }
      if (kExpTurns) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&exp_tok[1 - t]);  // the other tile's turn
      }
      {
        float rs0, rs1;
        uf2(rs2, rs0, rs1);
        l += rs0 + rs1;
      }
      // Keys 64-127 of P_t(j) -> columns 32-63 of S_t.
      tmem_st32(s_tmem + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // Epilogue: O / l -> this warp's 32 rows of the tile's Q buffer (idle now: every MMA that
    // reads Q_t is complete once o_full_t is), 128B-swizzled like a TMA tile, then TMA stores
    // of 64-column x 32-row boxes; rows past M are clipped by the copy.  Row-per-thread global
    // stores would touch 32 cache lines per instruction.
    if (ok && nb[t] > 0) {
      if (mbar_wait_warp(&o_full[t], 0, kSiteSoftO)) {
        tc_fence_after();
        const float inv = 1.f / l;
        if (p.lse != nullptr && m < p.M) {
          // l = sum_n 2^(x_n - m_used) with x = scale * log2(e) * s: ln(sum_n e^(scale * s_n))
          // = (m_used + log2(l)) * ln(2).
          p.lse[(int64_t)(b * p.H + h) * p.lse_ld + m] = (m_used + log2f(l)) * 0.69314718055994531f;
        }
        uint8_t* stage = sQ + t * C::kTileBytes + quad * (32 * 128);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32(o_tmem + c * 32, ov);
          tmem_wait_ld();
          uint8_t* box_row = stage + (c >> 1) * (kTileM * 128) + lane * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack2<kBf16>(__uint_as_float(ov[8 * q + 0]) * inv, __uint_as_float(ov[8 * q + 1]) * inv);
            w.y = pack2<kBf16>(__uint_as_float(ov[8 * q + 2]) * inv, __uint_as_float(ov[8 * q + 3]) * inv);
            w.z = pack2<kBf16>(__uint_as_float(ov[8 * q + 4]) * inv, __uint_as_float(ov[8 * q + 5]) * inv);
            w.w = pack2<kBf16>(__uint_as_float(ov[8 * q + 6]) * inv, __uint_as_float(ov[8 * q + 7]) * inv);
            const int piece = (c & 1) * 4 + q;  // 16-byte piece of the 128-byte box row
            *reinterpret_cast<uint4*>(box_row + ((piece ^ (lane & 7)) << 4)) = w;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        const int row0 = q0 + t * kTileM + quad * 32;
        if (lane == 0 && row0 < p.M) {
          for (int x = 0; x < C::kQBoxes; ++x) tma_store_4d(&tmO, stage + x * (kTileM * 128), 64 * x, row0, h, b);
          bulk_commit_group();
          bulk_wait_group<0>();  // the copy has read shared memory and written O
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}

template <int D, bool kBf16>
int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& to, const Params& p,
           cudaStream_t s) {
  using C = Cfg<D>;
  auto kern = fa_fwd_kernel<D, kBf16>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    configured.fetch_or(bit);
  }
  const int64_t grid = (int64_t)p.num_qblocks * p.B * p.H;
  kern<<<(unsigned)grid, kThreads, C::kSmemBytes, s>>>(tq, tk, tv, to, p);
  return check_launch();
}

int make_map(CUtensorMap* map, bool bf16, const void* base, int64_t B, int64_t H, int64_t S, int64_t D,
             const int64_t* st, uint32_t box_rows) {
  if (st[3] != 1) return LK_ERR_INVALID_ARG;
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {64, box_rows, 1, 1};
  return make_tmap(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims,
                   strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace fa
}  // namespace lk

extern "C" int lk_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int dtype, int64_t B,
                                 int64_t H, int64_t M, int64_t N, int64_t D, const int64_t* q_strides,
                                 const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                 int causal, float softmax_scale, void* stream) {
  return lk_flash_attn_fwd_gqa(q, k, v, o, dtype, B, H, H, M, N, D, q_strides, k_strides, v_strides, o_strides,
                               causal, softmax_scale, stream);
}

namespace lk {
namespace fa {
int forward(const void* q, const void* k, const void* v, void* o, float* lse, int64_t lse_ld, int dtype, int64_t B,
            int64_t H, int64_t H_kv, int64_t M, int64_t N, int64_t D, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides, int causal,
            float softmax_scale, void* stream) {
  if (B < 0 || H < 0 || M < 0 || N < 0) return LK_ERR_INVALID_ARG;
  if (lse != nullptr && lse_ld < M) return LK_ERR_INVALID_ARG;
  if (H > 0 && (H_kv <= 0 || H % H_kv != 0)) return LK_ERR_INVALID_ARG;
  if (B == 0 || H == 0 || M == 0) return LK_OK;
  if (!q || !k || !v || !o || !q_strides || !k_strides || !v_strides || !o_strides || N == 0)
    return LK_ERR_INVALID_ARG;
  if (dtype != LK_BF16 && dtype != LK_F16) return LK_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return LK_ERR_UNSUPPORTED;
  if (M > (1 << 30) || N > (1 << 30) || B * H > (1 << 30)) return LK_ERR_INVALID_ARG;
  if (o_strides[3] != 1 || ((uintptr_t)o & 15)) return LK_ERR_ALIGNMENT;
  for (int i = 0; i < 3; ++i)
    if (o_strides[i] % 8) return LK_ERR_ALIGNMENT;
  const int64_t nqb = (M + 2 * fa::kTileM - 1) / (2 * fa::kTileM);
  if (nqb * B * H > 0x7FFFFFFF) return LK_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = bind_stream(s)) return st;
  const bool bf16 = dtype == LK_BF16;
  CUtensorMap tq, tk, tv;
  if (int st = fa::make_map(&tq, bf16, q, B, H, M, D, q_strides)) return st;
  if (int st = fa::make_map(&tk, bf16, k, B, H_kv, N, D, k_strides)) return st;
  if (int st = fa::make_map(&tv, bf16, v, B, H_kv, N, D, v_strides)) return st;
  CUtensorMap to;  // O: 32-row boxes, one per softmax warp
  if (int st = fa::make_map(&to, bf16, o, B, H, M, D, o_strides, 32)) return st;
  fa::Params p{};
  p.B = (int)B;
  p.H = (int)H;
  p.M = (int)M;
  p.N = (int)N;
  p.num_qblocks = (int)nqb;
  p.kv_group = (int)(H / H_kv);
  {
    // causal: several waves per group, so heavy-first ordering still balances the tail
#ifndef LK_FA_CAUSAL_WAVES
#define LK_FA_CAUSAL_WAVES 3
#endif
    const int64_t g = LK_FA_GROUP_HEADS ? (causal ? LK_FA_CAUSAL_WAVES : 1) * sm_count() / nqb : B * H;
    p.group_heads = (int)(g < 1 ? 1 : (g > B * H ? B * H : g));
  }
  p.causal = causal ? 1 : 0;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_sm = o_strides[2];
  p.lse = lse;
  p.lse_ld = lse_ld;
  {
    const Injection inj = take_injection(LK_INJECT_FA_DROP_LOAD);
    p.drop_block = inj.kind ? inj.block : -1;
    p.drop_item = inj.item;
  }
  if (D == 128)
    return bf16 ? fa::launch<128, true>(tq, tk, tv, to, p, s) : fa::launch<128, false>(tq, tk, tv, to, p, s);
  return bf16 ? fa::launch<64, true>(tq, tk, tv, to, p, s) : fa::launch<64, false>(tq, tk, tv, to, p, s);
}
}  // namespace fa
}  // namespace lk

extern "C" int lk_flash_attn_fwd_gqa(const void* q, const void* k, const void* v, void* o, int dtype, int64_t B,
                                     int64_t H, int64_t H_kv, int64_t M, int64_t N, int64_t D,
                                     const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                     const int64_t* o_strides, int causal, float softmax_scale, void* stream) {
  return lk::fa::forward(q, k, v, o, nullptr, 0, dtype, B, H, H_kv, M, N, D, q_strides, k_strides, v_strides,
                         o_strides, causal, softmax_scale, stream);
}

extern "C" int lk_flash_attn_fwd_lse(const void* q, const void* k, const void* v, void* o, float* lse,
                                     int64_t lse_ld, int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t M,
                                     int64_t N, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                                     const int64_t* v_strides, const int64_t* o_strides, int causal,
                                     float softmax_scale, void* stream) {
  if (!lse && B > 0 && H > 0 && M > 0) return LK_ERR_INVALID_ARG;
  return lk::fa::forward(q, k, v, o, lse, lse_ld, dtype, B, H, H_kv, M, N, D, q_strides, k_strides, v_strides,
                         o_strides, causal, softmax_scale, stream);
}
