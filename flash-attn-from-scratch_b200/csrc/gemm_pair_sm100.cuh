// gemm_pair_sm100.cuh — the GEMM of gemm_sm100.cuh on a CTA pair (cluster of 2, tcgen05
// cta_group::2): output tiles of 256 x 256 per pair, 128 rows per CTA.
//
// Why: with one CTA per 128 x 256 tile every SM streams 16 KB of A and 32 KB of B per 128-byte
// K slice; on a pair each CTA streams only its own 16 KB of A and its 16 KB half of B, and the
// even CTA's single MMA instruction (M=256, N=256) multiplies both halves.  Operand traffic
// per SM (L2 -> SMEM and SMEM -> tensor core) drops by a third for the same work.
//
// Roles per CTA (6 warps, as in the one-CTA kernel):
//   warp 0     TMA producer in BOTH CTAs: each loads its own A rows and its half of B into its
//              own shared memory; completion bytes of both are counted on the EVEN CTA's
//              barrier, on which only the even CTA's producer arrives (announcing both CTAs'
//              bytes) — a remote release-arrive from the peer was measured to serialise the
//              ring (~1200 cycles per slot).
//   warp 1     TMEM owner in both CTAs (pair allocation); MMA issuer in the even CTA only:
//              tcgen05.mma.cta_group::2, then one commit to each CTA's ring-slot barrier and,
//              per tile, to each CTA's accumulator barrier (two plain commits; the peer's
//              barrier is addressed through mapa).
//   warps 2-5  epilogue in both CTAs: each drains its own 128 rows x 256 columns from its TMEM
//              and tells the even CTA (local or remote arrive) when the buffer is free.
// The pair synchronises with barrier.cluster after set-up and before TMEM is released, so no
// CTA exits while its peer may still read its shared memory.  All mbarrier waits are bounded.
//
// Split tail.  When the tiles do not fill a whole number of rounds, the leftover tiles (fewer
// than the pairs) are cut along K into `split` parts, and those parts are every pair's FIRST
// unit, so the partial round trip overlaps the pair's next tile (the accumulator is double
// buffered) instead of ending the kernel.  Per warp slot (32 rows x 256 columns) the parts meet
// in the epilogue: each takes a ticket from an arrival counter; the first split-1 tickets write
// their raw accumulator to a workspace and publish it (one fence, one counter bump); the last
// ticket adds those partials to its own accumulator and runs the op's epilogue.  It waits only
// on parts that already hold a ticket, i.e. are running, so no residency assumption is made;
// it re-zeroes the counters for the next launch.  Integer partial sums are exact, so the int8
// result is bit-identical to the unsplit one.
#pragma once

#include "gemm_sm100.cuh"
#include "quant_common.cuh"

namespace lk {
namespace gemm {

template <Kind kKind, bool kBMN>
struct PairConfig {
  using KT = KindTraits<kKind>;
  static constexpr int kBN = 256;     // pair tile N
  static constexpr int kHalfN = 128;  // B columns held by each CTA
  static constexpr int kBK = kBKBytes / KT::kElemBytes;
  static constexpr int kMmasPerStage = kBK / KT::kMmaK;
  static constexpr int kABytes = kBM * kBKBytes;     // 16 KB
  static constexpr int kBBytes = kHalfN * kBKBytes;  // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 6;
  static constexpr int kBBoxes = kBMN ? (kHalfN * KT::kElemBytes) / 128 : 1;
  static constexpr int kBBoxBytes = kBMN ? kBK * 128 : kBBytes;
  static constexpr int kTmemCols = 2 * kBN;  // double-buffered 256-column accumulator
  static constexpr int kSbStageBytes = 4 * 256 * 4;  // per epilogue warp: the tile's 256 column scales
  // Per epilogue warp: two 2 KB store tiles of 32 rows x 64 bytes (64-byte swizzle) for TMA stores of C.
  static constexpr int kCStageBytes = 4 * 2 * 2048;
  static constexpr int kBarBytes = 512;  // mbarriers, TMEM slot, abort flag
  static constexpr int kSmemBytes = kStages * kStageBytes + kCStageBytes + 1024 + kBarBytes + kSbStageBytes;
  static constexpr uint32_t kIdesc =
      make_idesc(KT::kCFmt, KT::kAFmt, KT::kBFmt, 0u, kBMN ? 1u : 0u, 2u * kBM, (uint32_t)kBN);
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum PairSite : int {
  kSitePairEmpty = 121,
  kSitePairAccEmpty = 122,
  kSitePairFull = 123,
  kSitePairAccFull = 124,
  kSitePairTeardown = 125,
  kSitePairSplit = 126,
  kSitePairRequant = 127,
};

// Bounded wait until *ctr >= target, polling L2 every ~0.1 us (many warps may poll one
// counter); records a timeout at `site` and returns false when it runs out.
__device__ __forceinline__ bool wait_count_sleep(const int* ctr, int target, int site) {
  if (ld_acquire_gpu(ctr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_gpu(ctr) < target) {
    __nanosleep(128);
    if (device_failed()) return false;
    if (globaltimer_ns() - t0 > LK_WAIT_LIMIT_NS) {
      record_failure(kDevTimeout, site);
      return false;
    }
  }
  return true;
}

// The re-quantising epilogue runs two more warps (its second pass, two TMEM quadrants each):
// 8 warps keep two warps per SM sub-partition, so a thread may use up to 255 registers.
__host__ __device__ constexpr int pair_threads(Epi e) { return e == Epi::DequantQuant ? 256 : kThreads; }

struct Unit {
  int tile, kb0, kb1, part;  // part < 0: the whole tile
};

// Units [0, tail units) are the split parts of tiles full_tiles.. (so every pair with one
// starts with it); the rest are the whole tiles 0..full_tiles-1 in raster order.
__device__ __forceinline__ Unit decode_unit(int u, const Params& p, int num_kb) {
  Unit w;
  const int tail_units = p.split > 1 ? (p.num_tiles - p.full_tiles) * p.split : 0;
  if (u >= tail_units) {
    w.tile = u - tail_units;
    w.kb0 = 0;
    w.kb1 = num_kb;
    w.part = -1;
    return w;
  }
  const int v = u;
  const int tail = v / p.split;
  w.part = v - tail * p.split;
  w.tile = p.full_tiles + tail;
  w.kb0 = (int)((int64_t)num_kb * w.part / p.split);
  w.kb1 = (int)((int64_t)num_kb * (w.part + 1) / p.split);
  return w;
}

template <Kind kKind, bool kBMN, Epi kEpi>
__global__ void __launch_bounds__(pair_threads(kEpi), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const Params p) {
  using Cfg = PairConfig<kKind, kBMN>;
  using KT = typename Cfg::KT;
  constexpr int S = Cfg::kStages;
  constexpr int kPairM = 2 * kBM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint8_t* c_stage = smem + S * Cfg::kStageBytes;  // [4 warps][2][32 rows x 64 B], 1024-aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(c_stage + Cfg::kCStageBytes);
  uint64_t* full = bars;               // [S]  (even CTA's copy used) both CTAs' TMA bytes -> MMA
  uint64_t* empty = bars + S;          // [S]  MMA commit -> each CTA's producer
  uint64_t* acc_full = bars + 2 * S;   // [2]  MMA commit -> each CTA's epilogue
  uint64_t* acc_empty = acc_full + 2;  // [2]  (even CTA's copy used) 8 epilogue warps -> MMA
  uint64_t* drain = acc_empty + 2;     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* sb_stage = reinterpret_cast<float*>(c_stage + Cfg::kCStageBytes + Cfg::kBarBytes);  // [4 warps][256]
  // DequantQuant: parked-tile handoff between the pass-1 and pass-2 warps of a TMEM quadrant.
  uint64_t* parked_full = reinterpret_cast<uint64_t*>(c_stage + Cfg::kCStageBytes + 256);  // [4 quads][2 slots]
  uint64_t* parked_empty = parked_full + 8;                                                 // [4 quads][2 slots]

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = (int)(blockIdx.x >> 1);
  const int npairs = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    if (kEpi == Epi::DequantQuant) {
      for (int i = 0; i < 8; ++i) {
        mbar_init(&parked_full[i], 1);
        mbar_init(&parked_empty[i], 1);
      }
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.c_tma) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.K + Cfg::kBK - 1) / Cfg::kBK;
  // Producer state kept to the end of the kernel, where copies are drained after a failure.
  uint32_t issued_mask = 0;       // stages this CTA has loaded into at least once
  uint32_t last_parity_bits = 0;  // phase parity of the last load into each stage
  bool prod_ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < p.num_units && ok; u += npairs) {
        const Unit w = decode_unit(u, p, num_kb);
        int mb, nb;
        tile_coords(w.tile, p.tiles_m, p.tiles_n, mb, nb, p.group_m);
        const int m0 = mb * kPairM + (int)rank * kBM;
        const int n0 = nb * Cfg::kBN + (int)rank * Cfg::kHalfN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, kSitePairEmpty) || *(volatile int*)abort_flag) {
            ok = false;
            break;
          }
          // Only the even CTA arrives, announcing both CTAs' bytes; the peer's copies just
          // complete their bytes on that barrier (its transaction count may dip below zero
          // until the announcement lands, which mbarriers allow).  A remote release-arrive
          // from the peer would wait for its earlier copies and serialise the ring.
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          const uint32_t lbar = pair_leader_addr(&full[stage]);
          const int kx = kb * kBKBytes / KT::kElemBytes;
          tma_load_2d_pair(sA + stage * Cfg::kABytes, &tmA, lbar, kx, m0);
          uint8_t* dstB = sB + stage * Cfg::kBBytes;
          if constexpr (kBMN) {
#pragma unroll
            for (int b = 0; b < Cfg::kBBoxes; ++b)
              tma_load_2d_pair(dstB + b * Cfg::kBBoxBytes, &tmB, lbar, n0 + b * (128 / KT::kElemBytes), kx);
          } else {
            tma_load_2d_pair(dstB, &tmB, lbar, kx, n0);
          }
          issued_mask |= 1u << stage;
          last_parity_bits = (last_parity_bits & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) *(volatile int*)abort_flag = 1;
      prod_ok = ok;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    // The whole warp runs the loop (voted waits) and one elected lane issues each MMA and commit
    // (7-13% faster than a loop of lane 0 alone), except in the re-quantising epilogue's
    // kernel, where lane 0 alone measured 3% faster at 131072 rows under the power cap.
    constexpr bool kWarpIssue = kEpi != Epi::DequantQuant;
    auto wait_bar = [&](uint64_t* bar, uint32_t parity, int site) {
      if constexpr (kWarpIssue)
        return mbar_wait_cluster_warp(bar, parity, site);
      else
        return mbar_wait_cluster(bar, parity, site);
    };
    auto commit = [&](uint32_t bar_cluster) {
      if constexpr (kWarpIssue)
        tc_commit_pair_warp(bar_cluster);
      else
        tc_commit_pair(bar_cluster);
    };
    if (leader && (kWarpIssue || lane == 0)) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int u = pair; u < p.num_units && ok; u += npairs, ++local) {
        const Unit w = decode_unit(u, p, num_kb);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_bar(&acc_empty[acc], acc_phase ^ 1u, kSitePairAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kBN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!wait_bar(&full[stage], phase, kSitePairFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int ks = 0; ks < Cfg::kMmasPerStage; ++ks) {
            const uint64_t adesc = sdesc_sw128(a_base + ks * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (kBMN)
              bdesc = sdesc_sw128(b_base + ks * KT::kMmaK * 128, Cfg::kBBoxBytes, 1024);
            else
              bdesc = sdesc_sw128(b_base + ks * 32, 16, 1024);
            const uint32_t accumulate = (kb != w.kb0) || (ks != 0);
            if constexpr (kKind == Kind::I8 && kWarpIssue)
              mma_i8_ss_pair_warp(d_tmem, adesc, bdesc, Cfg::kIdesc, accumulate);
            else if constexpr (kKind == Kind::I8)
              mma_i8_ss_pair(d_tmem, adesc, bdesc, Cfg::kIdesc, accumulate);
            else if constexpr (kWarpIssue)
              mma_f16_ss_pair_warp(d_tmem, adesc, bdesc, Cfg::kIdesc, accumulate);
            else
              mma_f16_ss_pair(d_tmem, adesc, bdesc, Cfg::kIdesc, accumulate);
          }
          commit(cluster_addr(&empty[stage], 0));
          commit(cluster_addr(&empty[stage], 1));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        commit(cluster_addr(&acc_full[acc], 0));
        commit(cluster_addr(&acc_full[acc], 1));
      }
      if (!ok) *(volatile int*)abort_flag = 1;
      commit(cluster_addr(drain, 0));
      mbar_wait_drain(drain, 0, kSitePairTeardown);
    }
  } else if (kEpi == Epi::DequantQuant && warp >= 6) {
    // ------------------------------------------------------------------ codes (DequantQuant, both)
    // Pass 2 of the re-quantising epilogue; warp 6 serves TMEM quadrants 0-1, warp 7 quadrants
    // 2-3.  Per tile and quadrant: take the parked tile, wait until every tile of its row block
    // has published its row maxima, write the int8 codes and the row scales, hand the slot back.
    // A tile waits only for tiles of its own row block, which the host keeps within 2 * pairs
    // consecutive tiles, so every wait points at work that does not depend on it (and all
    // waits are bounded).
    uint8_t* my_cst = c_stage + (warp - 6) * 4096;
    int cbuf = 0;
    int lt = 0;
    bool ok = true;
    for (int u = pair; u < p.num_units && ok; u += npairs, ++lt) {
      const Unit w = decode_unit(u, p, num_kb);
      int mb, nb;
      tile_coords(w.tile, p.tiles_m, p.tiles_n, mb, nb, p.group_m);
      const int n_base = nb * Cfg::kBN;
      const int slot = lt & 1;
#pragma unroll 1
      for (int qi = 0; qi < 2; ++qi) {
        const int quad = (warp - 6) * 2 + qi;
        const int m_warp = mb * kPairM + (int)rank * kBM + quad * 32;
        const int m = m_warp + lane;
        const bool row_ok = m < p.M;
        if (!mbar_wait_warp(&parked_full[quad * 2 + slot], (lt >> 1) & 1, kSitePairRequant)) {
          ok = false;
          break;
        }
        const uint4* slot_base = p.q_park + (size_t)(blockIdx.x * 4 + quad) * 2048 + slot * 1024;
        // The whole parked row (256 fp16 values) in flight at once, while the row block's
        // maxima are awaited: one L2 round trip per tile and quadrant.
        uint4 pv[32];
        if (m_warp < p.M) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pv[i] = __ldcg(slot_base + i * 32 + lane);
          int g = 1;
          if (lane == 0) g = wait_count_sleep(p.q_slice_ctr + (m_warp >> 5), p.tiles_n, kSitePairRequant) ? 1 : 0;
          if (__shfl_sync(0xffffffffu, g, 0) == 0) {
            ok = false;
            break;
          }
          RowScale rs;
          rs.scale = 0.f;
          rs.rcp = 0.f;
          rs.fast = false;
          if (row_ok) {
            const uint32_t amax = (uint32_t)ld_acquire_gpu(reinterpret_cast<const int*>(p.q_absmax + m));
            rs = make_row_scale(__half2float(__ushort_as_half((unsigned short)amax)));
            if (nb == 0) p.q_scale[m] = rs.scale;
          }
#pragma unroll
          for (int st = 0; st < Cfg::kBN / 64; ++st) {
            const int x0 = n_base + st * 64;
            if (x0 >= p.N) break;
            uint32_t words[16];  // the codes of columns x0 .. x0+63 of this lane's row
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint64_t x2[16];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint4 q = pv[(2 * st + h) * 4 + j];
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
                  x2[4 * j + e] = f2(f.x, f.y);
                }
              }
              uint32_t b[32];
              codes_x2<16>(x2, rs, b);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                words[h * 8 + j] = pack4_codes(b[4 * j], b[4 * j + 1], b[4 * j + 2], b[4 * j + 3]);
            }
            // 32 rows x 64 codes through this warp's store tile (64-byte swizzle) and one TMA
            // store; rows past M and columns past N are clipped by the copy.
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            uint8_t* tile = my_cst + cbuf * 2048;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(tile + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(words[4 * q], words[4 * q + 1], words[4 * q + 2], words[4 * q + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, tile, x0, m_warp);
              bulk_commit_group();
            }
            cbuf ^= 1;
          }
        }
        __syncwarp();  // every parked value of this slot has been read
        if (lane == 0) mbar_arrive(&parked_empty[quad * 2 + slot]);
      }
      if (*(volatile int*)abort_flag) break;
    }
    if (!ok) *(volatile int*)abort_flag = 1;
    if (lane == 0) bulk_wait_group<0>();  // code stores complete before shared memory goes
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (both)
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const int wslot = (int)rank * 4 + quad;  // this warp's 32 rows of the pair tile
    const int nwriters = p.split - 1;
    int* arrive_ctr = p.split_flags;                                    // [tail tiles][8]
    int* ready_ctr = p.split_flags + (p.num_tiles - p.full_tiles) * 8;  // [tail writers][8]
    float* my_sb = sb_stage + (warp - 2) * 256;
    uint8_t* my_cst = c_stage + (warp - 2) * 4096;
    int cbuf = 0;  // next store tile of this warp
    // DequantQuant: this quadrant's ring of two parked fp16 tiles (32 rows x 256 columns each),
    // filled here (pass 1) and drained by the quadrant's codes warp (pass 2).
    uint4* park = (kEpi == Epi::DequantQuant) ? p.q_park + (size_t)(blockIdx.x * 4 + quad) * 2048 : nullptr;
    int local = 0;
    for (int u = pair; u < p.num_units; u += npairs, ++local) {
      const Unit w = decode_unit(u, p, num_kb);
      int mb, nb;
      tile_coords(w.tile, p.tiles_m, p.tiles_n, mb, nb, p.group_m);
      const int m = mb * kPairM + (int)rank * kBM + row_in_tile;
      const int m_warp = m - lane;  // first row of this warp's 32
      const int n_base = nb * Cfg::kBN;
      const bool row_ok = m < p.M;
      float row_scale = 0.f;
      if constexpr (kEpi == Epi::DequantF16 || kEpi == Epi::DequantQuant) {
        row_scale = row_ok ? __ldg(p.sa + m) : 0.f;
        // The tile's column scales go to this warp's shared slice while the MMAs run, so the
        // chunk loop below reads them without a round trip to L2.  (The warp finished reading
        // the previous tile's slice before it got here.)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int n = n_base + i * 32 + lane;
          my_sb[i * 32 + lane] = n < p.N ? __ldg(p.sb + n) : 0.f;
        }
        __syncwarp();
      } else if constexpr (kEpi == Epi::RowRsqrt) {
        if (local == 0) griddep_wait();
        row_scale = row_ok ? __ldcg(p.rstd + m) : 0.f;
      }
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_cluster_warp(&acc_full[acc], acc_phase, kSitePairAccFull)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * Cfg::kBN);
      if constexpr (kEpi == Epi::DequantQuant) {
        // Pass 1 of this tile: dequantise each 32-column chunk, round it to fp16 (writing C if
        // asked), take this row's max magnitude and park the fp16 values in this warp's ring
        // slot (L2-resident); the accumulator goes back to the MMA warp as soon as its last
        // chunk is in registers.  Then publish the row maxima, and write the codes of the
        // PREVIOUS tile (pass 2), whose row block has normally finished its pass 1 by now.
        constexpr int kChunks = Cfg::kBN / 32;
        uint32_t mag2 = 0;  // two fp16 magnitude maxima, packed
        const int slot = local & 1;
        // The codes warp has drained this slot's previous tile.
        if (!mbar_wait_warp(&parked_empty[quad * 2 + slot], ((local >> 1) & 1) ^ 1u, kSitePairRequant)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        uint4* slot_base = park + slot * 1024;
        auto pass1 = [&](int c, const uint32_t(&r)[32]) {
          float v[32];
          chunk_values<kKind, Epi::DequantF16>(r, row_scale, 0, p, my_sb + c * 32, true, v);
          uint32_t hw[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            hw[j] = pack_half2(v[2 * j], v[2 * j + 1]);
            mag2 = __vmaxu2(mag2, hw[j] & 0x7FFF7FFFu);
          }
          // Slot layout [chunk][4][32 lanes] of 16 bytes: each store writes 512 contiguous bytes.
#pragma unroll
          for (int j = 0; j < 4; ++j)
            __stcg(slot_base + (c * 4 + j) * 32 + lane, make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]));
          const int n0 = n_base + c * 32;
          if (p.C != nullptr && row_ok && n0 < p.N) {
            uint16_t* crow = static_cast<uint16_t*>(p.C) + (int64_t)m * p.ldc + n0;
            if (n0 + 32 <= p.N && (p.ldc % 8) == 0 && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0)) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(crow)[j] = make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (n0 + j < p.N) crow[j] = (uint16_t)((j & 1) ? (hw[j >> 1] >> 16) : (hw[j >> 1] & 0xFFFFu));
            }
          }
        };
        {
          uint32_t ra[32], rb[32];
          tmem_ld32(t_row, ra);
          tmem_wait_ld_regs(ra);
#pragma unroll 1
          for (int c = 0; c < kChunks; c += 2) {
            tmem_ld32(t_row + (c + 1) * 32, rb);
            pass1(c, ra);
            tmem_wait_ld_regs(rb);
            if (c + 2 < kChunks) {
              tmem_ld32(t_row + (c + 2) * 32, ra);
            } else {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                if (leader)
                  mbar_arrive(&acc_empty[acc]);
                else
                  mbar_arrive_remote(&acc_empty[acc], 0);
              }
            }
            pass1(c + 1, rb);
            if (c + 2 < kChunks) tmem_wait_ld_regs(ra);
          }
        }
        if (m_warp < p.M) {
          const uint32_t mag = max(mag2 & 0xFFFFu, mag2 >> 16);
          if (row_ok) atomicMax(p.q_absmax + m, mag);
          __syncwarp();
          const bool skip = p.inj_kind == LK_INJECT_REQUANT_SKIP_PUBLISH && p.inj_block == (int)blockIdx.x &&
                            p.inj_item == local && quad == 0;
          if (lane == 0 && !skip) {
            __threadfence();  // the warp's maxima are visible before the count that announces them
            atomicAdd(p.q_slice_ctr + (m_warp >> 5), 1);
          }
        }
        __threadfence_block();  // parked values visible to the codes warp before the handoff
        __syncwarp();
        if (lane == 0) mbar_arrive(&parked_full[quad * 2 + slot]);
        if (*(volatile int*)abort_flag) break;
        continue;
      }
      // Split-tail role of this warp slot: a ticket below nwriters writes its partial, the
      // last ticket finishes the tile.
      const int tail = w.tile - p.full_tiles;
      int ticket = -1;
      if (w.part >= 0) {
        if (lane == 0) ticket = atomicAdd(arrive_ctr + tail * 8 + wslot, 1);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
      }
      const bool writer = ticket >= 0 && ticket < nwriters;
      const bool finisher = ticket >= 0 && !writer;
      bool ok = true;
      if (finisher) {
        for (int wi = 0; wi < nwriters; ++wi) {
          int good = 1;
          if (lane == 0) good = wait_counter_gt(ready_ctr + (tail * nwriters + wi) * 8 + wslot, 0, kSitePairSplit);
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) ok = false;
        }
        __syncwarp();
      }
      const int widx = writer ? tail * nwriters + ticket : 0;

      // One 32-column chunk, its accumulator in r.
      auto process = [&](int c, uint32_t (&r)[32]) {
        if (writer) {
          // Chunk layout [8 x 32 lanes] of uint4: every store instruction writes 512 contiguous bytes.
          uint4* dst = p.split_partial + ((size_t)(widx * 8 + wslot) * 8 + c) * 256 + lane;
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[j * 32] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          return;
        }
        if (!ok) return;
        if (finisher) {
          for (int wi = 0; wi < nwriters; ++wi) {
            const uint4* src =
                p.split_partial + ((size_t)((tail * nwriters + wi) * 8 + wslot) * 8 + c) * 256 + lane;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 q = __ldcg(src + j * 32);
              if constexpr (kKind == Kind::I8) {
                r[4 * j + 0] += q.x;
                r[4 * j + 1] += q.y;
                r[4 * j + 2] += q.z;
                r[4 * j + 3] += q.w;
              } else {
                r[4 * j + 0] = __float_as_uint(__uint_as_float(r[4 * j + 0]) + __uint_as_float(q.x));
                r[4 * j + 1] = __float_as_uint(__uint_as_float(r[4 * j + 1]) + __uint_as_float(q.y));
                r[4 * j + 2] = __float_as_uint(__uint_as_float(r[4 * j + 2]) + __uint_as_float(q.z));
                r[4 * j + 3] = __float_as_uint(__uint_as_float(r[4 * j + 3]) + __uint_as_float(q.w));
              }
            }
          }
        }
        const int n0 = n_base + c * 32;
        if (n0 >= p.N || m_warp >= p.M) return;
        if constexpr (kEpi == Epi::DequantF16) {
          if (p.num_dst > 0 && n0 + 32 <= p.N) {
            // Scatter of a whole chunk: staged in this warp's store tile (same swizzle as the
            // TMA path), then copied out so that every store instruction writes 8 rows x 64
            // contiguous bytes to each destination -- full segments for the NVLink writes.
            uint4 wv[8];
            pack_chunk<kKind, kEpi>(r, row_scale, p, my_sb + c * 32, wv);
            uint8_t* tile = my_cst + cbuf * 2048;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(tile + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = wv[q];
            __syncwarp();
            uint4 pc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int piece = lane + 32 * i, row = piece >> 2, q = piece & 3;
              pc[i] = *reinterpret_cast<const uint4*>(tile + row * 64 + ((q ^ ((row >> 1) & 3)) << 4));
            }
            __syncwarp();  // the tile is free again for the next chunk
#pragma unroll
            for (int d = 0; d < kMaxScatter; ++d) {
              if (d >= p.num_dst) break;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int piece = lane + 32 * i, row = piece >> 2, q = piece & 3;
                if (m_warp + row < p.M)
                  store16_dst(static_cast<uint16_t*>(p.c_dst[d]) + (int64_t)(m_warp + row) * p.ldc + n0 + q * 8, pc[i],
                              p.dst_multimem);
              }
            }
            return;
          }
        }
        if (!p.c_tma) {
          if (row_ok) store_chunk<kKind, kEpi>(r, row_scale, m, n0, p, my_sb + c * 32);
          return;
        }
        // Staged store: each lane writes its row's 64-byte pieces into a 32-row tile (64-byte
        // swizzle: 16-byte piece q of row r at q ^ ((r >> 1) & 3), conflict-free), then lane 0
        // stores the tile with TMA; rows past M and columns past N are clipped by the copy.
        uint4 wv[8];
        pack_chunk<kKind, kEpi>(r, row_scale, p, my_sb + c * 32, wv);
        constexpr int kPieces = (kEpi == Epi::RawI32) ? 2 : 1;  // 64-byte tiles per chunk
        constexpr int kColsPerPiece = (kEpi == Epi::RawI32) ? 16 : 32;
#pragma unroll
        for (int h = 0; h < kPieces; ++h) {
          const int x = n0 + h * kColsPerPiece;
          if (x >= p.N) break;
          if (lane == 0) bulk_wait_group_read<1>();  // the tile's previous store has read it
          __syncwarp();
          uint8_t* tile = my_cst + cbuf * 2048;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(tile + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = wv[h * 4 + q];
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, tile, x, m_warp);
            bulk_commit_group();
          }
          cbuf ^= 1;
        }
      };

      // TMEM loads run one chunk ahead of the processing; the buffer is handed back to the MMA
      // warp as soon as the last chunk is in registers.
      constexpr int kChunks = Cfg::kBN / 32;
      uint32_t ra[32], rb[32];
      tmem_ld32(t_row, ra);
      tmem_wait_ld_regs(ra);
#pragma unroll 1
      for (int c = 0; c < kChunks; c += 2) {
        tmem_ld32(t_row + (c + 1) * 32, rb);
        process(c, ra);
        tmem_wait_ld_regs(rb);
        if (c + 2 < kChunks) {
          tmem_ld32(t_row + (c + 2) * 32, ra);
        } else {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              mbar_arrive(&acc_empty[acc]);
            else
              mbar_arrive_remote(&acc_empty[acc], 0);
          }
        }
        process(c + 1, rb);
        if (c + 2 < kChunks) tmem_wait_ld_regs(ra);
      }
      if (writer) {
        __threadfence();
        __syncwarp();
        const bool skip = p.inj_kind == LK_INJECT_SPLIT_SKIP_PUBLISH && tail == p.inj_item && wslot == 0;
        if (lane == 0 && !skip) atomicAdd(ready_ctr + widx * 8 + wslot, 1);
      }
      if (!ok) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      if (finisher && lane == 0) {
        // Every part holds a ticket and every writer has published its partial: reset for the
        // next launch on this workspace.
        arrive_ctr[tail * 8 + wslot] = 0;
        for (int wi = 0; wi < nwriters; ++wi) ready_ctr[(tail * nwriters + wi) * 8 + wslot] = 0;
      }
      __syncwarp();
      if (*(volatile int*)abort_flag) break;
    }
    if (p.dst_multimem) multimem_release();
    if (lane == 0) bulk_wait_group<0>();  // C stores complete before the CTA's shared memory goes
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the even CTA's MMAs are drained: no peer smem is read after this
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  if (warp == 0 && lane == 0 && (!prod_ok || device_failed())) {
    // After a failure some stages may never have been consumed, and nothing consumes or
    // refills the ring any more.  Copies still in flight must land before their CTA exits.
    // Both CTAs' copies into a stage complete on the even CTA's barrier, whose phase completes
    // once both halves have landed: the even CTA waits for every stage it announced.  A copy
    // the odd CTA issued into a phase the even CTA never announced completes no phase; the
    // grace period covers it (a 16 KB copy lands in microseconds).  No cluster barrier follows:
    // whether a CTA is on this path depends on when it read the status word.
    if (leader)
      for (int s = 0; s < S; ++s)
        if (issued_mask & (1u << s))
          mbar_wait_cluster_drain(&full[s], (last_parity_bits >> s) & 1u, kSitePairTeardown);
    spin_ns(50000);
  }
}

template <Kind kKind, bool kBMN, Epi kEpi>
cudaError_t configure_pair() {
  using Cfg = PairConfig<kKind, kBMN>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<kKind, kBMN, kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  return cudaSuccess;
}

// How many CTA pairs of this kernel the device can hold at once (<= SMs / 2).
template <Kind kKind, bool kBMN, Epi kEpi>
cudaError_t resident_pairs(int num_sms, int* out) {
  using Cfg = PairConfig<kKind, kBMN>;
  if (cudaError_t e = configure_pair<kKind, kBMN, kEpi>()) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms & ~1);
  cfg.blockDim = dim3(pair_threads(kEpi));
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaError_t e = cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<kKind, kBMN, kEpi>, &cfg)) return e;
  *out = n < num_sms / 2 ? n : num_sms / 2;
  return cudaSuccess;
}

// max_pairs > 0 caps the grid (the re-quantising epilogue needs every pair resident at once).
template <Kind kKind, bool kBMN, Epi kEpi>
int launch_pair(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, const Params& p, int num_sms,
                cudaStream_t stream, int max_pairs = 0) {
  using Cfg = PairConfig<kKind, kBMN>;
  auto kern = gemm_pair_kernel<kKind, kBMN, kEpi>;
  if (cudaError_t e = configure_pair<kKind, kBMN, kEpi>()) return (int)e;
  // Every unit (tile or split part) of the first round gets its own pair.
  int pairs = p.num_units < num_sms / 2 ? p.num_units : num_sms / 2;
  if (max_pairs > 0 && pairs > max_pairs) pairs = max_pairs;
  Params pl = p;
  if (p.split > 1 || kEpi == Epi::DequantQuant) {
    const Injection inj =
        take_injection(kEpi == Epi::DequantQuant ? LK_INJECT_REQUANT_SKIP_PUBLISH : LK_INJECT_SPLIT_SKIP_PUBLISH);
    pl.inj_kind = inj.kind;
    pl.inj_block = inj.block;
    pl.inj_item = inj.item;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(pair_threads(kEpi));
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = (kEpi == Epi::RowRsqrt) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return (int)cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmC, pl);
}

}  // namespace gemm
}  // namespace lk
