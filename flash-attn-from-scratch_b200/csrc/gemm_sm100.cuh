// gemm_sm100.cuh — persistent warp-specialised tcgen05 GEMM used by the int8 GEMM+dequant and
// the RMSNorm+Linear ops.
//
//   C[M, N] = epilogue( A[M, K] · B(K, N) )
//
// A is K-major (row-major [M, K]).  B is either K-major (row-major [N, K], a weight) or
// MN-major (row-major [K, N], the reference int8 API's layout); both are legal tcgen05
// operand majors for kind::i8 and kind::f16, so neither needs a transpose pass.
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles:
//   warp 0      TMA producer: streams 128-byte-wide K slices of A and B through a
//               kStages-deep shared-memory ring (128B swizzle, one mbarrier pair per stage).
//   warp 1      TMEM owner + MMA issuer: one elected lane issues tcgen05.mma (M=128, N=BN,
//               K = 32 bytes per instruction) into a double-buffered TMEM accumulator and
//               releases ring slots / publishes finished accumulators with tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld the accumulator (warp w owns TMEM lanes 32*(w%4)..+31,
//               i.e. 32 output rows), apply the op's epilogue in registers and store to HBM.
//               The accumulator buffer is handed back as soon as its last column is in
//               registers, so tile i's epilogue overlaps tile i+1's main loop.
//
// Every mbarrier wait is bounded (lk::mbar_wait); on a failure all roles unwind, in-flight
// TMA copies and MMAs are waited for (bounded), TMEM is freed and the kernel returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <type_traits>

#include "lk_abi.h"
#include "lk_sm100.cuh"

namespace lk {
namespace gemm {

enum class Kind : int { I8 = 0, F16 = 1, BF16 = 2 };
enum class Epi : int {
  DequantF16 = 0,  // C fp16 = fp16((fp32(acc) * sa[m]) * sb[n])
  RawI32 = 1,      // C int32 = acc
  RowRsqrt = 2,    // C (f16/bf16) = rstd[m] * acc; rstd written by the preceding row kernel
  // CTA-pair kernel only: the DequantF16 values, re-quantised per row as quantize_symmetric
  // would quantise the fp16 C (int8 codes through the tmC map, fp32 row scales); C itself is
  // written only when Params::C is set.
  DequantQuant = 3,
};

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  void* C;
  int64_t ldc;
  const float* sa;  // DequantF16
  const float* sb;
  const float* rstd;  // RowRsqrt: per-row rsqrt(mean(x^2)+eps) from the programmatic predecessor
  // CTA-pair kernel only: work units.  Units below full_tiles are whole tiles; the remaining
  // (num_tiles - full_tiles) tail tiles are each cut into `split` K ranges so the last round
  // occupies every pair.  split <= 1 means no split (num_units = num_tiles).
  int full_tiles, split, num_units;
  uint4* split_partial;  // [tail writers][8 warp slots][8 chunks][8][32] partial accumulators
  int c_tma;             // CTA-pair kernel: C is written by TMA stores through the tmC map
  int group_m;           // CTA-pair kernel: M-blocks per raster group
  int* split_flags;      // [tail tiles x 8] arrival counters, then [tail writers x 8] chunk counters
  // Scatter epilogue (DequantF16 only): num_dst > 0 writes every output element to each of
  // c_dst[0 .. num_dst) (each already offset to this GEMM's column block, row pitch ldc)
  // instead of C -- e.g. the replicated outputs of all ranks of a column-sharded layer, peers'
  // buffers mapped into this process over NVLink.
  void* c_dst[8];
  int num_dst;
  int dst_multimem;  // c_dst[0] (num_dst == 1) is an NVLink multicast address: multimem stores
  // Test hooks armed by lk_debug_inject (inj_kind 0, the zero-initialised value, = none):
  // LK_INJECT_GEMM_DROP_LOAD  the one-CTA kernel's CTA inj_block skips its inj_item-th stage load;
  // LK_INJECT_REQUANT_SKIP_PUBLISH  the re-quantising pair kernel: CTA inj_block's quadrant-0
  //                               epilogue warp does not publish its inj_item-th tile's maxima;
  // LK_INJECT_SPLIT_SKIP_PUBLISH  the pair kernel's split-tail writer of leftover tile inj_item,
  //                               warp slot 0, never publishes its partial.
  int inj_kind, inj_block, inj_item;
  // DequantQuant: the row absmax exchange between the tiles of one row (zeroed by the host
  // before every launch) and the row scales.
  uint32_t* q_absmax;  // [M] max |fp16 output| bits of each row, combined with atomicMax
  int* q_slice_ctr;    // [ceil(M / 32)] tiles that have published their absmax, per 32-row slice
  float* q_scale;      // [M] scale = absmax / 127
  uint4* q_park;       // [CTAs][4 warps][2 slots][8 chunks][4][32 lanes] fp16 values of a tile
};
constexpr int kMaxScatter = 8;

constexpr int kBM = 128;
constexpr int kBKBytes = 128;  // one 128-byte swizzle atom of K per stage
constexpr int kThreads = 192;
constexpr int kGroupM = 8;  // tile raster: groups of 8 M-blocks sweep all N-blocks

template <Kind K>
struct KindTraits;
template <>
struct KindTraits<Kind::I8> {
  static constexpr int kElemBytes = 1;
  static constexpr int kMmaK = 32;
  static constexpr uint32_t kCFmt = 2, kAFmt = 1, kBFmt = 1;  // s32 accum, signed int8
};
template <>
struct KindTraits<Kind::F16> {
  static constexpr int kElemBytes = 2;
  static constexpr int kMmaK = 16;
  static constexpr uint32_t kCFmt = 1, kAFmt = 0, kBFmt = 0;  // f32 accum, f16
};
template <>
struct KindTraits<Kind::BF16> {
  static constexpr int kElemBytes = 2;
  static constexpr int kMmaK = 16;
  static constexpr uint32_t kCFmt = 1, kAFmt = 1, kBFmt = 1;  // f32 accum, bf16
};

template <Kind kKind, int BN, bool kBMN>
struct Config {
  using KT = KindTraits<kKind>;
  static constexpr int kBK = kBKBytes / KT::kElemBytes;  // K elements per stage
  static constexpr int kMmasPerStage = kBK / KT::kMmaK;  // = 4
  static constexpr int kABytes = kBM * kBKBytes;         // 16 KB
  static constexpr int kBBytes = BN * kBKBytes;          // 32 KB (BN=256) / 16 KB (BN=128)
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  // MN-major B: boxes of [kBK k-rows x 128 bytes of N]; BN*elem/128 boxes side by side.
  static constexpr int kBBoxes = kBMN ? (BN * KT::kElemBytes) / 128 : 1;
  static constexpr int kBBoxBytes = kBMN ? kBK * 128 : kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
  // Per epilogue warp: one 32-row x 64-byte tile that stages a chunk for the scatter epilogue.
  static constexpr int kScatterStageBytes = 4 * 2048;
  static constexpr int kSmemBytes = kStages * kStageBytes + kScatterStageBytes + 1024 /*align slack*/ +
                                    256 /*barriers*/;
  static constexpr uint32_t kIdesc =
      make_idesc(KT::kCFmt, KT::kAFmt, KT::kBFmt, 0u, kBMN ? 1u : 0u, (uint32_t)kBM, (uint32_t)BN);
  static_assert(kMmasPerStage * KT::kMmaK == kBK, "stage must hold whole MMAs");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Tile raster: groups of `group_m` M-blocks sweep all N-blocks, so a group's A rows stay in
// L2 while every B tile is read once per group.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mb, int& nb, int group_m = kGroupM) {
  const int per_group = group_m * tiles_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gsz = min(tiles_m - first_m, group_m);
  const int r = t - g * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

// Site ids recorded in the status word when a wait runs out.
enum Site : int {
  kSiteProdEmpty = 101,
  kSiteMmaAccEmpty = 102,
  kSiteMmaFull = 103,
  kSiteEpiAccFull = 104,
  kSiteTeardownTma = 105,
  kSiteTeardownMma = 106,
};

// ---- epilogue helpers --------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf162(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Epilogue values of one 32-column chunk of an accumulator row.  `sbp` points at the column
// scales of the chunk (DequantF16 only; global or shared memory); with vec_sb they are read as
// eight 16-byte vectors, otherwise one by one up to column N.
template <Kind kKind, Epi kEpi>
__device__ __forceinline__ void chunk_values(const uint32_t (&r)[32], float row_scale, int n0, const Params& p,
                                             const float* sbp, bool vec_sb, float (&v)[32]) {
  if constexpr (kEpi == Epi::DequantF16) {
    // Bit-exact order of the reference epilogue: (fp32(acc) * sa[m]) * sb[n].
    if (vec_sb) {
      const float4* sb4 = reinterpret_cast<const float4*>(sbp);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 s4 = sb4[j];
        v[4 * j + 0] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[4 * j + 0]), row_scale), s4.x);
        v[4 * j + 1] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[4 * j + 1]), row_scale), s4.y);
        v[4 * j + 2] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[4 * j + 2]), row_scale), s4.z);
        v[4 * j + 3] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[4 * j + 3]), row_scale), s4.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float sbj = (n0 + j < p.N) ? sbp[j] : 0.f;
        v[j] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), row_scale), sbj);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * row_scale;
  }
}

template <Kind kKind, Epi kEpi>
__device__ __forceinline__ uint32_t pack_out2(float a, float b) {
  if constexpr (kEpi == Epi::RowRsqrt && kKind == Kind::BF16)
    return pack_bf162(a, b);
  else
    return pack_half2(a, b);
}

// Stores one 32-column chunk of accumulator row m (columns n0..n0+31) with the op's epilogue.
template <Kind kKind, Epi kEpi>
__device__ __forceinline__ void store_chunk(const uint32_t (&r)[32], float row_scale, int m, int n0, const Params& p,
                                            const float* sbp) {
  const bool full_chunk = (n0 + 32 <= p.N);
  if constexpr (kEpi == Epi::RawI32) {
    int32_t* crow = static_cast<int32_t*>(p.C) + (int64_t)m * p.ldc + n0;
    if (full_chunk && (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        reinterpret_cast<uint4*>(crow)[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) crow[j] = (int32_t)r[j];
    }
  } else {
    float v[32];
    chunk_values<kKind, kEpi>(r, row_scale, n0, p, sbp,
                              full_chunk && ((reinterpret_cast<uintptr_t>(sbp) & 15) == 0), v);
    constexpr bool kBf16Out = (kEpi == Epi::RowRsqrt && kKind == Kind::BF16);
    if constexpr (kEpi == Epi::DequantF16) {
      if (p.num_dst > 0) {
        // Scatter: the chunk is packed once and stored to every destination (16-byte stores
        // where the pitch and every base allow them; the host checks both).
        uint4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w[j] = make_uint4(pack_out2<kKind, kEpi>(v[8 * j], v[8 * j + 1]), pack_out2<kKind, kEpi>(v[8 * j + 2], v[8 * j + 3]),
                            pack_out2<kKind, kEpi>(v[8 * j + 4], v[8 * j + 5]),
                            pack_out2<kKind, kEpi>(v[8 * j + 6], v[8 * j + 7]));
#pragma unroll
        for (int d = 0; d < kMaxScatter; ++d) {
          if (d >= p.num_dst) break;
          uint16_t* drow = static_cast<uint16_t*>(p.c_dst[d]) + (int64_t)m * p.ldc + n0;
          if (full_chunk) {
#pragma unroll
            for (int j = 0; j < 4; ++j) store16_dst(drow + 8 * j, w[j], p.dst_multimem);
          } else {
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) drow[j] = __half_as_ushort(__float2half_rn(v[j]));
          }
        }
        return;
      }
    }
    uint16_t* crow = static_cast<uint16_t*>(p.C) + (int64_t)m * p.ldc + n0;
    if (full_chunk && (p.ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        reinterpret_cast<uint4*>(crow)[j] =
            make_uint4(pack_out2<kKind, kEpi>(v[8 * j], v[8 * j + 1]), pack_out2<kKind, kEpi>(v[8 * j + 2], v[8 * j + 3]),
                       pack_out2<kKind, kEpi>(v[8 * j + 4], v[8 * j + 5]),
                       pack_out2<kKind, kEpi>(v[8 * j + 6], v[8 * j + 7]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (n0 + j >= p.N) continue;
        if constexpr (kBf16Out)
          crow[j] = __bfloat16_as_ushort(__float2bfloat16_rn(v[j]));
        else
          crow[j] = __half_as_ushort(__float2half_rn(v[j]));
      }
    }
  }
}

// The chunk as 16-byte words of the output type (4 for 16-bit outputs, 8 for int32), for a
// staged store.  sbp: 32 scales, 16-byte aligned, zero past column N.
template <Kind kKind, Epi kEpi>
__device__ __forceinline__ void pack_chunk(const uint32_t (&r)[32], float row_scale, const Params& p, const float* sbp,
                                           uint4 (&w)[8]) {
  if constexpr (kEpi == Epi::RawI32) {
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
  } else {
    float v[32];
    chunk_values<kKind, kEpi>(r, row_scale, 0, p, sbp, true, v);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = make_uint4(pack_out2<kKind, kEpi>(v[8 * j], v[8 * j + 1]), pack_out2<kKind, kEpi>(v[8 * j + 2], v[8 * j + 3]),
                        pack_out2<kKind, kEpi>(v[8 * j + 4], v[8 * j + 5]),
                        pack_out2<kKind, kEpi>(v[8 * j + 6], v[8 * j + 7]));
  }
}

// ---- the kernel ---------------------------------------------------------------------------
template <Kind kKind, int BN, bool kBMN, Epi kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  using Cfg = Config<kKind, BN, kBMN>;
  using KT = typename Cfg::KT;
  constexpr int S = Cfg::kStages;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled operand tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint8_t* scatter_stage = smem + S * Cfg::kStageBytes;  // [4 warps][32 rows x 64 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(scatter_stage + Cfg::kScatterStageBytes);
  uint64_t* full = bars;               // [S]  TMA -> MMA
  uint64_t* empty = bars + S;          // [S]  MMA -> TMA (tcgen05.commit)
  uint64_t* acc_full = bars + 2 * S;   // [2]  MMA -> epilogue (tcgen05.commit)
  uint64_t* acc_empty = acc_full + 2;  // [2]  epilogue -> MMA (4 warp arrivals)
  uint64_t* drain = acc_empty + 2;     // [1]  teardown: MMA completion
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (p.K + Cfg::kBK - 1) / Cfg::kBK;
  // Producer state kept to the end of the kernel, where copies are drained after a failure.
  uint32_t issued_mask = 0;       // stages that have received at least one load
  uint32_t last_parity_bits = 0;  // parity of the last load issued into each stage
  bool prod_ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const int drop = (p.inj_kind == LK_INJECT_GEMM_DROP_LOAD && p.inj_block == (int)blockIdx.x) ? p.inj_item : -1;
      int nload = 0;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, p.tiles_m, p.tiles_n, mb, nb);
        const int m0 = mb * kBM, n0 = nb * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          if (*(volatile int*)abort_flag) {
            ok = false;
            break;
          }
          if (nload++ == drop) {  // test hook: this stage never fills, the MMA's wait runs out
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          const int kx = kb * kBKBytes / KT::kElemBytes;  // K element coordinate
          tma_load_2d(sA + stage * Cfg::kABytes, &tmA, &full[stage], kx, m0);
          uint8_t* dstB = sB + stage * Cfg::kBBytes;
          if constexpr (kBMN) {
            // B row-major [K, N]: coordinates (n, k); one box per 128 bytes of N.
#pragma unroll
            for (int b = 0; b < Cfg::kBBoxes; ++b)
              tma_load_2d(dstB + b * Cfg::kBBoxBytes, &tmB, &full[stage], n0 + b * (128 / KT::kElemBytes), kx);
          } else {
            tma_load_2d(dstB, &tmB, &full[stage], kx, n0);
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
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (voted waits); one elected lane issues each MMA and commit.
    // Measured 7-13% faster across the GEMM shapes than a loop of lane 0 alone.
    {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_warp(&acc_empty[acc], acc_phase ^ 1u, kSiteMmaAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_warp(&full[stage], phase, kSiteMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int ks = 0; ks < Cfg::kMmasPerStage; ++ks) {
            // K-major operands advance 32 bytes inside the swizzle atom per MMA-K step.
            const uint64_t adesc = sdesc_sw128(a_base + ks * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (kBMN) {
              // MN-major: each MMA-K step is kMmaK k-rows of 128 bytes.
              bdesc = sdesc_sw128(b_base + ks * KT::kMmaK * 128, Cfg::kBBoxBytes, 1024);
            } else {
              bdesc = sdesc_sw128(b_base + ks * 32, 16, 1024);
            }
            if constexpr (kKind == Kind::I8)
              mma_i8_ss_warp(d_tmem, adesc, bdesc, Cfg::kIdesc, (kb | ks) != 0);
            else
              mma_f16_ss_warp(d_tmem, adesc, bdesc, Cfg::kIdesc, (kb | ks) != 0);
          }
          tc_commit_warp(&empty[stage]);  // ring slot free once these MMAs have read it
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_warp(&acc_full[acc]);
      }
      if (!ok) *(volatile int*)abort_flag = 1;
      // Teardown: wait for every MMA issued by this warp before TMEM is released.
      tc_commit_warp(drain);
      mbar_wait_drain(drain, 0, kSiteTeardownMma);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(t, p.tiles_m, p.tiles_n, mb, nb);
      const int m = mb * kBM + row_in_tile;
      const int n_base = nb * BN;
      const bool row_ok = m < p.M;
      float row_scale = 0.f;
      if constexpr (kEpi == Epi::DequantF16) {
        row_scale = row_ok ? __ldg(p.sa + m) : 0.f;
      } else if constexpr (kEpi == Epi::RowRsqrt) {
        // rstd comes from the row kernel launched just before this grid (programmatic
        // dependent launch): only these epilogue threads wait for it, the TMA/MMA warps
        // start the main loop immediately.
        if (local == 0) griddep_wait();
        row_scale = row_ok ? __ldcg(p.rstd + m) : 0.f;
      }
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, kSiteEpiAccFull)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          // Accumulator fully in registers: hand the TMEM buffer back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        const int n0 = n_base + c * 32;
        if constexpr (kEpi == Epi::DequantF16) {
          const int m_warp = mb * kBM + quad * 32;  // first row of this warp's 32
          if (p.num_dst > 0 && n0 + 32 <= p.N && m_warp < p.M) {
            // Scatter of a whole chunk (the column-sharded layer's fused gather): staged in this
            // warp's tile (64-byte swizzle: piece q of row r at q ^ ((r >> 1) & 3)), then copied
            // out so that every store instruction writes 8 rows x 64 contiguous bytes to each
            // destination -- whole segments for the NVLink writes, where storing each lane's row
            // from registers writes 32 scattered 16-byte pieces.
            uint4 wv[8];
            pack_chunk<kKind, kEpi>(r, row_scale, p, p.sb + n0, wv);
            uint8_t* tile = scatter_stage + (warp - 2) * 2048;
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
            continue;
          }
        }
        if (!row_ok || n0 >= p.N) continue;
        store_chunk<kKind, kEpi>(r, row_scale, m, n0, p, kEpi == Epi::DequantF16 ? p.sb + n0 : nullptr);
      }
      if (*(volatile int*)abort_flag) break;
    }
    if (p.dst_multimem) multimem_release();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
  if (warp == 0 && lane == 0 && (!prod_ok || device_failed())) {
    // After a failure some stages may never have been consumed.  Every other role is done
    // (past the barrier above), so nothing consumes or refills the ring any more: every copy
    // issued lands and completes its stage's phase, and must before the CTA exits.
    for (int s = 0; s < S; ++s)
      if (issued_mask & (1u << s)) mbar_wait_drain(&full[s], (last_parity_bits >> s) & 1u, kSiteTeardownTma);
  }
}

// ---- host side ----------------------------------------------------------------------------
template <Kind kKind, int BN, bool kBMN, Epi kEpi>
int launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const Params& p, int num_sms, cudaStream_t stream) {
  using Cfg = Config<kKind, BN, kBMN>;
  auto kern = gemm_kernel<kKind, BN, kBMN, kEpi>;
  // The dynamic-smem opt-in is per function and per device.
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return (int)e;
    configured.fetch_or(bit);
  }
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  Params pl = p;
  const Injection inj = take_injection(LK_INJECT_GEMM_DROP_LOAD);
  pl.inj_kind = inj.kind;
  pl.inj_block = inj.block;
  pl.inj_item = inj.item;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (kEpi == Epi::RowRsqrt) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, kern, tmA, tmB, pl);
}

}  // namespace gemm
}  // namespace lk
