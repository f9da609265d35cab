// gemm_split.h — host side of the CTA-pair GEMM's split tail (see gemm_pair_sm100.cuh).
#pragma once

#include <cuda_runtime.h>


#include "gemm_sm100.cuh"

#ifndef LK_GEMM_SPLIT
#define LK_GEMM_SPLIT 1
#endif

namespace lk {
namespace gemm {

// Workspace of the pair kernel's split tail, one per (device, stream): launches on one stream
// never overlap, and each launch that completes leaves its counters zero, so nothing is shared
// between concurrent launches.  Sized for the most tail writers a launch can have (fewer than
// the pairs): 256 KB of partials and 16 counters per pair.  Allocated on first use outside
// stream capture; a launch captured before its stream has a workspace simply runs unsplit.
// A launch that gave up (a bounded wait ran out, recorded in the device status word) can leave
// counters non-zero; lk_clear_device_status re-zeroes the counters of every workspace of the
// device, so split launches after the clear start from clean counters again.
struct SplitWorkspace {
  uint4* partial = nullptr;
  int* flags = nullptr;
  size_t flag_bytes = 0;
};

// Looks up (or, outside stream capture, creates) the workspace of (current device, stream).
// Defined in lk_common.cu: one table for the whole library.
bool split_workspace(cudaStream_t stream, int npairs, SplitWorkspace* out);

// Synchronously zeroes the counters of every split workspace of the current device (the
// device must be idle).  Returns a cudaError_t.
int reset_split_workspaces();

// Splits the tiles left over after whole rounds of `npairs` (all tiles, when there are fewer
// than pairs) along K when that would leave pairs idle and the saved K blocks outweigh the
// partial round trip.  Returns the number of parts (1 = none), at most max_split.
inline int choose_split(int num_tiles, int npairs, int num_kb, int max_split) {
  if (!LK_GEMM_SPLIT) return 1;
  const int tail = num_tiles % npairs;
  if (tail == 0) return 1;
  int s = npairs / tail;
  if (s > max_split) s = max_split;
  // Each part must keep enough K blocks that halving the tail beats writing and re-reading
  // 128 KB of partials per CTA.
  while (s > 1 && num_kb < 8 * s) --s;
  return s;
}

// Fills p.full_tiles / split / num_units (and the workspace) for a pair launch over
// p.num_tiles tiles.  Float accumulators use at most 2 parts, so their sum does not depend on
// which part finishes last.
inline void apply_split(Params& p, int npairs_max, int num_kb, int max_split, cudaStream_t stream) {
  p.full_tiles = p.num_tiles;
  p.split = 1;
  p.num_units = p.num_tiles;
  const int split = choose_split(p.num_tiles, npairs_max, num_kb, max_split);
  SplitWorkspace ws;
  if (split > 1 && split_workspace(stream, npairs_max, &ws)) {
    p.full_tiles = p.num_tiles - p.num_tiles % npairs_max;
    p.split = split;
    p.num_units = p.full_tiles + (p.num_tiles - p.full_tiles) * split;
    p.split_partial = ws.partial;
    p.split_flags = ws.flags;
  }
}

}  // namespace gemm
}  // namespace lk
