// Work schedule of the CTA-pair GEMM (gemm2_tcgen05.cuh): which output tiles, and which K
// range of each, a cluster of two CTAs computes. Plain integer logic shared by the kernel
// (device), the launcher (host) and the host-side tests, which check over a sweep of tile and
// cluster counts that every tile's K range is covered exactly once.
#pragma once

#if defined(__CUDACC__)
#define C3CU_SCHED_HD __host__ __device__ __forceinline__
#else
#define C3CU_SCHED_HD inline
#endif

namespace c3cu {
namespace gemm2 {

// One unit of work: K blocks [kb0, kb1) of output tile `tile`; `split` is the tile's slot in
// the split workspace when the tile runs as two K halves, -1 when it runs whole.
struct Item {
  int tile, kb0, kb1, split;
};

// Work of cluster `c` of `C`: the tiles c, c + C, ... below sk_first (whole waves; all
// tiles when sk_mode is 0), then, with sk_mode 1, K half (c & 1) of tail tile
// sk_first + (c >> 1) for c < 2 * (num_tiles - sk_first). Returns false past the last item.
C3CU_SCHED_HD bool work_item(int i, int c, int C, int num_tiles, int sk_mode, int sk_first,
                             int k_blocks, Item& it) {
  const int t_dp = sk_mode == 1 ? sk_first : num_tiles;
  const int n_dp = t_dp > c ? (t_dp - c + C - 1) / C : 0;
  if (i < n_dp) {
    it = Item{c + i * C, 0, k_blocks, -1};
    return true;
  }
  if (sk_mode != 1 || i != n_dp || c >= 2 * (num_tiles - t_dp)) return false;
  const int kmid = k_blocks / 2;
  const bool hi = (c & 1) != 0;
  it = Item{t_dp + (c >> 1), hi ? kmid : 0, hi ? k_blocks : kmid, c >> 1};
  return true;
}

struct SplitPlan {
  int sk_mode;   // 0: whole tiles round robin; 1: whole waves, then the tail split in K halves
  int sk_first;  // first tail tile (sk_mode 1)
  int clusters;  // clusters to launch (each two CTAs)
};

// The launcher's choice for `tiles` output tiles on at most `clusters` co-resident clusters.
// Split-K tail (automatic variant 0 only, K at least 64 blocks): when the last wave would leave
// at least half of the clusters idle, its tiles run as two K halves on two clusters each. With
// shorter K the fp32 partial exchange costs about as much as a half's main loop. More split
// slots than `split_slots` (the workspace's capacity) fall back to whole tiles. Never launches
// more clusters than there is work for. tiles, clusters >= 1.
inline SplitPlan plan_split(int tiles, int clusters, int k_blocks, int variant, int split_slots) {
  SplitPlan p{0, 0, clusters};
  if (variant == 0 && k_blocks >= 64) {
    const int tail = tiles % clusters;
    if (tail > 0 && 2 * tail <= clusters) {
      p.sk_mode = 1;
      p.sk_first = tiles - tail;
      if (tiles < clusters) p.clusters = 2 * tiles;
    }
  }
  if (p.sk_mode != 0 && p.clusters > split_slots) {
    p.sk_mode = 0;
    p.sk_first = 0;
  }
  if (p.sk_mode == 0 && tiles < p.clusters) p.clusters = tiles;
  return p;
}

}  // namespace gemm2
}  // namespace c3cu
