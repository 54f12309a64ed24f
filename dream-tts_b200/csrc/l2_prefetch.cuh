// L2 prefetch of the next projection's first weight blocks, issued by a kernel once its own
// stream from HBM is out, so the HBM keeps working through this kernel's epilogue and the next
// kernel's launch (see L2Prefetch).
#pragma once
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

// This CTA's share (CTA `cta` of `ncta`) of the prefetch `pf`, issued by one lane. Blocks are
// dealt round-robin so every CTA issues a few and every range of the next GEMM gets its head.
__device__ __forceinline__ void issue_l2_prefetch(const L2Prefetch& pf, int cta, int ncta) {
  if (!pf.w || pf.depth <= 0 || pf.splits <= 0) return;
  const uint64_t pol = l2_policy_evict_last();
  const int per_tile = pf.splits * pf.depth;
  const int units = pf.tiles * per_tile;
  for (int u = cta; u < units; u += ncta) {
    const int tile = u / per_tile, rem = u % per_tile;
    const int split = rem / pf.depth, d = rem % pf.depth;
    const int kb0 = split * pf.kb_total / pf.splits, kb1 = (split + 1) * pf.kb_total / pf.splits;
    const int kb = kb0 + d;
    if (kb >= kb1) continue;
    l2_prefetch_bulk(pf.w + ((size_t)tile * pf.kb_total + kb) * (128 * 64), 128 * 64 * 2, pol);
  }
}

}  // namespace tts
