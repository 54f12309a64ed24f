// The talker's greedy pick rule on four logits, shared by the codec head's GEMM epilogue and
// the standalone pick kernel (crates/qwen3tts/src/talker.rs:154-189, 940, 971-981).
#pragma once
#include <cstdint>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

// Logits v[0..3] of ids id0 .. id0 + 3 (id0 % 4 == 0) of row j, in the order sample_with_u
// treats them: a banned id (and eos while the row has fewer than min_new frames) becomes -inf;
// then, for every time the row has emitted the id, a finite logit is divided by the penalty
// when positive and multiplied by it otherwise, one f32 operation per occurrence as the
// reference's loop over its history (with repeats) does. (A power of the penalty would round
// differently.) A logit that turns -inf on the way stays -inf, as in the reference, where the
// finiteness test runs before each occurrence.
TTS_DEV void pick_rule4(const PickRule& p, int j, int id0, float v[4]) {
  const int w = id0 >> 5, sh = id0 & 31;  // the 4 ids share one ban word
  const uint32_t ban = p.ban ? p.ban[w] >> sh : 0u;
  const bool young = p.frames && p.frames[j] < p.min_new;
  uint2 c = make_uint2(0u, 0u);
  if (p.counts) c = *reinterpret_cast<const uint2*>(p.counts + (size_t)j * p.vocab + id0);
  const uint32_t k[4] = {c.x & 0xffffu, c.x >> 16, c.y & 0xffffu, c.y >> 16};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (((ban >> i) & 1u) || (young && id0 + i == p.eos)) {
      v[i] = -INFINITY;
    } else if (isfinite(v[i])) {
      float x = v[i];
      for (uint32_t r = 0; r < k[i]; ++r) x = x > 0.f ? __fdiv_rn(x, p.penalty) : x * p.penalty;
      v[i] = x;
    }
  }
}

// Records row j's pick `c` in its history (unless it is eos or outside the vocabulary) and
// counts the row's frame (talker.rs:984-996).
TTS_DEV void pick_record(const PickRule& p, int j, unsigned c) {
  if (p.counts && int(c) != p.eos && c < unsigned(p.vocab)) {
    uint16_t& n = p.counts[(size_t)j * p.vocab + c];
    if (n < 0xffffu) n = uint16_t(n + 1);
  }
  if (p.frames) p.frames[j] += 1;
}

}  // namespace tts
