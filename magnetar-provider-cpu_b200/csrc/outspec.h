// Where a packed matmul writes its output: one rank's y, or the y of every
// rank of a tensor-parallel group (the all-gather fused into the epilogue).
#pragma once

#include <stdint.h>

namespace mgb {

constexpr int MAX_TP = 8;

// Output element (row, col) of a call goes to y_ranks[r] + row * ldy + col0 +
// col for every r < world (plain call: world 1, y_ranks[0] = y, ldy = n,
// col0 = 0).  With cta_counter set, the call publishes its completion: every
// CTA fences its stores at system scope and counts itself on cta_counter
// (zero before the call); the last one resets it and stores the call's epoch
// with system-scope release into done_ranks[r][rank] for every r.  The epoch
// is `epoch`, or, with epoch_src set (device epochs), *epoch_src + 1 read by
// that last CTA: the rank's epoch word, which its stream-ordered wait advances
// after every call, so a captured sequence of calls publishes fresh epochs on
// every replay.
struct OutSpec {
  float *y_ranks[MAX_TP];
  uint32_t *done_ranks[MAX_TP];
  uint32_t *cta_counter;
  const uint32_t *epoch_src;
  uint64_t ldy, col0;
  uint32_t epoch;
  int world, rank;
};

inline OutSpec plain_out(float *y, uint64_t n) {
  OutSpec o = {};
  o.y_ranks[0] = y;
  o.ldy = n;
  o.col0 = 0;
  o.world = 1;
  o.rank = 0;
  o.cta_counter = nullptr;
  o.epoch_src = nullptr;
  o.epoch = 0;
  return o;
}

// The same destination with its completion left to a later launch.
inline OutSpec without_completion(OutSpec o) {
  o.cta_counter = nullptr;
  return o;
}

// The destination of output rows m0.. (activation rows m0.. of the call).
inline OutSpec rows_from(OutSpec o, uint64_t m0) {
  for (int r = 0; r < o.world; ++r) o.y_ranks[r] += m0 * o.ldy;
  return o;
}

}  // namespace mgb
