// Where a packed matmul writes its output: one rank's y, or the y of every
// rank of a tensor-parallel group (the all-gather fused into the epilogue).
#pragma once

#include <stdint.h>

namespace mgb {

constexpr int MAX_TP = 8;

// Output element (row, col) of a call goes to y_ranks[r] + row * ldy + col0 +
// col for every r < world (plain call: world 1, y_ranks[0] = y, ldy = n,
// col0 = 0).  With cta_counter set (a tensor-parallel call), a one-CTA kernel
// after the call's last launch publishes its completion (mgb_tp_publish_kernel):
// it stores the call's epoch into done_ranks[r][rank] for every r.  The epoch
// is `epoch`, or, with epoch_word set (device epochs), *epoch_word + 1, to
// which that kernel also advances *epoch_word: a captured sequence of calls
// then publishes fresh epochs on every replay.  With wait_done set, the kernel that
// reads x first waits (after its griddepcontrol.wait) until every one of
// wait_world ranks has published wait_epoch (0: the value of the epoch word of
// that synchronisation buffer) into wait_done.
struct OutSpec {
  float *y_ranks[MAX_TP];
  uint32_t *done_ranks[MAX_TP];
  uint32_t *cta_counter;
  uint32_t *epoch_word;
  const uint32_t *wait_done;
  uint64_t ldy, col0;
  uint64_t wait_timeout_ns;
  uint32_t epoch, wait_epoch;
  int world, rank, wait_world;
};

inline OutSpec plain_out(float *y, uint64_t n) {
  OutSpec o = {};
  o.y_ranks[0] = y;
  o.ldy = n;
  o.col0 = 0;
  o.world = 1;
  o.rank = 0;
  o.cta_counter = nullptr;
  o.epoch_word = nullptr;
  o.wait_done = nullptr;
  o.epoch = 0;
  return o;
}

// The same call without its input wait (a later launch of a call whose first
// launch waited).
inline OutSpec without_input_wait(OutSpec o) {
  o.wait_done = nullptr;
  return o;
}

// The destination of output rows m0.. (activation rows m0.. of the call).
inline OutSpec rows_from(OutSpec o, uint64_t m0) {
  for (int r = 0; r < o.world; ++r) o.y_ranks[r] += m0 * o.ldy;
  return o;
}

}  // namespace mgb
