// Host-side flag arithmetic shared by the ring engines.
#pragma once

#include <cstdint>

namespace mgfa {

// Host-side flag arithmetic of the ring engines: the per-slot use counters and
// the call counter every rank advances identically, and the values a step's
// kernels get from them. RingEngine::run() and RingBwdEngine::backward() take
// their flag values from here, and their static plan() replays the same
// arithmetic without a GPU.
struct RingCounters {
  static constexpr int kSlots = 3;
  uint32_t uses[kSlots] = {0, 0, 0};  // finished uses of each receive slot
  uint32_t calls = 0;                 // transport calls so far

  struct Step {
    int slot, next_slot;       // read at step t (t > 0) / pushed into at step t
    uint32_t credit_target;    // the push waits until the right neighbour released
                               // next_slot this many times
    uint32_t credit_value;     // what this step publishes when it releases slot
    uint32_t tag;              // (owner + 1) | (call << 8) of the shard in flight
  };
  Step step(int t, int owner) const {
    const int s = t % kSlots, sn = (t + 1) % kSlots;
    return {s, sn, uses[sn], uses[s] + 1, uint32_t(owner + 1) | (calls << 8)};
  }
  void finish_step(int t) {
    if (t > 0) uses[t % kSlots] += 1;
  }
  void finish_call() { calls += 1; }
};

}  // namespace mgfa
