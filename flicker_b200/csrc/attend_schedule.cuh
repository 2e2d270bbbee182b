// How one attention call's work items are cut over KV (host side; shared by the launcher, the
// C ABI and the allocation-free entry point).
//
// A work item is two 128-row query tiles of one (batch, head) against all S / 128 KV blocks.
// Items are numbered (batch * H + head) * n_pairs + pair, which also orders their output rows.
// The schedule keeps items [0, n_full) whole, splits the next n_a items s_a ways over KV and the
// remaining ones s_b ways. A split item's pieces write un-normalised fp32 partials (acc, l) that
// a combine pass adds up; without a running max they simply add.
#pragma once

#include <cstddef>

namespace flk {

struct AttendSchedule {
  int n_items = 0;  // B * H * query-tile pairs
  int n_full = 0;   // items [0, n_full) whole
  int n_a = 0;      // items [n_full, n_full + n_a) split s_a ways
  int s_a = 1;
  int s_b = 1;      // items [n_full + n_a, n_items) split s_b ways
  bool split() const { return n_full < n_items; }
  long long units() const {
    return static_cast<long long>(n_full) + static_cast<long long>(n_a) * s_a +
           static_cast<long long>(n_items - n_full - n_a) * s_b;
  }
};

// Every item whole.
AttendSchedule attend_unsplit(int B, int H, int S);
// The schedule a call of this shape uses on a device with `sms` SMs when it has the workspace.
AttendSchedule attend_schedule(int B, int H, int S, int sms);
// Workspace bytes of a schedule's partials (0 when nothing is split).
size_t attend_workspace_bytes(int B, int H, int S, const AttendSchedule& sch);

}  // namespace flk
