// peer.cuh — the per-device peer mailbox used by the fused multi-GPU
// reduction: every rank owns a small device buffer that the other ranks map
// through CUDA IPC, so the last block of a reduction kernel can hand its
// partial to every peer over NVLink and collect theirs, with no separate
// collective launch.
#pragma once

#include "mk_common.cuh"

#define MK_MAX_PEERS 8

namespace mk {

// Mailbox layout (one per rank): slots[2][MK_MAX_PEERS] fp64 partials (by
// epoch parity, by source rank), then flags[MK_MAX_PEERS] u64 (the last epoch
// each source rank published).
struct PeerArgs {
  int world = 0;  // 0: no exchange (single-GPU reduction)
  int rank = 0;
  unsigned long long epoch = 0;
  unsigned long long limit = 0;  // bounded-wait budget in SM cycles
  double* slots[MK_MAX_PEERS] = {};               // peer p's slot array
  unsigned long long* flags[MK_MAX_PEERS] = {};   // peer p's flag array
};

constexpr size_t kMailboxSlotsBytes = 2 * MK_MAX_PEERS * sizeof(double);
constexpr size_t kMailboxBytes = 4096;

// Next epoch's arguments for the current device; fails when the mailbox of
// this device is not connected.
int peer_args_next(Device* dev, PeerArgs* out);

}  // namespace mk
