// peer.cuh — the per-device peer mailbox used by the fused multi-GPU
// reduction: every rank owns a small device buffer that the other ranks map
// through CUDA IPC, so the last block of a reduction kernel can hand its
// partial to every peer over NVLink and collect theirs, with no separate
// collective launch.
#pragma once

#include "mk_common.cuh"
#include "reduce_ops.cuh"

#define MK_MAX_PEERS 8

namespace mk {

// Mailbox layout (one per rank): slots[kMailboxRing][MK_MAX_PEERS] fp64
// partials (by epoch mod kMailboxRing, by source rank), then
// flags[MK_MAX_PEERS] u64 (the last epoch each source rank published).
//
// Why a ring of 4: a call publishes its own epoch e and then folds epoch e-1
// (pipelined form) or e (blocking form).  A peer can publish e+4 only after
// folding e+2, which needs this rank's e+2 partial; this rank publishes e+2 in
// a later kernel than the one that read epoch e.  So slot e mod 4 is never
// overwritten before it has been read.  (A ring of 3 would not do: e+3 needs
// only this rank's e+1, published in the same kernel that still reads e.)
constexpr int kMailboxRing = 4;

struct PeerArgs {
  int world = 0;  // 0: no exchange (single-GPU reduction)
  int rank = 0;
  unsigned long long epoch = 0;  // epoch this call publishes; 0: publishes nothing
  unsigned long long limit = 0;  // bounded-wait budget in SM cycles
  int wait_own = 0;              // blocking form: also fold this call's epoch
  // an earlier pipelined call whose global result this launch writes
  unsigned long long pend_epoch = 0;  // 0: none
  double* pend_out = nullptr;
  int pend_op = 0;
  double pend_init = 0.0;
  double* slots[MK_MAX_PEERS] = {};               // peer p's slot array
  unsigned long long* flags[MK_MAX_PEERS] = {};   // peer p's flag array
};

constexpr size_t kMailboxSlotsBytes = (size_t)kMailboxRing * MK_MAX_PEERS * sizeof(double);
constexpr size_t kMailboxBytes = 4096;

// Arguments of the next exchanging call on the current device: a new epoch,
// plus the pending pipelined result (if any), which this launch completes.
// blocking=false makes this call's result the new pending one (written to
// `out` with `op`/`init` by the next exchanging launch).  Fails when the
// mailbox of this device is not connected.
int peer_args_next(Device* dev, PeerArgs* out, bool blocking, double* res, int op, double init);
// Arguments that complete the pending pipelined result without publishing;
// *has_pending = false when there is none.
int peer_args_complete(Device* dev, PeerArgs* out, bool* has_pending);

namespace peerdev {

using namespace rops;

__device__ __forceinline__ double combine_rt(int op, double a, double b) {
  switch (op) {
    case MK_OP_MUL: return combine<MK_OP_MUL>(a, b);
    case MK_OP_MAX: return combine<MK_OP_MAX>(a, b);
    case MK_OP_MIN: return combine<MK_OP_MIN>(a, b);
    default: return combine<MK_OP_ADD>(a, b);
  }
}

__device__ __forceinline__ double neutral_rt(int op) {
  switch (op) {
    case MK_OP_MUL: return neutral<MK_OP_MUL>();
    case MK_OP_MAX: return neutral<MK_OP_MAX>();
    case MK_OP_MIN: return neutral<MK_OP_MIN>();
    default: return neutral<MK_OP_ADD>();
  }
}

// One thread: write this rank's partial of `peer.epoch` into every rank's
// mailbox over NVLink, then raise this rank's flag in every mailbox.
__device__ __forceinline__ void publish(double mine, const PeerArgs& peer) {
  const int slot = (int)(peer.epoch % kMailboxRing);
  for (int p = 0; p < peer.world; ++p)
    asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(peer.slots[p] + slot * MK_MAX_PEERS + peer.rank),
                 "d"(mine)
                 : "memory");
  __threadfence_system();
  for (int p = 0; p < peer.world; ++p)
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(peer.flags[p] + peer.rank), "l"(peer.epoch) : "memory");
}

// One thread: wait (bounded) for every rank's partial of `epoch` in this
// rank's mailbox and fold them in rank order, so every rank gets the same
// bits.  A rank that never arrives sets ERRBIT_TIMEOUT; what is there is
// folded.
__device__ __forceinline__ double fold(const PeerArgs& peer, unsigned long long epoch, int op, unsigned* err) {
  const unsigned long long* my_flags = peer.flags[peer.rank];
  const double* my_slots = peer.slots[peer.rank] + (int)(epoch % kMailboxRing) * MK_MAX_PEERS;
  const long long t0 = clock64();
  double acc = neutral_rt(op);
  bool late = false;
  for (int q = 0; q < peer.world; ++q) {
    unsigned long long f;
    do {
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(f) : "l"(my_flags + q) : "memory");
      if (f < epoch && (unsigned long long)(clock64() - t0) > peer.limit) {
        late = true;
        break;
      }
    } while (f < epoch);
    double v;
    asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(my_slots + q) : "memory");
    acc = combine_rt(op, acc, v);
  }
  if (late) atomicOr(err, ERRBIT_TIMEOUT);
  return acc;
}

// One thread: finish the pending pipelined result, if the launch carries one.
__device__ __forceinline__ void complete_pending(const PeerArgs& peer, unsigned* err) {
  if (peer.pend_epoch == 0) return;
  const double g = fold(peer, peer.pend_epoch, peer.pend_op, err);
  peer.pend_out[0] = combine_rt(peer.pend_op, peer.pend_init, g);
}

}  // namespace peerdev
}  // namespace mk
