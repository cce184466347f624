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

// Mailbox layout (one per rank): slots[kMailboxRing][MK_MAX_PEERS] u64
// (by epoch mod kMailboxRing, by source rank).  A slot word is a tagged fp64
// partial: the partial's bits with the lowest kTagBits mantissa bits replaced
// by the epoch mod 2^kTagBits.  The word is its own "ready" flag: a reader
// polls its LOCAL slot until the tag equals the epoch it wants, so a writer
// needs one 8-byte store per peer and no fence (an aligned 64-bit store is
// single-copy atomic).
//
// What the tag costs: the low 4 of 52 mantissa bits of each partial.  Every
// fp32-derived value (max, min, identity maps) has those bits zero as an fp64,
// so those reductions stay exact; an fp64 sum partial is truncated by at most
// 2^-48 relative.  +-0 and +-Inf survive (the tag is cleared on decode), and a
// NaN stays a NaN.
//
// Why a ring of 4: a call publishes its own epoch e and then folds epoch e-1
// (pipelined form) or e (blocking form).  A peer can publish e+4 only after
// folding e+2, which needs this rank's e+2 partial; this rank publishes e+2 in
// a later kernel than the one that read epoch e.  So slot e mod 4 is never
// overwritten before it has been read.  (A ring of 3 would not do: e+3 needs
// only this rank's e+1, published in the same kernel that still reads e.)
// With 16 tags and 4 slots, a slot's previous content (epoch e-4) never
// carries epoch e's tag, and the zeroed mailbox (tag 0) matches no epoch
// before the slot is first written (epochs start at 1; slot 0 is first
// written at epoch 4).
constexpr int kMailboxRing = 4;
constexpr int kTagBits = 4;

struct PeerArgs {
  int world = 0;  // 0: no exchange (single-GPU reduction)
  int rank = 0;
  unsigned long long epoch = 0;  // epoch this call publishes; 0: publishes nothing
  unsigned long long limit = 0;  // bounded-wait budget in SM cycles
  int wait_own = 0;              // blocking form: also fold this call's epoch
  // an earlier pipelined call whose global result this launch writes
  unsigned long long pend_epoch = 0;  // 0: none
  void* pend_out = nullptr;           // double* (reduction) or uint32_t* (histogram)
  int pend_op = 0;                    // reduction: operator; histogram: number of bins
  double pend_init = 0.0;
  unsigned long long* slots[MK_MAX_PEERS] = {};   // peer p's slot array
  // optional device-clock trace (mk_peer_trace): 4 u64 per epoch, ring of
  // trace_len entries: [kernel start, last block's exchange start, published,
  // pending result folded]
  unsigned long long* trace = nullptr;
  int trace_len = 0;
};

constexpr size_t kMailboxSlotsBytes = (size_t)kMailboxRing * MK_MAX_PEERS * sizeof(unsigned long long);

// Histogram region of the mailbox, after the reduction slots: u64 words
// hist[kMailboxRing][MK_MAX_PEERS][kHistMaxBins], word = (epoch << 32) | count.
// The full 32-bit epoch is the tag, so the word is again its own flag.
constexpr int kHistMaxBins = 16384;
constexpr size_t kHistRegionOffset = 4096;
constexpr size_t kMailboxBytes =
    kHistRegionOffset + (size_t)kMailboxRing * MK_MAX_PEERS * kHistMaxBins * sizeof(unsigned long long);

// Independent streams of exchanging calls, each with its own epochs and
// pending result.
enum : int { CH_REDUCE = 0, CH_HIST = 1, CH_COUNT = 2 };

// Arguments of the next exchanging call on the current device: a new epoch,
// plus the pending pipelined result (if any), which this launch completes.
// blocking=false makes this call's result the new pending one (written to
// `out` with `op`/`init` by the next exchanging launch).  Fails when the
// mailbox of this device is not connected.
int peer_args_next(Device* dev, int ch, PeerArgs* out, bool blocking, void* res, int op, double init);
// Arguments that complete the pending pipelined result without publishing;
// *has_pending = false when there is none.
int peer_args_complete(Device* dev, int ch, PeerArgs* out, bool* has_pending);

namespace peerdev {

using namespace rops;

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Trace slot k (0..3) of this launch's epoch, if tracing is on.
__device__ __forceinline__ void stamp(const PeerArgs& peer, int k) {
  if (peer.trace && peer.epoch) peer.trace[(peer.epoch % (unsigned long long)peer.trace_len) * 4 + k] = now_ns();
}

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

constexpr unsigned long long kTagMask = (1ull << kTagBits) - 1ull;

__device__ __forceinline__ unsigned long long tag_word(double v, unsigned long long epoch) {
  unsigned long long bits = (unsigned long long)__double_as_longlong(v);
  const bool nan = (bits & 0x7ff0000000000000ull) == 0x7ff0000000000000ull && (bits & 0x000fffffffffffffull);
  if (nan) bits |= 0x0008000000000000ull;  // keep a mantissa bit above the tag: still a NaN after decode
  return (bits & ~kTagMask) | (epoch & kTagMask);
}

__device__ __forceinline__ double untag(unsigned long long w) { return __longlong_as_double((long long)(w & ~kTagMask)); }

// One warp (all 32 lanes): lane p writes this rank's tagged partial of
// `peer.epoch` into rank p's mailbox over NVLink (one relaxed 8-byte store
// each, no fence).  `mine` must be the same on every lane.
__device__ __forceinline__ void publish(double mine, const PeerArgs& peer) {
  const int lane = threadIdx.x & 31;
  if (lane < peer.world) {
    const unsigned long long w = tag_word(mine, peer.epoch);
    const int slot = (int)(peer.epoch % kMailboxRing);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(peer.slots[lane] + slot * MK_MAX_PEERS + peer.rank),
                 "l"(w)
                 : "memory");
  }
}

// One warp: lane q waits (bounded) until rank q's partial of `epoch` is in
// this rank's mailbox (all lanes poll at once), then the partials are folded
// in rank order, so every rank gets the same bits.  Returns the fold on every
// lane.  A rank that never arrives sets ERRBIT_TIMEOUT and is left out.
__device__ __forceinline__ double fold(const PeerArgs& peer, unsigned long long epoch, int op, unsigned* err) {
  const int lane = threadIdx.x & 31;
  const unsigned long long* mine = peer.slots[peer.rank] + (int)(epoch % kMailboxRing) * MK_MAX_PEERS;
  const unsigned long long want = epoch & kTagMask;
  unsigned long long w = 0;
  int ok = 1;
  if (lane < peer.world) {
    const long long t0 = clock64();
    while (true) {
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(mine + lane) : "memory");
      if ((w & kTagMask) == want) break;
      if ((unsigned long long)(clock64() - t0) > peer.limit) {
        ok = 0;
        break;
      }
    }
  }
  double acc = neutral_rt(op);
  bool late = false;
  for (int q = 0; q < peer.world; ++q) {
    const unsigned long long wq = __shfl_sync(0xffffffffu, w, q);
    if (__shfl_sync(0xffffffffu, ok, q)) acc = combine_rt(op, acc, untag(wq));
    else late = true;
  }
  if (late && lane == 0) atomicOr(err, ERRBIT_TIMEOUT);
  return acc;
}

// One warp: finish the pending pipelined result, if the launch carries one.
__device__ __forceinline__ void complete_pending(const PeerArgs& peer, unsigned* err) {
  if (peer.pend_epoch == 0) return;
  const double g = fold(peer, peer.pend_epoch, peer.pend_op, err);
  if ((threadIdx.x & 31) == 0) static_cast<double*>(peer.pend_out)[0] = combine_rt(peer.pend_op, peer.pend_init, g);
}

}  // namespace peerdev
}  // namespace mk
