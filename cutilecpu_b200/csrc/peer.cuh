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

// Per-channel exchange state, kept in the rank's OWN mailbox (peers never
// read it) so that no launch depends on host-side bookkeeping: a launch reads
// the last published epoch E from here, publishes E+1, and the pipelined
// form records where its global result goes; the next launch (or the
// completion kernel) finds that record here.  Launches of the exchanging entry
// points can therefore be captured in a CUDA graph and replayed.
struct PendingResult {
  unsigned long long epoch;  // the epoch this record describes; cleared to 0 once written
  void* out;                 // double* (reduction) or uint32_t* (histogram)
  int op;                    // reduction: operator; histogram: number of bins
  int pad;
  double init;
};
struct ChannelState {
  unsigned long long epoch;  // last epoch this rank published on the channel
  unsigned long long pad;
  PendingResult pend[2];     // by epoch parity: launch E+1 writes pend[(E+1)&1] while pend[E&1] is finished
};

// What a launch does with the channel.
enum : int { XMODE_NONE = 0, XMODE_PIPELINED = 1, XMODE_BLOCKING = 2, XMODE_COMPLETE = 3 };

struct PeerArgs {
  int world = 0;  // 0: no exchange (single-GPU reduction)
  int rank = 0;
  int mode = XMODE_NONE;
  unsigned long long limit = 0;  // bounded-wait budget in SM cycles
  ChannelState* st = nullptr;    // this rank's channel state (device memory)
  // this call's result: where it goes and how it is finished
  void* out = nullptr;
  int op = 0;                    // reduction: operator; histogram: number of bins
  double init = 0.0;
  unsigned long long* slots[MK_MAX_PEERS] = {};   // peer p's slot array
  // optional device-clock trace (mk_peer_trace): 4 u64 per epoch, ring of
  // trace_len entries: [kernel start, last block's exchange start, published,
  // pending result folded]
  unsigned long long* trace = nullptr;
  int trace_len = 0;
};

constexpr size_t kMailboxSlotsBytes = (size_t)kMailboxRing * MK_MAX_PEERS * sizeof(unsigned long long);
constexpr size_t kChannelStateOffset = 2048;  // the local channel states, after the reduction slots

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
static_assert(kMailboxSlotsBytes <= kChannelStateOffset, "reduction slots overlap the channel states");
static_assert(kChannelStateOffset + CH_COUNT * sizeof(ChannelState) <= kHistRegionOffset,
              "channel states overlap the histogram region");

// Arguments of an exchanging launch on the current device (mode, and this
// call's result description).  Reads no per-call host state, so the launch
// may be captured in a graph.  Fails when the mailbox is not connected.
int peer_args(Device* dev, int ch, int mode, void* out, int op, double init, PeerArgs* a);

namespace peerdev {

using namespace rops;

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Trace slot k (0..3) of epoch e, if tracing is on.
__device__ __forceinline__ void stamp(const PeerArgs& peer, unsigned long long e, int k) {
  if (peer.trace) peer.trace[(e % (unsigned long long)peer.trace_len) * 4 + k] = now_ns();
}

// The channel's last published epoch.  Read by thread 0 of every block
// BEFORE its ticket: the increment happens only in the last block, after all
// tickets, so every block of a launch reads the same value.
__device__ __forceinline__ unsigned long long read_epoch(const PeerArgs& peer) {
  unsigned long long e;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(e) : "l"(&peer.st->epoch) : "memory");
  return e;
}

// One thread, at the end of the last block: epoch E+1 is now the channel's
// last published epoch; in the pipelined form, record where its result goes.
__device__ __forceinline__ void finish_epoch(const PeerArgs& peer, unsigned long long e1) {
  if (peer.mode == XMODE_PIPELINED) {
    PendingResult& r = peer.st->pend[e1 & 1];
    r.out = peer.out;
    r.op = peer.op;
    r.init = peer.init;
    __threadfence();
    r.epoch = e1;
  }
  __threadfence();
  peer.st->epoch = e1;
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

// One warp (all 32 lanes): lane p writes this rank's tagged partial of epoch
// e into rank p's mailbox over NVLink (one relaxed 8-byte store each, no
// fence).  `mine` must be the same on every lane.
__device__ __forceinline__ void publish(double mine, const PeerArgs& peer, unsigned long long e) {
  const int lane = threadIdx.x & 31;
  if (lane < peer.world) {
    const unsigned long long w = tag_word(mine, e);
    const int slot = (int)(e % kMailboxRing);
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

// One warp: if epoch e's result is pending (pipelined), fold it and write it.
__device__ __forceinline__ void complete_pending(const PeerArgs& peer, unsigned long long e, unsigned* err) {
  if (e == 0) return;
  PendingResult& r = peer.st->pend[e & 1];
  unsigned long long re;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(re) : "l"(&r.epoch) : "memory");
  if (re != e) return;  // nothing pending (blocking call, or already written)
  const int op = r.op;
  const double g = fold(peer, e, op, err);
  if ((threadIdx.x & 31) == 0) {
    static_cast<double*>(r.out)[0] = combine_rt(op, r.init, g);
    r.epoch = 0;
  }
}

}  // namespace peerdev
}  // namespace mk
