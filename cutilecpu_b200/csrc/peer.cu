// peer.cu — set-up of the peer mailboxes (see peer.cuh).  One process per
// GPU: each rank creates its mailbox, the host side exchanges the CUDA IPC
// handles (torch.distributed all_gather in the Python layer), and every rank
// maps the others' mailboxes.  Epochs start at 1 and only grow; the tagged
// slot ring of peer.cuh needs no resetting and bounds how far ranks may drift.
// The epochs and the pending pipelined results live in the device mailbox
// (peer.cuh: ChannelState), not here.
#include <cstring>
#include <mutex>

#include "peer.cuh"

namespace {

struct Mailbox {
  int world = 0, rank = -1;
  void* local = nullptr;
  void* peers[MK_MAX_PEERS] = {};
  bool opened[MK_MAX_PEERS] = {};
  bool connected = false;
  unsigned long long* trace = nullptr;
  int trace_len = 0;
};

std::mutex g_mu;
Mailbox g_box[64];

}  // namespace

namespace mk {

namespace {

void fill_common(const Mailbox& m, PeerArgs* a) {
  a->world = m.world;
  a->rank = m.rank;
  a->limit = wait_limit_cycles();
  a->trace = m.trace;
  a->trace_len = m.trace_len;
  for (int p = 0; p < m.world; ++p) a->slots[p] = static_cast<unsigned long long*>(m.peers[p]);
}

}  // namespace

int peer_args(Device* dev, int ch, int mode, void* out, int op, double init, PeerArgs* a) {
  std::lock_guard<std::mutex> lk(g_mu);
  Mailbox& m = g_box[dev->id];
  if (!m.connected) return fail(MK_ERR_INVALID, "peer mailbox of this device is not connected (mk_peer_connect)");
  PeerArgs p;
  fill_common(m, &p);
  p.mode = mode;
  p.st = reinterpret_cast<ChannelState*>(static_cast<char*>(m.local) + kChannelStateOffset) + ch;
  p.out = out;
  p.op = op;
  p.init = init;
  *a = p;
  return MK_OK;
}

}  // namespace mk

extern "C" int mk_peer_create(int world, int rank, void* handle_out) {
  MK_ENTRY_DEVICE(dev);
  if (world < 2 || world > MK_MAX_PEERS || rank < 0 || rank >= world)
    return mk::fail(MK_ERR_INVALID, "mk_peer_create: need 2 <= world <= 8 and 0 <= rank < world");
  if (!handle_out) return mk::fail(MK_ERR_INVALID, "mk_peer_create: null handle buffer");
  std::lock_guard<std::mutex> lk(g_mu);
  Mailbox& m = g_box[dev->id];
  if (m.local) return mk::fail(MK_ERR_INVALID, "mk_peer_create: mailbox already exists (mk_peer_destroy first)");
  cudaError_t e = cudaMalloc(&m.local, mk::kMailboxBytes);
  // zeroed and complete before any stream (blocking or not) can use it
  if (e == cudaSuccess) e = cudaMemset(m.local, 0, mk::kMailboxBytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, m.local);
  if (e != cudaSuccess) {
    if (m.local) cudaFree(m.local);
    m.local = nullptr;
    return mk::fail_cuda(e, "mk_peer_create");
  }
  std::memcpy(handle_out, &h, sizeof(h));
  m.world = world;
  m.rank = rank;
  m.connected = false;
  return MK_OK;
}

extern "C" int mk_peer_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int mk_peer_connect(const void* handles) {
  MK_ENTRY_DEVICE(dev);
  std::lock_guard<std::mutex> lk(g_mu);
  Mailbox& m = g_box[dev->id];
  if (!m.local) return mk::fail(MK_ERR_INVALID, "mk_peer_connect: no mailbox (mk_peer_create first)");
  if (!handles) return mk::fail(MK_ERR_INVALID, "mk_peer_connect: null handles");
  const char* hb = static_cast<const char*>(handles);
  for (int p = 0; p < m.world; ++p) {
    if (p == m.rank) {
      m.peers[p] = m.local;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + (size_t)p * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return mk::fail_cuda(e, "mk_peer_connect: cudaIpcOpenMemHandle");
    m.peers[p] = ptr;
    m.opened[p] = true;
  }
  m.connected = true;
  return MK_OK;
}

extern "C" int mk_peer_destroy(void) {
  MK_ENTRY_DEVICE(dev);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_peer_destroy: synchronize");
  std::lock_guard<std::mutex> lk(g_mu);
  Mailbox& m = g_box[dev->id];
  for (int p = 0; p < MK_MAX_PEERS; ++p) {
    if (m.opened[p]) cudaIpcCloseMemHandle(m.peers[p]);
    m.opened[p] = false;
    m.peers[p] = nullptr;
  }
  if (m.local) cudaFree(m.local);
  m = Mailbox();
  return MK_OK;
}

extern "C" int mk_peer_trace(unsigned long long* log_dev, int entries) {
  MK_ENTRY_DEVICE(dev);
  if (entries < 0 || (entries > 0 && !log_dev))
    return mk::fail(MK_ERR_INVALID, "mk_peer_trace: need entries >= 0 and a device buffer of 4*entries u64");
  std::lock_guard<std::mutex> lk(g_mu);
  Mailbox& m = g_box[dev->id];
  if (!m.local) return mk::fail(MK_ERR_INVALID, "mk_peer_trace: no mailbox (mk_peer_create first)");
  m.trace = entries ? log_dev : nullptr;
  m.trace_len = entries;
  return MK_OK;
}
