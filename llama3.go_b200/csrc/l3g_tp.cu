// Tensor-parallel exchange set-up: peer receive buffers over NVLink.
#include "l3g_rt.h"


// Tensor-parallel exchange buffer: a receive buffer [2][world][n_emb] of
// {value, epoch} words per rank (zero: no epoch yet), mapped into every other
// rank's address space with CUDA IPC (ranks in other processes) or reached
// through unified addressing with peer access (ranks that are threads of the
// same process); the handles and pointers travel over the model's NCCL
// communicator.  All ranks agree (an NCCL min) on whether every mapping
// succeeded; otherwise the step uses NCCL allreduces instead.  L3G_TP_NCCL=1
// forces the NCCL path.  Collective: every rank creates its workspaces in
// the same order.
int tp_setup(l3g_workspace* ws) {
  l3g_model* m = ws->m;
  const int W = m->world, R = m->rank, ne = m->hp.n_emb;
  const NcclApi* api = nccl();
  if (!api->ok) return l3g_fail(L3G_E_NCCL, "NCCL unavailable");
  const size_t bytes = (size_t)2 * W * ne * 8;
  int ok = W <= MAX_WORLD && !getenv("L3G_TP_NCCL");
  if (ok && (cudaMalloc(&ws->tp_recv, bytes) != cudaSuccess ||
             cudaMemset(ws->tp_recv, 0, bytes) != cudaSuccess))
    ok = 0;
  // per rank: the IPC handle, then its process id and raw device pointer
  // (ranks that are threads of one process use the pointer directly: an
  // IPC handle cannot be opened in the process that exported it)
  constexpr int HI = (int)sizeof(cudaIpcMemHandle_t);
  constexpr int HB = HI + 16;
  std::vector<uint8_t> h((size_t)W * HB, 0);
  if (ok) {
    cudaIpcMemHandle_t a;
    if (cudaIpcGetMemHandle(&a, ws->tp_recv) != cudaSuccess) {
      ok = 0;
    } else {
      const int64_t pid = (int64_t)getpid();
      const uint64_t ptr = (uint64_t)(uintptr_t)ws->tp_recv;
      memcpy(&h[(size_t)R * HB], &a, HI);
      memcpy(&h[(size_t)R * HB + HI], &pid, 8);
      memcpy(&h[(size_t)R * HB + HI + 8], &ptr, 8);
    }
  }
  cudaGetLastError();
  // exchange the handles and agree on `ok`, then on the mappings
  auto agree = [&](int* v) -> int {
    int* d_v = nullptr;
    CUDA_TRY(cudaMalloc(&d_v, 4));
    cudaError_t e = cudaMemcpy(d_v, v, 4, cudaMemcpyHostToDevice);
    ncclResult_t r = ncclSuccess;
    if (e == cudaSuccess) {
      r = api->AllReduce(d_v, d_v, 1, ncclInt32, ncclMin, m->comm, ws->stream);
      e = cudaStreamSynchronize(ws->stream);
    }
    if (e == cudaSuccess) e = cudaMemcpy(v, d_v, 4, cudaMemcpyDeviceToHost);
    cudaFree(d_v);
    if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "tp exchange: %s", cudaGetErrorString(e));
    if (r != ncclSuccess) return l3g_fail(L3G_E_NCCL, "tp exchange: %s", api->GetErrorString(r));
    return L3G_OK;
  };
  {
    uint8_t* d = nullptr;
    CUDA_TRY(cudaMalloc(&d, h.size()));
    cudaError_t e = cudaMemcpy(d, h.data(), h.size(), cudaMemcpyHostToDevice);
    ncclResult_t r = ncclSuccess;
    if (e == cudaSuccess) {
      r = api->AllGather(d + (size_t)R * HB, d, HB, ncclUint8, m->comm, ws->stream);
      e = cudaStreamSynchronize(ws->stream);
    }
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), d, h.size(), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "tp exchange: %s", cudaGetErrorString(e));
    if (r != ncclSuccess) return l3g_fail(L3G_E_NCCL, "tp exchange: %s", api->GetErrorString(r));
  }
  if (int rc = agree(&ok)) return rc;
  int mapped = ok;
  for (int r = 0; r < W && mapped; ++r) {
    if (r == R) {
      ws->tp_peer_recv[r] = ws->tp_recv;
      continue;
    }
    int64_t pid = 0;
    uint64_t ptr = 0;
    memcpy(&pid, &h[(size_t)r * HB + HI], 8);
    memcpy(&ptr, &h[(size_t)r * HB + HI + 8], 8);
    if (pid == (int64_t)getpid()) {  // same process: unified addressing
      int peer_dev = -1;
      cudaPointerAttributes pa{};
      if (cudaPointerGetAttributes(&pa, (void*)(uintptr_t)ptr) == cudaSuccess) peer_dev = pa.device;
      int can = 0;
      if (peer_dev >= 0 && peer_dev != m->device)
        cudaDeviceCanAccessPeer(&can, m->device, peer_dev);
      if (!can) {
        mapped = 0;
        break;
      }
      const cudaError_t pe = cudaDeviceEnablePeerAccess(peer_dev, 0);
      if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) {
        mapped = 0;
        break;
      }
      ws->tp_peer_same_process[r] = true;
      ws->tp_peer_recv[r] = reinterpret_cast<unsigned long long*>((uintptr_t)ptr);
      continue;
    }
    cudaIpcMemHandle_t a;
    memcpy(&a, &h[(size_t)r * HB], HI);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, a, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      mapped = 0;
      break;
    }
    ws->tp_peer_recv[r] = static_cast<unsigned long long*>(p);
  }
  cudaGetLastError();
  if (ok)
    if (int rc = agree(&mapped)) return rc;
  ws->tp_p2p = ok && mapped;
  if (!ws->tp_p2p) {  // the NCCL path: drop whatever was set up
    for (int r = 0; r < MAX_WORLD; ++r) {
      if (ws->tp_peer_recv[r] && ws->tp_peer_recv[r] != ws->tp_recv && !ws->tp_peer_same_process[r])
        cudaIpcCloseMemHandle(ws->tp_peer_recv[r]);
      ws->tp_peer_recv[r] = nullptr;
      ws->tp_peer_same_process[r] = false;
    }
    if (ws->tp_recv) cudaFree(ws->tp_recv);
    ws->tp_recv = nullptr;
  }
  return L3G_OK;
}


// Exchange descriptor of reduction phase `phase` (2 * layer + 0 after Wo,
// + 1 after down) for this rank.
TpExchange tp_exchange(const l3g_workspace* ws, int phase) {
  const l3g_model* m = ws->m;
  TpExchange t{};
  t.world = m->world;
  t.rank = m->rank;
  t.n = m->hp.n_emb;
  t.nphase = 2 * m->hp.n_layers;
  t.phase = phase;
  t.step = ws->d_step;
  for (int r = 0; r < m->world && r < MAX_WORLD; ++r) t.recv[r] = ws->tp_peer_recv[r];
  t.my_recv = ws->tp_recv;
  return t;
}
