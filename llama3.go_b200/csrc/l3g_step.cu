// Host runtime of libl3g: model upload and repack, KV state, workspaces and
// the per-step CUDA graphs, behind the C ABI of include/l3g.h.
//
// One decode step is one CUDA graph: a host->device copy of {token, pos},
// the embed kernel, per layer five kernels (QKV+RoPE+KV-append, split-K
// attention, Wo, up/gate+SwiGLU, down; plus an NCCL all-reduce after Wo and
// down when tensor-parallel), the logits kernel with fused argmax, and a
// device->host copy of the 16-byte result.  Kernels are launched with
// programmatic stream serialization so each one's weight prefetch overlaps
// the tail of its predecessor.
#include "l3g_rt.h"


// Kernel attributes belong to the device (context) they were set on: once
// per device, with that device current.
int setup_kernels() {
  static int rcs[64];
  static std::once_flag onces[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return l3g_fail(L3G_E_CUDA, "kernel attribute set-up: no current device");
  int& rc = rcs[dev];
  std::call_once(onces[dev], [&rc] {
    const int big = 227 * 1024;
    cudaError_t e = cudaSuccess;
    // Every kernel asks for the largest shared-memory carveout: the SM's
    // split is fixed while CTAs are resident, and the next kernel's CTA
    // (programmatic dependent launch) only fits beside the current one when
    // the SM already runs with the maximum shared memory.
#define SETK(k) \
  if (e == cudaSuccess) e = set_max_shared(k, big)
#define SETMV4(P, E, VK)             \
  SETK((k_matvec<P, E, 1, VK>));     \
  SETK((k_matvec<P, E, 2, VK>));     \
  SETK((k_matvec<P, E, 4, VK>));     \
  SETK((k_matvec<P, E, 8, VK>))
#define SETRMS(E)      \
  SETMV4(PRO_RMS, E, 2); \
  SETMV4(PRO_RMS, E, 4); \
  SETMV4(PRO_RMS, E, 8)
    SETMV4(PRO_PREQ, EPI_STORE, 1);
    SETMV4(PRO_PREQ, EPI_PUSH, 1);
    SETRMS(EPI_QKV);
    SETRMS(EPI_SWIGLU);
    SETRMS(EPI_LOGITS);
#undef SETRMS
#undef SETMV4
#define SETCL(k)                                                                   \
  SETK(k);                                                                         \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)
#define SETAT(D, T)                      \
  SETK((k_attention<D, T, 1, false>));   \
  SETK((k_attention<D, T, 2, false>));   \
  SETK((k_attention<D, T, 4, false>));   \
  SETK((k_attention<D, T, 8, false>));   \
  SETCL((k_attention<D, T, 1, true>));   \
  SETCL((k_attention<D, T, 2, true>));   \
  SETCL((k_attention<D, T, 4, true>));   \
  SETCL((k_attention<D, T, 8, true>))
    SETAT(1, float);
    SETAT(2, float);
    SETAT(4, float);
    SETAT(2, __half);
    SETAT(4, __half);
#undef SETAT
#undef SETCL
    SETK(k_topk_final);
    SETK(k_embed);
    SETK(k_advance);
    SETK(k_tp_reduce);
    SETK(k_sample);
    SETK(k_topk_partial);
#undef SETK
    rc = e == cudaSuccess ? 0 : (int)e;
  });
  if (rc) return l3g_fail(L3G_E_CUDA, "kernel attribute set-up: %s", cudaGetErrorString((cudaError_t)rc));
  return L3G_OK;
}

// Eager profiling launches every kernel fully serialized (no programmatic
// dependent launch) so CUDA events between kernels time each one alone.
static thread_local bool g_serialize = false;

template <typename... KArgs, typename... Args>
static cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                          size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_serialize ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}



void ws_release(l3g_workspace* ws) {
  for (auto& g : ws->graphs) cudaGraphExecDestroy(g.exec);
  ws->graphs.clear();
  for (int r = 0; r < MAX_WORLD; ++r) {
    if (ws->tp_peer_recv[r] && ws->tp_peer_recv[r] != ws->tp_recv && !ws->tp_peer_same_process[r])
      cudaIpcCloseMemHandle(ws->tp_peer_recv[r]);
    ws->tp_peer_recv[r] = nullptr;
  }
  void* tp_ptrs[] = {ws->d_step, ws->d_sync, ws->tp_recv, ws->d_bar};
  for (void* p : tp_ptrs)
    if (p) cudaFree(p);
  void* dptrs[] = {ws->d_io, ws->d_res, ws->d_gather, ws->x[0], ws->x[1], ws->y, ws->q,
                   ws->attn, ws->act, ws->attn_d, ws->attn_q, ws->act_d, ws->act_q, ws->logits, ws->logits_full, ws->part_o, ws->part_ml,
                   ws->att_cnt, ws->am_val, ws->am_idx, ws->am_cnt, ws->tk_part,
                   ws->d_tk_ids, ws->d_tk_logits, ws->d_tokens, ws->d_trace, ws->d_samp};
  for (void* p : dptrs)
    if (p) cudaFree(p);
  void* pf[] = {ws->pf_ids, ws->pf_x, ws->pf_y, ws->pf_qkv, ws->pf_q, ws->pf_att, ws->pf_ug,
                ws->pf_act, ws->pf_part, ws->attf_scores, ws->attf_pmax, ws->attf_psum,
                ws->attf_po};
  for (void* p : pf)
    if (p) cudaFree(p);
  void* hptrs[] = {ws->h_io, ws->h_res, ws->h_logits, ws->h_tk_ids, ws->h_tk_logits, ws->h_samp};
  for (void* p : hptrs)
    if (p) cudaFreeHost(p);
  if (ws->stream) cudaStreamDestroy(ws->stream);
}

void ws_clear_device_error(l3g_workspace* ws) {
  cudaMemset(ws->d_res, 0, sizeof(Result));
  if (ws->att_cnt) cudaMemset(ws->att_cnt, 0, (size_t)ws->att_cnt_n * 4);
  if (ws->am_cnt) cudaMemset(ws->am_cnt, 0, 4);
}

void ws_detach(l3g_workspace* ws) {
  for (auto& g : ws->graphs) cudaGraphExecDestroy(g.exec);
  ws->graphs.clear();
  ws->m = nullptr;
}

extern "C" void l3g_workspace_free(l3g_workspace* ws) {
  if (!ws) return;
  if (ws->m) {
    std::lock_guard<std::mutex> lk(ws->m->ws_mu);
    auto& v = ws->m->workspaces;
    v.erase(std::remove(v.begin(), v.end(), ws), v.end());
  }
  cudaSetDevice(ws->device);
  ws_release(ws);
  delete ws;
}
// Cluster merge of the attention splits: 16 splits per kv head as one
// thread-block cluster, used when clusters for every local kv head can be
// resident at once (a 148-SM B200 holds at most 7) and the global merge
// would need 32 or more splits per kv head (4 or fewer kv heads per rank:
// TP2 and up), where its wait and merge over that many partials grow (TP8
// tail 11.8 vs 5.2 us).  With 8 kv heads the distributed global merge keeps
// one CTA per SM streaming.  L3G_ATT_CLUSTER=0 forces the global merge, =N
// (2..16) clusters of N whenever they fit.
template <int DPL, typename KT>
static void max_attention_clusters(const l3g_workspace* ws, int cs, int* n) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ws->m->hkv_l, cs);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = ws->att_smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = cs;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (ws->att_gp) {
    case 1: e = cudaOccupancyMaxActiveClusters(n, k_attention<DPL, KT, 1, true>, &cfg); break;
    case 2: e = cudaOccupancyMaxActiveClusters(n, k_attention<DPL, KT, 2, true>, &cfg); break;
    case 4: e = cudaOccupancyMaxActiveClusters(n, k_attention<DPL, KT, 4, true>, &cfg); break;
    case 8: e = cudaOccupancyMaxActiveClusters(n, k_attention<DPL, KT, 8, true>, &cfg); break;
    default: e = cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    *n = 0;
  }
}

static void choose_attention_cluster(l3g_workspace* ws) {
  const l3g_model* m = ws->m;
  ws->att_cluster = 0;
  const char* env = getenv("L3G_ATT_CLUSTER");
  const int knob = env ? atoi(env) : (m->nsm / m->hkv_l >= 32 ? 16 : 0);
  if (knob <= 0) return;
  const int cs = knob >= 2 && knob <= 16 ? knob : 16;
  int n = 0;
  const int dpl = m->hd / 32;
  if (m->kv_f16) {
    if (dpl == 2) max_attention_clusters<2, __half>(ws, cs, &n);
    if (dpl == 4) max_attention_clusters<4, __half>(ws, cs, &n);
  } else {
    if (dpl == 1) max_attention_clusters<1, float>(ws, cs, &n);
    if (dpl == 2) max_attention_clusters<2, float>(ws, cs, &n);
    if (dpl == 4) max_attention_clusters<4, float>(ws, cs, &n);
  }
  if (n < m->hkv_l) return;
  ws->att_cluster = cs;
  ws->n_splits = cs;
  return;
}

extern "C" int l3g_workspace_new(l3g_model* m, int32_t ctx, int32_t topk, l3g_workspace** out) {
  if (!m || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  if (ctx <= 0) ctx = m->hp.ctx_len;  // workspace.go:36-41
  if (ctx > m->hp.ctx_len) ctx = m->hp.ctx_len;
  if (topk <= 0) topk = 40;           // workspace.go:42-44
  if (topk > MAX_TOPK) return l3g_fail(L3G_E_INVALID, "top_k %d above %d", topk, MAX_TOPK);
  CUDA_TRY(cudaSetDevice(m->device));
  auto* ws = new l3g_workspace();
  ws->m = m;
  ws->ctx = ctx;
  ws->topk = topk;
  const int ne = m->hp.n_emb, hd = m->hd;
  const int G = m->group;
  const size_t es = m->kv_f16 ? 2 : 4;
  // attention geometry: splits fill the SMs; a stage holds the interleaved
  // K|V rows of P positions, one ~32 KB bulk copy; four or six stages in flight
  // (a power of two, so stages start at multiples of P that divide KV_PAGE)
  ws->att_P = NW;
  while (ws->att_P * 2 <= std::min(KV_PAGE, (int)(32768 / (2 * hd * es)))) ws->att_P *= 2;
  ws->att_stage = 2 * ws->att_P * hd * (int)es;
  // four stages in flight (measured 428 vs 418 tok/s for three at one GPU);
  // six under tensor parallelism, where fewer CTAs stream a rank's heads
  // (541 vs 527 tok/s at two GPUs)
  ws->att_ns = m->world > 1 ? 6 : 4;
  if (const char* e = getenv("L3G_ATT_STAGES")) {  // ring depth override, 2..6 stages
    const int v = atoi(e);
    if (v >= 2 && v <= 6) ws->att_ns = v;
  }
  ws->att_gp = 1;
  while (ws->att_gp < G) ws->att_gp <<= 1;
  ws->n_splits = std::max(1, std::min(m->nsm / m->hkv_l, (ctx + ws->att_P - 1) / ws->att_P));
  const int scratch = std::max(at_scratch_floats(G, hd) * 4, NW * align_up(ws->n_splits, 32) * 4);
  ws->att_smem = at_ring_offset() + std::max(ws->att_ns * ws->att_stage, scratch);
  choose_attention_cluster(ws);
  const int vloc = m->v_l;
  ws->tk_chunks = (m->v_l * m->world + TOPK_CHUNK - 1) / TOPK_CHUNK;
  cudaError_t e = cudaStreamCreateWithFlags(&ws->stream, cudaStreamNonBlocking);
#define DM(p, bytes) \
  if (e == cudaSuccess) e = cudaMalloc(&(p), (bytes))
#define HM(p, bytes) \
  if (e == cudaSuccess) e = cudaMallocHost(&(p), (bytes))
  DM(ws->d_io, 16);
  HM(ws->h_io, 16);
  DM(ws->d_res, sizeof(Result));
  HM(ws->h_res, sizeof(Result));
  DM(ws->d_gather, sizeof(Result) * m->world);
  DM(ws->x[0], ne * 4);
  DM(ws->x[1], ne * 4);
  DM(ws->y, ne * 4);
  DM(ws->q, (size_t)m->hq_l * hd * 4);
  DM(ws->attn, (size_t)m->hq_l * hd * 4);
  DM(ws->act, (size_t)m->ff_l * 4);
  DM(ws->attn_d, (size_t)m->hq_l * hd / 32 * 4);
  DM(ws->attn_q, (size_t)m->hq_l * hd);
  DM(ws->act_d, (size_t)m->ff_l / 32 * 4);
  DM(ws->act_q, (size_t)m->ff_l);
  DM(ws->logits, (size_t)vloc * 4);
  DM(ws->logits_full, (size_t)vloc * m->world * 4);
  HM(ws->h_logits, (size_t)vloc * m->world * 4);
  // partials for the per-kernel step's splits or the persistent kernel's
  // (at most one CTA per SM each)
  const int part_splits = std::max(ws->n_splits, std::max(1, m->nsm / m->hkv_l));
  DM(ws->part_o, (size_t)m->hkv_l * part_splits * G * hd * 4);
  DM(ws->part_ml, (size_t)m->hkv_l * part_splits * G * 2 * 4);
  ws->att_cnt_n = m->hkv_l * 2;  // arrivals, departures
  DM(ws->att_cnt, (size_t)ws->att_cnt_n * 4);
  DM(ws->am_val, (size_t)m->nsm * 4);
  DM(ws->am_idx, (size_t)m->nsm * 4);
  DM(ws->am_cnt, 4);
  DM(ws->tk_part, (size_t)ws->tk_chunks * MAX_TOPK * 8);
  DM(ws->d_tokens, (size_t)ctx * 4);
  DM(ws->d_trace, kTraceBytes);
  HM(ws->h_samp, sizeof(SampleParams));
  DM(ws->d_samp, sizeof(SampleParams));
  DM(ws->d_step, 4);
  if (e == cudaSuccess) e = cudaMemset(ws->d_step, 0, 4);
  DM(ws->d_sync, 4);
  if (e == cudaSuccess) e = cudaMemset(ws->d_sync, 0, 4);
  DM(ws->d_tk_ids, MAX_TOPK * 4);
  DM(ws->d_tk_logits, MAX_TOPK * 4);
  HM(ws->h_tk_ids, MAX_TOPK * 4);
  HM(ws->h_tk_logits, MAX_TOPK * 4);
#undef DM
#undef HM
  if (e == cudaSuccess) e = cudaMemset(ws->d_res, 0, sizeof(Result));
  if (e == cudaSuccess) e = cudaMemset(ws->att_cnt, 0, (size_t)ws->att_cnt_n * 4);
  if (e == cudaSuccess) e = cudaMemset(ws->am_cnt, 0, 4);
  if (e == cudaSuccess) e = cudaMemset(ws->x[0], 0, ne * 4);
  if (e == cudaSuccess) e = cudaMemset(ws->x[1], 0, ne * 4);
  if (e == cudaSuccess) {
    // logits shards beyond the vocabulary stay -inf
    std::vector<float> ninf((size_t)vloc * m->world, -INFINITY);
    e = cudaMemcpy(ws->logits, ninf.data(), (size_t)vloc * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(ws->logits_full, ninf.data(), ninf.size() * 4, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    ws_release(ws);
    delete ws;
    return l3g_fail(L3G_E_CUDA, "workspace allocation: %s", cudaGetErrorString(e));
  }
  ws->device = m->device;
  if (m->world > 1) {
    const int rc = tp_setup(ws);
    if (rc) {
      ws_release(ws);
      delete ws;
      return rc;
    }
  }
  {
    const int rc = persist_setup(ws);  // after tp_setup: needs the exchange's state
    if (rc) {
      ws_release(ws);
      delete ws;
      return rc;
    }
  }
  {
    std::lock_guard<std::mutex> lk(m->ws_mu);
    m->workspaces.push_back(ws);
  }
  *out = ws;
  return L3G_OK;
}

// grid / launch helpers -------------------------------------------------------
static MatvecArgs mv_args(const DevMat& w) {
  MatvecArgs a{};
  a.w = w.t;
  a.wait_ns = WAIT_TIMEOUT_NS;
  a.nstages = w.nstages;
  a.row_lo = 0;
  a.row_hi = w.t.rows;
  return a;
}

// float4 per thread of a PRO_RMS input row of `cols` values (a power of two)
static int rms_vk(int cols) {
  int vk = 2;
  while (vk * 1024 < cols) vk <<= 1;
  return vk;
}

template <int PRO, int EPI, int RPW>
static cudaError_t launch_mv_r(const DevMat& w, const MatvecArgs& a, dim3 grid, cudaStream_t st) {
  if constexpr (PRO == PRO_RMS) {
    switch (rms_vk(w.t.cols)) {
      case 2: return launch(k_matvec<PRO, EPI, RPW, 2>, grid, dim3(NTHREADS), (size_t)w.smem, st, a);
      case 4: return launch(k_matvec<PRO, EPI, RPW, 4>, grid, dim3(NTHREADS), (size_t)w.smem, st, a);
      case 8: return launch(k_matvec<PRO, EPI, RPW, 8>, grid, dim3(NTHREADS), (size_t)w.smem, st, a);
      default: return cudaErrorInvalidValue;
    }
  } else {
    return launch(k_matvec<PRO, EPI, RPW, 1>, grid, dim3(NTHREADS), (size_t)w.smem, st, a);
  }
}

template <int PRO, int EPI>
static cudaError_t launch_mv(const DevMat& w, const MatvecArgs& a, int nsm, cudaStream_t st) {
  const int gl = a.row_lo / w.t.wr;
  const int ng = (a.row_hi + w.t.wr - 1) / w.t.wr - gl;
  const dim3 grid(std::max(1, std::min(ng, nsm)));
  switch (w.t.wr / NW) {
    case 1: return launch_mv_r<PRO, EPI, 1>(w, a, grid, st);
    case 2: return launch_mv_r<PRO, EPI, 2>(w, a, grid, st);
    case 4: return launch_mv_r<PRO, EPI, 4>(w, a, grid, st);
    case 8: return launch_mv_r<PRO, EPI, 8>(w, a, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

// Launch with programmatic dependent launch and, when cluster_y > 0, thread
// block clusters of (1, cluster_y, 1).
template <typename... KArgs, typename... Args>
static cudaError_t launch_cl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, int cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (!g_serialize) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int DPL, typename KT, bool CL>
static cudaError_t launch_attention_c(int gp, const AttnArgs& a, cudaStream_t st, dim3 grid,
                                      size_t smem, int cluster_y) {
  switch (gp) {
    case 1: return launch_cl(k_attention<DPL, KT, 1, CL>, grid, dim3(NTHREADS), smem, st, cluster_y, a);
    case 2: return launch_cl(k_attention<DPL, KT, 2, CL>, grid, dim3(NTHREADS), smem, st, cluster_y, a);
    case 4: return launch_cl(k_attention<DPL, KT, 4, CL>, grid, dim3(NTHREADS), smem, st, cluster_y, a);
    case 8: return launch_cl(k_attention<DPL, KT, 8, CL>, grid, dim3(NTHREADS), smem, st, cluster_y, a);
    default: return cudaErrorInvalidValue;
  }
}

template <int DPL, typename KT>
static cudaError_t launch_attention_g(const l3g_workspace* ws, const AttnArgs& a, cudaStream_t st,
                                      dim3 grid, size_t smem) {
  if (ws->att_cluster)
    return launch_attention_c<DPL, KT, true>(ws->att_gp, a, st, grid, smem, ws->att_cluster);
  return launch_attention_c<DPL, KT, false>(ws->att_gp, a, st, grid, smem, 0);
}

static cudaError_t launch_attention(const l3g_workspace* ws, const AttnArgs& a, cudaStream_t st) {
  const l3g_model* m = ws->m;
  dim3 grid(m->hkv_l, ws->n_splits);
  const int dpl = m->hd / 32;
  const size_t smem = ws->att_smem;
  if (m->kv_f16) {
    if (dpl == 2) return launch_attention_g<2, __half>(ws, a, st, grid, smem);
    if (dpl == 4) return launch_attention_g<4, __half>(ws, a, st, grid, smem);
    return cudaErrorInvalidValue;
  }
  if (dpl == 1) return launch_attention_g<1, float>(ws, a, st, grid, smem);
  if (dpl == 2) return launch_attention_g<2, float>(ws, a, st, grid, smem);
  if (dpl == 4) return launch_attention_g<4, float>(ws, a, st, grid, smem);
  return cudaErrorInvalidValue;
}

// The top-K path's attention (fastExp of score - max over all positions,
// infer.go:376-423) in three passes: 0 scores, 1 values, 2 merge + act-quant.
template <int DPL, typename KT>
static cudaError_t launch_attf_g(const AttfArgs& a, dim3 grid, cudaStream_t st, int pass) {
  if (pass == 0)
    return launch(k_attf_scores<DPL, KT>, grid, dim3(ATTF_THREADS), sizeof(AttfScoresSmem), st, a);
  return launch(k_attf_values<DPL, KT>, grid, dim3(ATTF_THREADS), sizeof(AttfValuesSmem), st, a);
}

static cudaError_t launch_attention_fast(const l3g_workspace* ws, const AttfArgs& a,
                                         cudaStream_t st, int pass) {
  const l3g_model* m = ws->m;
  if (pass == 2)
    return launch(k_attf_merge, dim3((a.n_blocks + NW - 1) / NW), dim3(ATTF_THREADS), 0, st, a);
  const dim3 grid(m->hkv_l, ws->attf_splits);
  const int dpl = m->hd / 32;
  if (m->kv_f16) {
    if (dpl == 2) return launch_attf_g<2, __half>(a, grid, st, pass);
    if (dpl == 4) return launch_attf_g<4, __half>(a, grid, st, pass);
    return cudaErrorInvalidValue;
  }
  if (dpl == 1) return launch_attf_g<1, float>(a, grid, st, pass);
  if (dpl == 2) return launch_attf_g<2, float>(a, grid, st, pass);
  if (dpl == 4) return launch_attf_g<4, float>(a, grid, st, pass);
  return cudaErrorInvalidValue;
}

// Whether a step of this variant runs the top-K path's fastExp attention:
// the top-K and sampled calls (ForwardTopKIntoWorkspace, infer.go:269-511)
// once the workspace asked for it; the logits, argmax, greedy and prefill
// calls (ForwardIntoWorkspace, infer.go:21-267) always use the exact exp.
static bool uses_fast_attention(const l3g_workspace* ws, int variant) {
  return ws->topk_fast && (variant == V_TOPK || variant == V_SAMPLE || variant == V_SAMPLE_DEV);
}
// Graphs of a variant captured with the fastExp attention are cached under
// this bit added to the variant.
constexpr int kFastGraphKey = 0x100;

// merges the per-rank argmax results gathered by NCCL (largest logit, lowest
// id on ties; first error wins)
__global__ void k_merge_argmax(const Result* g, int world, Result* out) {
  pdl_wait();
  if (threadIdx.x != 0) return;
  Result best = g[0];
  int err = g[0].err, where = g[0].where;
  for (int r = 1; r < world; ++r) {
    const Result c = g[r];
    if (c.logit > best.logit || (c.logit == best.logit && c.token < best.token)) best = c;
    if (!err && c.err) {
      err = c.err;
      where = c.where;
    }
  }
  out->token = best.token;
  out->logit = best.logit;
  out->err = err;
  out->where = where;
}


static int enqueue_step(l3g_workspace* ws, const l3g_state* s, int variant, int k) {
  const bool traced = variant == V_TRACE;
  if (traced) variant = V_GREEDY_DEV;
  unsigned long long* tr = traced ? ws->d_trace : nullptr;
  if (traced) ws->trace_kinds.clear();
  l3g_model* m = ws->m;
  const l3g_hparams& hp = m->hp;
  cudaStream_t st = ws->stream;
  const int ne = hp.n_emb, hd = m->hd;
  const size_t es = m->kv_f16 ? 2 : 4;
  const unsigned long long wait_ns = m->world > 1 ? WAIT_TIMEOUT_PEER_NS : WAIT_TIMEOUT_NS;
  ws->kernels = 0;
#define KL(kind, expr)                                 \
  do {                                                 \
    CUDA_TRY(expr);                                    \
    ++ws->kernels;                                     \
    if (tr) ws->trace_kinds.push_back(kind);           \
    if (ws->profiling) {                               \
      cudaEvent_t ev_;                                 \
      CUDA_TRY(cudaEventCreate(&ev_));                 \
      CUDA_TRY(cudaEventRecord(ev_, st));              \
      ws->prof_kind.push_back(kind);                   \
      ws->prof_ev.push_back(ev_);                      \
    }                                                  \
  } while (0)
  const bool device_fed = variant == V_GREEDY_DEV || variant == V_SAMPLE_DEV;
  const bool sampled = variant == V_SAMPLE || variant == V_SAMPLE_DEV;
  const bool fast_att = uses_fast_attention(ws, variant);
  const bool persistent = ws->ps_on && !fast_att;  // k_layers has the exact-exp attention only
  if (!device_fed)
    CUDA_TRY(cudaMemcpyAsync(ws->d_io, ws->h_io, 16, cudaMemcpyHostToDevice, st));
  if (variant == V_SAMPLE)
    CUDA_TRY(cudaMemcpyAsync(ws->d_samp, ws->h_samp, sizeof(SampleParams), cudaMemcpyHostToDevice, st));
  KL(L3G_K_EMBED, launch(k_embed, dim3((ne + 255) / 256), dim3(256), 0, st, (const uint8_t*)m->emb,
                  hp.vocab_size, ne, (const int*)ws->d_io, ws->x[0], ws->d_res, ws->d_step,
                  persistent ? ws->d_bar : nullptr, ws->ps_bar_words));
  if (persistent) {  // every layer in one persistent launch
    unsigned long long* stamps =
        tr && kPersistStampOff * 8 + persist_stamp_bytes(ws) <= kTraceBytes
            ? ws->d_trace + kPersistStampOff
            : nullptr;
    KL(L3G_K_LAYERS, launch_layers(ws, s, stamps, st));
  }
  // the per-kernel step (skipped when the persistent kernel ran the layers)
  for (int l = 0; !persistent && l < hp.n_layers; ++l) {
    const LayerW& L = m->layers[l];
    const KvMap kv = state_kv(s);
    {  // RMSNorm -> act-quant -> QKV -> RoPE -> KV append, infer.go:67-127
      MatvecArgs a = mv_args(L.qkv);
      a.wait_ns = wait_ns;
      a.x_in = ws->x[0];
      a.y_in = l ? ws->y : nullptr;
      a.norm_w = L.attn_norm;
      a.x_out = ws->x[1];
      a.eps = hp.rms_eps;
      a.out = ws->q;
      a.nq = m->hq_l * hd;
      a.nkv = m->hkv_l * hd;
      a.head_dim = hd;
      a.rope_half = m->rope_half;
      a.layer = l;
      a.kv_f16 = m->kv_f16;
      a.rope_cos = s->rope_cos;
      a.rope_sin = s->rope_sin;
      a.io = ws->d_io;
      a.kv = kv;
      a.res = ws->d_res;
      a.trace = ws->kernels < kTraceCap ? tr : nullptr;
      a.trace_seq = ws->kernels;
      KL(L3G_K_QKV, (launch_mv<PRO_RMS, EPI_QKV>(L.qkv, a, m->nsm, st)));
    }
    {  // attention, infer.go:130-175
      AttnArgs a{};
      a.wait_ns = wait_ns;
      a.q = ws->q;
      a.kv = kv;
      a.layer = l;
      a.hd = hd;
      a.group = m->group;
      a.n_splits = ws->n_splits;
      a.P = ws->att_P;
      a.nstages = ws->att_ns;
      a.stage_bytes = ws->att_stage;
      a.scale = (float)(1.0 / sqrt((double)hd));
      a.io = ws->d_io;
      a.part_o = ws->part_o;
      a.part_ml = ws->part_ml;
      a.counters = ws->att_cnt;
      a.out = ws->attn;
      a.out_d = ws->attn_d;
      a.out_q = ws->attn_q;
      a.res = ws->d_res;
      a.trace = ws->kernels < kTraceCap ? tr : nullptr;
      a.trace_seq = ws->kernels;
      if (fast_att) {  // the top-K path's fastExp softmax, infer.go:376-423
        AttfArgs f{};
        f.q = ws->q;
        f.kv = kv;
        f.layer = l;
        f.ctx = s->ctx;
        f.hd = hd;
        f.group = m->group;
        f.splits = ws->attf_splits;
        f.n_blocks = m->hq_l * hd / 32;
        f.scale = a.scale;
        f.io = ws->d_io;
        f.scores = ws->attf_scores;
        f.pmax = ws->attf_pmax;
        f.psum = ws->attf_psum;
        f.po = ws->attf_po;
        f.out = ws->attn;
        f.out_d = ws->attn_d;
        f.out_q = ws->attn_q;
        for (int pass = 0; pass < 3; ++pass) KL(L3G_K_ATTN, launch_attention_fast(ws, f, st, pass));
      } else {
        KL(L3G_K_ATTN, launch_attention(ws, a, st));
      }
    }
    {  // Wo on the attention output the merge quantized, infer.go:178-187
       // (residual add fused downstream)
      MatvecArgs a = mv_args(L.wo);
      a.wait_ns = wait_ns;
      a.xd_in = ws->attn_d;
      a.xqs_in = ws->attn_q;
      a.out = ws->y;
      a.res = ws->d_res;
      a.trace = ws->kernels < kTraceCap ? tr : nullptr;
      a.trace_seq = ws->kernels;
      if (ws->tp_p2p) {  // partial rows pushed to every rank (phase 2l)
        a.tp_out = tp_exchange(ws, 2 * l);
        KL(L3G_K_WO, (launch_mv<PRO_PREQ, EPI_PUSH>(L.wo, a, m->nsm, st)));
      } else {
        KL(L3G_K_WO, (launch_mv<PRO_PREQ, EPI_STORE>(L.wo, a, m->nsm, st)));
      }
    }
    if (ws->tp_p2p)
      KL(L3G_K_OTHER, launch(k_tp_reduce, dim3((ne / 4 + 255) / 256), dim3(256), 0, st,
                             tp_exchange(ws, 2 * l), ws->y, ws->d_res, wait_ns));
    else if (m->world > 1)
      NCCL_TRY(nccl()->AllReduce(ws->y, ws->y, ne, ncclFloat, ncclSum, m->comm, st));
    {  // residual -> RMSNorm -> act-quant -> up/gate -> SwiGLU, infer.go:189-230
      MatvecArgs a = mv_args(L.upgate);
      a.wait_ns = wait_ns;
      a.x_in = ws->x[1];
      a.y_in = ws->y;
      a.norm_w = L.ffn_norm;
      a.x_out = ws->x[0];
      a.eps = hp.rms_eps;
      a.out = ws->act;
      a.res = ws->d_res;
      a.trace = ws->kernels < kTraceCap ? tr : nullptr;
      a.trace_seq = ws->kernels;
      KL(L3G_K_UPGATE, (launch_mv<PRO_RMS, EPI_SWIGLU>(L.upgate, a, m->nsm, st)));
    }
    {  // act-quant of the SwiGLU output (once, not per CTA), infer.go:233-234
      const int nb = m->ff_l / 32;
      KL(L3G_K_ACT_QUANT, launch(k_quantize, dim3((nb + NW - 1) / NW), dim3(NW * 32), 0, st,
                                 (const float*)ws->act, m->ff_l, ws->act_d, ws->act_q));
    }
    {  // down, infer.go:235-242
      MatvecArgs a = mv_args(L.down);
      a.wait_ns = wait_ns;
      a.xd_in = ws->act_d;
      a.xqs_in = ws->act_q;
      a.out = ws->y;
      a.res = ws->d_res;
      a.trace = ws->kernels < kTraceCap ? tr : nullptr;
      a.trace_seq = ws->kernels;
      if (ws->tp_p2p) {  // phase 2l + 1
        a.tp_out = tp_exchange(ws, 2 * l + 1);
        KL(L3G_K_DOWN, (launch_mv<PRO_PREQ, EPI_PUSH>(L.down, a, m->nsm, st)));
      } else {
        KL(L3G_K_DOWN, (launch_mv<PRO_PREQ, EPI_STORE>(L.down, a, m->nsm, st)));
      }
    }
    if (ws->tp_p2p)
      KL(L3G_K_OTHER, launch(k_tp_reduce, dim3((ne / 4 + 255) / 256), dim3(256), 0, st,
                             tp_exchange(ws, 2 * l + 1), ws->y, ws->d_res, wait_ns));
    else if (m->world > 1)
      NCCL_TRY(nccl()->AllReduce(ws->y, ws->y, ne, ncclFloat, ncclSum, m->comm, st));
  }
  if (variant != V_PREFILL) {
    // residual -> final RMSNorm -> act-quant -> logits + argmax, infer.go:250-262
    MatvecArgs a = mv_args(m->logits);
      a.wait_ns = wait_ns;
    a.x_in = ws->x[0];
    a.y_in = ws->y;
    a.norm_w = m->out_norm;
    a.x_out = ws->x[1];
    a.eps = hp.rms_eps;
    a.out = ws->logits;
    a.row_offset = m->v_off;
    a.am_val = ws->am_val;
    a.am_idx = ws->am_idx;
    a.am_counter = ws->am_cnt;
    a.res = ws->d_res;
    a.trace = ws->kernels < kTraceCap ? tr : nullptr;
    a.trace_seq = ws->kernels;
    KL(L3G_K_LOGITS, (launch_mv<PRO_RMS, EPI_LOGITS>(m->logits, a, m->nsm, st)));
    const float* full = ws->logits;
    if (m->world > 1) {
      NCCL_TRY(nccl()->AllGather(ws->d_res, ws->d_gather, sizeof(Result) / 4, ncclInt32, m->comm, st));
      KL(L3G_K_OTHER, launch(k_merge_argmax, dim3(1), dim3(32), 0, st, (const Result*)ws->d_gather,
                      m->world, ws->d_res));
      if (variant == V_LOGITS || variant == V_TOPK || sampled) {
        NCCL_TRY(nccl()->AllGather(ws->logits, ws->logits_full, m->v_l, ncclFloat, m->comm, st));
        full = ws->logits_full;
      }
    }
    if (variant == V_LOGITS)
      CUDA_TRY(cudaMemcpyAsync(ws->h_logits, full, (size_t)hp.vocab_size * 4,
                               cudaMemcpyDeviceToHost, st));
    if (variant == V_TOPK || sampled) {
      const int nv = hp.vocab_size;
      const int chunks = (nv + TOPK_CHUNK - 1) / TOPK_CHUNK;
      KL(L3G_K_OTHER, launch(k_topk_partial, dim3(chunks), dim3(512), 0, st, full, nv, k, 0, ws->tk_part));
      int cap = 1;
      while (cap < chunks * k) cap <<= 1;
      KL(L3G_K_OTHER, launch(k_topk_final, dim3(1), dim3(1024), (size_t)cap * 8, st,
                      (const uint64_t*)ws->tk_part, chunks * k, cap, k, ws->d_tk_ids,
                      ws->d_tk_logits));
      if (sampled) {
        KL(L3G_K_OTHER, launch(k_sample, dim3(1), dim3(32), 0, st, (const int*)ws->d_tk_ids,
                               (const float*)ws->d_tk_logits, k, (const SampleParams*)ws->d_samp,
                               // the device-fed loop's step index offsets the draw
                               (const int*)(variant == V_SAMPLE_DEV ? ws->d_io : nullptr),
                               ws->d_res));
      } else {
        CUDA_TRY(cudaMemcpyAsync(ws->h_tk_ids, ws->d_tk_ids, k * 4, cudaMemcpyDeviceToHost, st));
        CUDA_TRY(cudaMemcpyAsync(ws->h_tk_logits, ws->d_tk_logits, k * 4, cudaMemcpyDeviceToHost, st));
      }
    }
  }
  if (device_fed)
    KL(L3G_K_OTHER, launch(k_advance, dim3(1), dim3(32), 0, st, ws->d_io, (const Result*)ws->d_res,
              ws->d_tokens));
  else
    CUDA_TRY(cudaMemcpyAsync(ws->h_res, ws->d_res, sizeof(Result), cudaMemcpyDeviceToHost, st));
#undef KL
  return L3G_OK;
}

static int get_graph(l3g_workspace* ws, const l3g_state* s, int variant, int k,
                     cudaGraphExec_t* out) {
  const int key = variant | (uses_fast_attention(ws, variant) ? kFastGraphKey : 0);
  for (auto& g : ws->graphs)
    if (g.variant == key && g.k == k && g.state_serial == s->serial) {
      *out = g.exec;
      return L3G_OK;
    }
  // a workspace serves one state at a time: drop graphs of other states
  for (auto it = ws->graphs.begin(); it != ws->graphs.end();) {
    if (it->state_serial != s->serial) {
      cudaGraphExecDestroy(it->exec);
      it = ws->graphs.erase(it);
    } else {
      ++it;
    }
  }
  CUDA_TRY(cudaStreamBeginCapture(ws->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(ws, s, variant, k);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(ws->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "graph capture: %s", cudaGetErrorString(e));
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
  ws->graphs.push_back({key, k, s->serial, exec});
  if (ws->m->world > 1) {
    // ranks capture at their own pace; line them up before the first launch
    // so that none waits on a peer that is still capturing
    NCCL_TRY(nccl()->AllReduce(ws->d_sync, ws->d_sync, 1, ncclInt32, ncclMax, ws->m->comm,
                               ws->stream));
    CUDA_TRY(cudaStreamSynchronize(ws->stream));
  }
  if (variant == V_GREEDY_DEV) ws->kernels_greedy = ws->kernels;
  if (variant == V_TRACE) ws->trace_kinds_graph = ws->trace_kinds;
  *out = exec;
  return L3G_OK;
}

// One step: the checks of ForwardIntoWorkspace (infer.go:22-33,514-516),
// the graph replay, the device error word, position advance (infer.go:265).
static int run_step(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token, int variant,
                    int k) {
  if (!m || !s) return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws) return l3g_fail(L3G_E_INVALID, "workspace is nil");
  if (s->m != m || ws->m != m)
    return l3g_fail(L3G_E_INVALID, "state or workspace belongs to another model");
  if (s->pos >= s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  if (ws->ctx < s->ctx)
    return l3g_fail(L3G_E_INVALID, "workspace ctxLen=%d < state ctxLen=%d", ws->ctx, s->ctx);
  if (token < 0 || token >= m->hp.vocab_size)
    return l3g_fail(L3G_E_TOKEN, "token out of range: %d", token);
  CUDA_TRY(cudaSetDevice(m->device));
  cudaGraphExec_t exec;
  int rc = get_graph(ws, s, variant, k, &exec);
  if (rc) return rc;
  if ((rc = state_map(s, s->pos + 1, ws->stream))) return rc;
  ws->h_io[0] = token;
  ws->h_io[1] = s->pos;
  ws->h_io[2] = 0;
  ws->h_io[3] = 0;
  CUDA_TRY(cudaGraphLaunch(exec, ws->stream));
  CUDA_TRY(cudaStreamSynchronize(ws->stream));
  if (ws->h_res->err) {
    const int code = ws->h_res->err, where = ws->h_res->where;
    ws_clear_device_error(ws);
    ws->logits_valid = false;
    return l3g_fail(L3G_E_DEVICE, "device check failed: code %d at site %d (%s)", code, where,
                    code == ERR_TIMEOUT ? "bounded wait ran out" : "bad input");
  }
  ws->logits_valid = variant != V_PREFILL;
  s->pos++;
  return L3G_OK;
}

extern "C" int l3g_forward(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token,
                           float* logits_out) {
  const int rc = run_step(m, s, ws, token, logits_out ? V_LOGITS : V_PREFILL, 0);
  if (rc == L3G_OK && logits_out)
    memcpy(logits_out, ws->h_logits, (size_t)m->hp.vocab_size * 4);
  return rc;
}

extern "C" int l3g_forward_argmax(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token,
                                  int32_t* next, float* logit) {
  const int rc = run_step(m, s, ws, token, V_ARGMAX, 0);
  if (rc == L3G_OK) {
    if (next) *next = ws->h_res->token;
    if (logit) *logit = ws->h_res->logit;
  }
  return rc;
}

extern "C" int l3g_forward_topk(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token,
                                int32_t top_k, l3g_topk_item* items, int32_t* n_items) {
  if (top_k <= 0) top_k = 40;  // infer.go:279-281
  if (top_k > MAX_TOPK) return l3g_fail(L3G_E_INVALID, "top_k %d above %d", top_k, MAX_TOPK);
  if (m && top_k > m->hp.vocab_size) top_k = m->hp.vocab_size;
  if (!items) return l3g_fail(L3G_E_INVALID, "null argument");
  const int rc = run_step(m, s, ws, token, V_TOPK, top_k);
  if (rc == L3G_OK) {
    for (int i = 0; i < top_k; ++i) {
      items[i].id = ws->h_tk_ids[i];
      items[i].logit = ws->h_tk_logits[i];
    }
    if (n_items) *n_items = top_k;
  }
  return rc;
}

extern "C" int l3g_prefill(l3g_model* m, l3g_state* s, l3g_workspace* ws, const int32_t* tokens,
                           int32_t n) {
  if (n > 0 && !tokens) return l3g_fail(L3G_E_INVALID, "null argument");
  for (int i = 0; i < n; ++i) {
    const int rc = run_step(m, s, ws, tokens[i], V_PREFILL, 0);
    if (rc) return rc;
  }
  return L3G_OK;
}

extern "C" int l3g_decode_greedy(l3g_model* m, l3g_state* s, l3g_workspace* ws,
                                 int32_t first_token, int32_t n, int32_t* out_tokens,
                                 float* device_ms) {
  if (!m || !s || !out_tokens) return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws) return l3g_fail(L3G_E_INVALID, "workspace is nil");
  if (s->m != m || ws->m != m)
    return l3g_fail(L3G_E_INVALID, "state or workspace belongs to another model");
  if (n <= 0) return L3G_OK;
  if (ws->ctx < s->ctx)
    return l3g_fail(L3G_E_INVALID, "workspace ctxLen=%d < state ctxLen=%d", ws->ctx, s->ctx);
  if (s->pos + n > s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  if (first_token < 0 || first_token >= m->hp.vocab_size)
    return l3g_fail(L3G_E_TOKEN, "token out of range: %d", first_token);
  CUDA_TRY(cudaSetDevice(m->device));
  cudaGraphExec_t exec;
  int rc = get_graph(ws, s, V_GREEDY_DEV, 0, &exec);
  if (rc) return rc;
  if ((rc = state_map(s, s->pos + n, ws->stream))) return rc;
  cudaEvent_t e0, e1;
  CUDA_TRY(cudaEventCreate(&e0));
  CUDA_TRY(cudaEventCreate(&e1));
  ws->h_io[0] = first_token;
  ws->h_io[1] = s->pos;
  ws->h_io[2] = 0;
  ws->h_io[3] = 0;
  cudaError_t e = cudaMemcpyAsync(ws->d_io, ws->h_io, 16, cudaMemcpyHostToDevice, ws->stream);
  if (e == cudaSuccess) e = cudaEventRecord(e0, ws->stream);
  for (int i = 0; i < n && e == cudaSuccess; ++i) e = cudaGraphLaunch(exec, ws->stream);
  if (e == cudaSuccess) e = cudaEventRecord(e1, ws->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(ws->h_res, ws->d_res, sizeof(Result), cudaMemcpyDeviceToHost, ws->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ws->stream);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  if (e == cudaSuccess)
    e = cudaMemcpy(out_tokens, ws->d_tokens, (size_t)n * 4, cudaMemcpyDeviceToHost);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "greedy decode: %s", cudaGetErrorString(e));
  if (ws->h_res->err) {
    const int code = ws->h_res->err, where = ws->h_res->where;
    ws_clear_device_error(ws);
    return l3g_fail(L3G_E_DEVICE, "device check failed: code %d at site %d", code, where);
  }
  if (device_ms) *device_ms = ms;
  ws->logits_valid = true;
  s->pos += n;
  return L3G_OK;
}

// Sampler defaults of NewSampler (sampling.go:19-30) for the device sampler.
static int sample_setup(l3g_workspace* ws, int32_t* top_k, float* temperature, uint64_t seed) {
  if (*temperature <= 0.0f) *temperature = 0.8f;
  if (*top_k <= 0) *top_k = ws->topk;
  if (*top_k > MAX_TOPK) return l3g_fail(L3G_E_INVALID, "top_k %d above %d", *top_k, MAX_TOPK);
  ws->h_samp->temperature = *temperature;
  ws->h_samp->seed = seed;
  ws->h_samp->counter = ws->draws;
  return L3G_OK;
}

extern "C" int l3g_forward_sample(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token,
                                  int32_t top_k, float temperature, uint64_t seed, int32_t* next) {
  if (!next) return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws) return l3g_fail(L3G_E_INVALID, "workspace is nil");
  int rc = sample_setup(ws, &top_k, &temperature, seed);
  if (rc) return rc;
  rc = run_step(m, s, ws, token, V_SAMPLE, top_k);
  if (rc) return rc;
  *next = ws->h_res->token;
  ws->draws += 1;
  return L3G_OK;
}

extern "C" int l3g_decode_sample(l3g_model* m, l3g_state* s, l3g_workspace* ws,
                                 int32_t first_token, int32_t n, int32_t top_k,
                                 float temperature, uint64_t seed, const int32_t* stop_ids,
                                 int32_t n_stop, int32_t* out_tokens, int32_t* n_out,
                                 float* device_ms) {
  if (!m || !s || !out_tokens || !n_out || (n_stop > 0 && !stop_ids))
    return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws) return l3g_fail(L3G_E_INVALID, "workspace is nil");
  if (s->m != m || ws->m != m)
    return l3g_fail(L3G_E_INVALID, "state or workspace belongs to another model");
  *n_out = 0;
  if (n <= 0) return L3G_OK;
  if (ws->ctx < s->ctx)
    return l3g_fail(L3G_E_INVALID, "workspace ctxLen=%d < state ctxLen=%d", ws->ctx, s->ctx);
  if (s->pos + n > s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  if (first_token < 0 || first_token >= m->hp.vocab_size)
    return l3g_fail(L3G_E_TOKEN, "token out of range: %d", first_token);
  int rc = sample_setup(ws, &top_k, &temperature, seed);
  if (rc) return rc;
  CUDA_TRY(cudaSetDevice(m->device));
  cudaGraphExec_t exec;
  rc = get_graph(ws, s, V_SAMPLE_DEV, top_k, &exec);
  if (rc) return rc;
  if ((rc = state_map(s, s->pos + n, ws->stream))) return rc;
  cudaEvent_t e0, e1;
  CUDA_TRY(cudaEventCreate(&e0));
  CUDA_TRY(cudaEventCreate(&e1));
  ws->h_io[0] = first_token;
  ws->h_io[1] = s->pos;
  ws->h_io[2] = 0;
  ws->h_io[3] = 0;
  cudaError_t e = cudaMemcpyAsync(ws->d_io, ws->h_io, 16, cudaMemcpyHostToDevice, ws->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(ws->d_samp, ws->h_samp, sizeof(SampleParams), cudaMemcpyHostToDevice,
                        ws->stream);
  if (e == cudaSuccess) e = cudaEventRecord(e0, ws->stream);
  for (int i = 0; i < n && e == cudaSuccess; ++i) e = cudaGraphLaunch(exec, ws->stream);
  if (e == cudaSuccess) e = cudaEventRecord(e1, ws->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(ws->h_res, ws->d_res, sizeof(Result), cudaMemcpyDeviceToHost, ws->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ws->stream);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  if (e == cudaSuccess)
    e = cudaMemcpy(out_tokens, ws->d_tokens, (size_t)n * 4, cudaMemcpyDeviceToHost);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "sampled decode: %s", cudaGetErrorString(e));
  if (ws->h_res->err) {
    const int code = ws->h_res->err, where = ws->h_res->where;
    ws_clear_device_error(ws);
    return l3g_fail(L3G_E_DEVICE, "device check failed: code %d at site %d", code, where);
  }
  ws->draws += (uint64_t)n;
  // the chat loop's stop rule (cmd/go-llama-chat/main.go:146-150): the
  // samples up to and including the first stop id count; the position
  // covers the tokens ingested up to the stop token's own ingestion (the
  // step after it was sampled), which the loop ran unless it was the last
  int kept = n;
  for (int i = 0; i < n && kept == n; ++i)
    for (int j = 0; j < n_stop; ++j)
      if (out_tokens[i] == stop_ids[j]) {
        kept = i + 1;
        break;
      }
  *n_out = kept;
  if (device_ms) *device_ms = ms;
  ws->logits_valid = kept == n;
  s->pos += kept < n ? kept + 1 : n;
  return L3G_OK;
}

extern "C" int l3g_profile_step(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token,
                                int32_t* kinds, float* us, int32_t* n) {
  if (!m || !s || !ws || !kinds || !us || !n) return l3g_fail(L3G_E_INVALID, "null argument");
  if (s->m != m || ws->m != m)
    return l3g_fail(L3G_E_INVALID, "state or workspace belongs to another model");
  if (s->pos >= s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  if (ws->ctx < s->ctx)
    return l3g_fail(L3G_E_INVALID, "workspace ctxLen=%d < state ctxLen=%d", ws->ctx, s->ctx);
  if (token < 0 || token >= m->hp.vocab_size)
    return l3g_fail(L3G_E_TOKEN, "token out of range: %d", token);
  CUDA_TRY(cudaSetDevice(m->device));
  if (int rc0 = state_map(s, s->pos + 1, ws->stream)) return rc0;
  cudaEvent_t e0;
  CUDA_TRY(cudaEventCreate(&e0));
  ws->h_io[0] = token;
  ws->h_io[1] = s->pos;
  ws->profiling = true;
  g_serialize = true;
  int rc = L3G_OK;
  cudaError_t e = cudaEventRecord(e0, ws->stream);
  if (e == cudaSuccess) rc = enqueue_step(ws, s, V_ARGMAX, 0);
  g_serialize = false;
  ws->profiling = false;
  if (e == cudaSuccess && rc == L3G_OK) e = cudaStreamSynchronize(ws->stream);
  const int cnt = (int)ws->prof_ev.size();
  if (e == cudaSuccess && rc == L3G_OK) {
    cudaEvent_t prev = e0;
    for (int i = 0; i < cnt && i < *n; ++i) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, prev, ws->prof_ev[i]);
      kinds[i] = ws->prof_kind[i];
      us[i] = ms * 1000.0f;
      prev = ws->prof_ev[i];
    }
  }
  for (auto ev : ws->prof_ev) cudaEventDestroy(ev);
  ws->prof_ev.clear();
  ws->prof_kind.clear();
  cudaEventDestroy(e0);
  if (rc) return rc;
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "profile step: %s", cudaGetErrorString(e));
  if (ws->h_res->err) {
    ws_clear_device_error(ws);
    return l3g_fail(L3G_E_DEVICE, "device check failed during profiling");
  }
  *n = std::min(cnt, *n);
  s->pos++;
  return L3G_OK;
}

extern "C" int l3g_trace_step(l3g_model* m, l3g_state* s, l3g_workspace* ws, int32_t token,
                              uint64_t* stamps, int32_t* kinds, int32_t* n) {
  if (!m || !s || !ws || !stamps || !kinds || !n) return l3g_fail(L3G_E_INVALID, "null argument");
  if (s->m != m || ws->m != m)
    return l3g_fail(L3G_E_INVALID, "state or workspace belongs to another model");
  if (s->pos >= s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  if (ws->ctx < s->ctx)
    return l3g_fail(L3G_E_INVALID, "workspace ctxLen=%d < state ctxLen=%d", ws->ctx, s->ctx);
  if (token < 0 || token >= m->hp.vocab_size)
    return l3g_fail(L3G_E_TOKEN, "token out of range: %d", token);
  CUDA_TRY(cudaSetDevice(m->device));
  cudaGraphExec_t exec;
  int rc = get_graph(ws, s, V_TRACE, 0, &exec);
  if (rc) return rc;
  if ((rc = state_map(s, s->pos + 1, ws->stream))) return rc;
  const int cnt = std::min<int>((int)ws->trace_kinds_graph.size(), kTraceCap);
  ws->h_io[0] = token;
  ws->h_io[1] = s->pos;
  ws->h_io[2] = 0;
  ws->h_io[3] = 0;
  CUDA_TRY(cudaMemsetAsync(ws->d_trace, 0, kTraceBytes, ws->stream));
  CUDA_TRY(cudaMemcpyAsync(ws->d_io, ws->h_io, 16, cudaMemcpyHostToDevice, ws->stream));
  CUDA_TRY(cudaGraphLaunch(exec, ws->stream));
  CUDA_TRY(cudaMemcpyAsync(ws->h_res, ws->d_res, sizeof(Result), cudaMemcpyDeviceToHost, ws->stream));
  CUDA_TRY(cudaStreamSynchronize(ws->stream));
  if (ws->h_res->err) {
    ws_clear_device_error(ws);
    return l3g_fail(L3G_E_DEVICE, "device check failed during trace");
  }
  const int out_n = std::min(cnt, *n);
  CUDA_TRY(cudaMemcpy(stamps, ws->d_trace, (size_t)out_n * TRACE_CTAS * 8 * 8,
                      cudaMemcpyDeviceToHost));
  for (int i = 0; i < out_n; ++i) kinds[i] = ws->trace_kinds_graph[i];
  *n = out_n;
  s->pos++;
  return L3G_OK;
}

extern "C" int l3g_workspace_set_topk_fast_exp(l3g_workspace* ws, int32_t on) {
  if (!ws) return l3g_fail(L3G_E_INVALID, "null argument");
  if (on != 0 && on != 1) return l3g_fail(L3G_E_INVALID, "on must be 0 or 1, got %d", on);
  const l3g_model* m = ws->m;
  if (on && !ws->attf_scores) {
    const int hd = m->hd, G = m->group;
    if (hd % 32 || hd > ATTF_MAX_HD || G > MAXG)
      return l3g_fail(L3G_E_INVALID, "fastExp attention: head dim %d, group %d unsupported", hd, G);
    // about two CTAs per SM over the kv heads, at least NW positions a split
    const int S = std::max(1, std::min({(2 * m->nsm + m->hkv_l - 1) / m->hkv_l,
                                        (ws->ctx + NW - 1) / NW, 64}));
    CUDA_TRY(cudaSetDevice(ws->device));
    const size_t parts = (size_t)m->hkv_l * S * G;
    float* p[4] = {nullptr, nullptr, nullptr, nullptr};
    const size_t floats[4] = {(size_t)m->hq_l * ws->ctx, parts, parts, parts * hd};
    for (int i = 0; i < 4; ++i) {
      if (cudaMalloc(&p[i], floats[i] * 4) != cudaSuccess) {
        cudaGetLastError();
        for (int j = 0; j < i; ++j) cudaFree(p[j]);
        return l3g_fail(L3G_E_CUDA, "fastExp attention scratch: out of device memory");
      }
    }
    ws->attf_scores = p[0];
    ws->attf_pmax = p[1];
    ws->attf_psum = p[2];
    ws->attf_po = p[3];
    ws->attf_splits = S;
  }
  ws->topk_fast = on == 1;
  return L3G_OK;
}

extern "C" int l3g_workspace_kernels_per_step(l3g_workspace* ws, int32_t* n) {
  if (!ws || !n) return l3g_fail(L3G_E_INVALID, "null argument");
  *n = ws->kernels_greedy;
  return L3G_OK;
}

extern "C" int l3g_workspace_attention_layout(const l3g_workspace* ws, int32_t* splits,
                                              int32_t* cluster) {
  if (!ws || !splits || !cluster) return l3g_fail(L3G_E_INVALID, "null argument");
  *splits = ws->n_splits;
  *cluster = ws->att_cluster;
  return L3G_OK;
}

extern "C" int l3g_workspace_tp_p2p(const l3g_workspace* ws, int32_t* p2p) {
  if (!ws || !p2p) return l3g_fail(L3G_E_INVALID, "null argument");
  *p2p = ws->tp_p2p ? 1 : 0;
  return L3G_OK;
}

extern "C" int l3g_workspace_read(const l3g_workspace* ws, int32_t which, float* out, int32_t n) {
  if (!ws || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  const l3g_model* m = ws->m;
  const float* src = nullptr;
  int cnt = 0;
  switch (which) {
    case L3G_BUF_HIDDEN: src = ws->x[1]; cnt = m->hp.n_emb; break;
    case L3G_BUF_Q: src = ws->q; cnt = m->hq_l * m->hd; break;
    case L3G_BUF_ATTN: src = ws->attn; cnt = m->hq_l * m->hd; break;
    case L3G_BUF_FFN_ACT: src = ws->act; cnt = m->ff_l; break;
    case L3G_BUF_LOGITS:
      if (!ws->logits_valid) return l3g_fail(L3G_E_INVALID, "no logits computed yet");
      src = m->world > 1 ? ws->logits_full : ws->logits;
      cnt = m->world > 1 ? m->hp.vocab_size : m->v_l;
      break;
    default: return l3g_fail(L3G_E_INVALID, "unknown buffer %d", which);
  }
  if (n < cnt) return l3g_fail(L3G_E_INVALID, "buffer needs %d floats", cnt);
  CUDA_TRY(cudaSetDevice(m->device));
  CUDA_TRY(cudaMemcpy(out, src, (size_t)cnt * 4, cudaMemcpyDeviceToHost));
  return L3G_OK;
}

// ---------------------------------------------------------------------------
// standalone matvec (matvec_q8_c drop-in) and quantization
// ---------------------------------------------------------------------------
struct l3g_matrix {
  DevMat w;
  int device = 0, nsm = 1;
  Result* d_res = nullptr;  // device error word of the kernel's bounded waits
};

extern "C" void l3g_matrix_free(l3g_matrix* w) {
  if (!w) return;
  cudaSetDevice(w->device);
  free_mat(w->w);
  if (w->d_res) cudaFree(w->d_res);
  delete w;
}

extern "C" int l3g_matrix_upload(const void* q8, int32_t rows, int32_t cols, int32_t device,
                                 l3g_matrix** out) {
  if (!q8 || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  if (rows <= 0 || cols <= 0 || cols % 32)
    return l3g_fail(L3G_E_INVALID, "matvec: cols=%d not multiple of 32", cols);
  int dev = device;
  if (dev < 0) CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaSetDevice(dev));
  int rc = setup_kernels();
  if (rc) return rc;
  auto* w = new l3g_matrix();
  w->device = dev;
  w->nsm = sm_count(dev);
  RowSrc seg{static_cast<const uint8_t*>(q8), 0, rows};
  size_t bytes = 0;
  rc = upload_tiled(w->w, &seg, 1, false, cols, 0, cols, w->nsm, &bytes);
  if (rc == L3G_OK && (cudaMalloc(&w->d_res, sizeof(Result)) != cudaSuccess ||
                       cudaMemset(w->d_res, 0, sizeof(Result)) != cudaSuccess))
    rc = l3g_fail(L3G_E_CUDA, "matrix result word allocation failed");
  if (rc) {
    l3g_matrix_free(w);
    return rc;
  }
  *out = w;
  return L3G_OK;
}

extern "C" int l3g_matrix_device_bytes(const l3g_matrix* w, uint64_t* bytes) {
  if (!w || !bytes) return l3g_fail(L3G_E_INVALID, "null argument");
  *bytes = w->w.bytes;
  return L3G_OK;
}

extern "C" int l3g_matvec_q8(const l3g_matrix* w, const float* x_scales, const int8_t* x_qs,
                             float* out, int32_t start, int32_t end, void* stream) {
  if (!w || !x_scales || !x_qs || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  if (start < 0 || end > w->w.t.rows || start >= end)
    return l3g_fail(L3G_E_INVALID, "row range [%d, %d) outside [0, %d)", start, end, w->w.t.rows);
  if (((uintptr_t)x_qs & 15) || ((uintptr_t)x_scales & 3) || ((uintptr_t)out & 3))
    return l3g_fail(L3G_E_INVALID, "x_qs must be 16-byte aligned, x_scales/out 4-byte");
  CUDA_TRY(cudaSetDevice(w->device));
  MatvecArgs a = mv_args(w->w);
  a.row_lo = start;
  a.row_hi = end;
  a.xd_in = x_scales;
  a.xqs_in = x_qs;
  a.out = out;
  a.res = w->d_res;
  CUDA_TRY((launch_mv<PRO_PREQ, EPI_STORE>(w->w, a, w->nsm, (cudaStream_t)stream)));
  return L3G_OK;
}

// ---------------------------------------------------------------------------
// matvec + argmax out of static device scratch (allocates nothing)
// ---------------------------------------------------------------------------
// Layout of the array: [0, S) per-CTA best value (float bits), [S, 2S) its
// row, [2S] the arrival counter, S = L3G_ARGMAX_STATIC_MAX_CTAS (8 KB + 256
// bytes).  The counter must be zero when a launch starts, so every call
// clears it on its stream before the launch (a 4-byte memset, no
// allocation); a counter left wrong by overlapping calls is therefore
// repaired by the next call.  The slots need no initial value: a CTA writes
// its own before it increments the counter.
constexpr int kArgmaxSlots = L3G_ARGMAX_STATIC_MAX_CTAS;
static __device__ __align__(256) uint32_t g_argmax_scratch[2 * kArgmaxSlots + 64];

struct ArgmaxStatic {   // per device, filled by the first successful set-up on it
  std::mutex mu;
  bool ready = false;
  uint32_t* scratch = nullptr;
};
static ArgmaxStatic g_argmax_static[64];

// Once per device, with that device current: the array's device address and
// the kernels' attributes.  Neither allocates.  Only success is latched: a
// failed set-up (for instance a first call made during stream capture)
// reports its CUDA error and the next call tries again.
static int argmax_static_setup(int dev, uint32_t** scratch) {
  if (dev < 0 || dev >= 64) return l3g_fail(L3G_E_INVALID, "device %d out of range", dev);
  ArgmaxStatic& st = g_argmax_static[dev];
  std::lock_guard<std::mutex> lock(st.mu);
  if (!st.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
    if (e == cudaSuccess) e = set_max_shared(k_matvec<PRO_PREQ, EPI_LOGITS, 1, 1>, 227 * 1024);
    if (e == cudaSuccess) e = set_max_shared(k_matvec<PRO_PREQ, EPI_LOGITS, 2, 1>, 227 * 1024);
    if (e == cudaSuccess) e = set_max_shared(k_matvec<PRO_PREQ, EPI_LOGITS, 4, 1>, 227 * 1024);
    if (e == cudaSuccess) e = set_max_shared(k_matvec<PRO_PREQ, EPI_LOGITS, 8, 1>, 227 * 1024);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return l3g_fail(L3G_E_CUDA, "static argmax scratch set-up on device %d: %s", dev,
                      cudaGetErrorString(e));
    }
    st.scratch = static_cast<uint32_t*>(p);
    st.ready = true;
  }
  *scratch = st.scratch;
  return L3G_OK;
}

// Makes a device current for the scope and puts the caller's back on exit.
struct DeviceScope {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int dev) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

extern "C" int l3g_matvec_q8_argmax_static(const l3g_matrix* w, const float* x_scales,
                                           const int8_t* x_qs, float* out,
                                           l3g_argmax_result* result, int32_t max_ctas,
                                           void* stream) {
  static_assert(sizeof(l3g_argmax_result) == sizeof(Result), "result layout");
  if (!w || !x_scales || !x_qs || !result) return l3g_fail(L3G_E_INVALID, "null argument");
  if (((uintptr_t)x_qs & 15) || ((uintptr_t)x_scales & 3) || ((uintptr_t)out & 3) ||
      ((uintptr_t)result & 15))
    return l3g_fail(L3G_E_INVALID, "x_qs and result must be 16-byte aligned, x_scales/out 4-byte");
  if (max_ctas < 0 || max_ctas > kArgmaxSlots)
    return l3g_fail(L3G_E_INVALID,
                    "max_ctas=%d outside [0, %d]: the static argmax scratch holds %d CTA slots",
                    max_ctas, kArgmaxSlots, kArgmaxSlots);
  const int ng = w->w.t.n_groups;
  const int grid = std::max(1, std::min(ng, max_ctas ? max_ctas : w->nsm));
  if (grid > kArgmaxSlots)
    return l3g_fail(L3G_E_INVALID,
                    "launch needs %d CTA slots, the static argmax scratch holds %d", grid,
                    kArgmaxSlots);
  DeviceScope dev(w->device);
  CUDA_TRY(dev.err);
  uint32_t* scratch = nullptr;
  if (int rc = argmax_static_setup(w->device, &scratch)) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  // index -1 until the merging CTA writes the result: a launch whose merge
  // never ran (its counter disturbed by an overlapping call) stays visible
  CUDA_TRY(cudaMemsetAsync(result, 0xff, sizeof(int32_t), st));
  CUDA_TRY(cudaMemsetAsync(reinterpret_cast<uint8_t*>(result) + sizeof(int32_t), 0,
                           sizeof(*result) - sizeof(int32_t), st));
  CUDA_TRY(cudaMemsetAsync(scratch + 2 * kArgmaxSlots, 0, sizeof(uint32_t), st));
  MatvecArgs a = mv_args(w->w);
  a.xd_in = x_scales;
  a.xqs_in = x_qs;
  a.out = out;
  a.row_offset = 0;
  a.am_val = reinterpret_cast<float*>(scratch);
  a.am_idx = reinterpret_cast<int*>(scratch + kArgmaxSlots);
  a.am_counter = scratch + 2 * kArgmaxSlots;
  a.res = reinterpret_cast<Result*>(result);
  const dim3 g(grid);
  cudaError_t e;
  switch (w->w.t.wr / NW) {
    case 1: e = launch_mv_r<PRO_PREQ, EPI_LOGITS, 1>(w->w, a, g, st); break;
    case 2: e = launch_mv_r<PRO_PREQ, EPI_LOGITS, 2>(w->w, a, g, st); break;
    case 4: e = launch_mv_r<PRO_PREQ, EPI_LOGITS, 4>(w->w, a, g, st); break;
    case 8: e = launch_mv_r<PRO_PREQ, EPI_LOGITS, 8>(w->w, a, g, st); break;
    default: e = cudaErrorInvalidValue;
  }
  CUDA_TRY(e);
  return L3G_OK;
}

extern "C" int l3g_quantize_q8_0(const float* x, int32_t n, float* d, int8_t* qs, void* stream) {
  if (!x || !d || !qs || n <= 0) return l3g_fail(L3G_E_INVALID, "bad argument");
  const int nb = (n + 31) / 32;
  const int threads = 256;
  const int blocks = (nb * 32 + threads - 1) / threads;
  k_quantize<<<blocks, threads, 0, (cudaStream_t)stream>>>(x, n, d, qs);
  CUDA_TRY(cudaGetLastError());
  return L3G_OK;
}
