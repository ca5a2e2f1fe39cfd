// The persistent layer kernel (k_layers): its plan for a workspace, its
// arguments for a state, its launch and its inspection entries.
#include "l3g_rt.h"

template <int DPL, typename KT>
static void* layers_kernel_t(int gp, bool fm) {
  switch (gp) {
    case 1: return fm ? (void*)k_layers<DPL, KT, 1, true> : (void*)k_layers<DPL, KT, 1, false>;
    case 2: return fm ? (void*)k_layers<DPL, KT, 2, true> : (void*)k_layers<DPL, KT, 2, false>;
    case 4: return fm ? (void*)k_layers<DPL, KT, 4, true> : (void*)k_layers<DPL, KT, 4, false>;
    case 8: return fm ? (void*)k_layers<DPL, KT, 8, true> : (void*)k_layers<DPL, KT, 8, false>;
    default: return nullptr;
  }
}
// The instantiation of k_layers for this model's head size, KV element type
// and query heads per kv head (rounded up to a power of two).
static void* layers_kernel(const l3g_model* m, int gp, bool fm) {
  const int dpl = m->hd / 32;
  if (m->kv_f16) {
    if (dpl == 2) return layers_kernel_t<2, __half>(gp, fm);
    if (dpl == 4) return layers_kernel_t<4, __half>(gp, fm);
  } else {
    if (dpl == 1) return layers_kernel_t<1, float>(gp, fm);
    if (dpl == 2) return layers_kernel_t<2, float>(gp, fm);
    if (dpl == 4) return layers_kernel_t<4, float>(gp, fm);
  }
  return nullptr;
}

// The persistent layer kernel's plan for this workspace, when the model was
// loaded for it: the four layer matrices' tile geometry (four rows per
// warp), the attention split (the per-kernel step's count, so both give the
// same partials), and a ring of as many slots as fit beside the phase
// scratch.  It stays off (the per-kernel step runs) when a tensor-parallel
// workspace has no peer-memory exchange, or the kernel cannot be resident
// on every SM.
int persist_setup(l3g_workspace* ws) {
  l3g_model* m = ws->m;
  ws->ps_on = false;
  if (!m->persist || (m->world > 1 && !ws->tp_p2p) || m->hkv_l > m->nsm) return L3G_OK;
  const LayerW& L0 = m->layers[0];
  const DevMat* mats[persist::N_MAT] = {&L0.qkv, &L0.wo, &L0.upgate, &L0.down};
  int rows[persist::N_MAT], cols[persist::N_MAT];
  for (int i = 0; i < persist::N_MAT; ++i) {
    rows[i] = mats[i]->t.rows;
    cols[i] = mats[i]->t.cols;
  }
  const size_t es = m->kv_f16 ? 2 : 4;
  persist::Plan& p = ws->ps_plan;
  p = persist::make_plan(m->nsm, m->hp.n_layers, rows, cols, m->hkv_l, ws->att_P,
                         2 * m->hd * (int)es, ws->ctx, NW, TILE_TARGET);
  // L3G_PERSIST_SPLITS=n caps the attention splits per kv head (fewer,
  // longer items: less merge work, more stages per item)
  if (const char* env = getenv("L3G_PERSIST_SPLITS"))
    if (atoi(env) >= 1) p.splits = std::min(p.splits, atoi(env));
  int slot = p.P * p.row_bytes, max_cols = 0;
  for (int i = 0; i < persist::N_MAT; ++i) {
    const Q8Tiles& t = mats[i]->t;  // the uploaded layout must be the plan's
    if (t.wr != p.wr[i] || t.ck != p.ck[i] || t.nslices != p.nsl[i] ||
        t.tile_bytes != p.tile_bytes[i] || t.n_groups != p.ng[i])
      return L3G_OK;
    slot = std::max(slot, t.tile_bytes);
    max_cols = std::max(max_cols, t.cols);
  }
  if (m->hp.n_emb > 8 * NW * 32 * 4) return L3G_OK;  // ps_rms holds 8 float4 per thread
  ws->ps_slot = align_up(slot, 128);
  ws->ps_xq_off = ps_xq_off(max_cols);
  ws->ps_union = ps_union_bytes(max_cols, m->group, m->hd, p.splits);
  const int limit = 227 * 1024;
  ws->ps_ns = std::min(MAX_STAGES, (limit - PS_HEAD - ws->ps_union) / ws->ps_slot);
  // L3G_PERSIST_STAGES=n caps the ring slots (a tuning knob for experiments)
  if (const char* env = getenv("L3G_PERSIST_STAGES"))
    if (atoi(env) >= 2) ws->ps_ns = std::min(ws->ps_ns, atoi(env));
  if (ws->ps_ns < 2) return L3G_OK;
  ws->ps_smem = PS_HEAD + ws->ps_union + ws->ps_ns * ws->ps_slot;
  int gp = 1;
  while (gp < m->group) gp <<= 1;
  // L3G_PERSIST_FUSE_MERGE=1: the split merge runs in the attention phase
  // (its own instantiation of the kernel)
  {
    const char* env = getenv("L3G_PERSIST_FUSE_MERGE");
    ws->ps_fuse_merge = env && atoi(env) == 1;
  }
  void* k = layers_kernel(m, gp, ws->ps_fuse_merge);
  // attributes of this instantiation only, here rather than at load, so the
  // per-kernel step never depends on the persistent kernel's set-up
  int per_sm = 0;
  if (!k || set_max_shared(k, limit) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, NTHREADS, ws->ps_smem) !=
          cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    return L3G_OK;
  }
  // L3G_PERSIST_FUSE_QUANT=1: the SwiGLU act-quant runs in the up/gate phase
  {
    const char* env = getenv("L3G_PERSIST_FUSE_QUANT");
    ws->ps_fuse = env && atoi(env) == 1 && p.wr[persist::M_UPGATE] == 32 &&
                  p.rows[persist::M_UPGATE] % 64 == 0;
  }
  ws->ps_bar_words = persist::BAR_QCNT + m->ff_l / 32 + m->hkv_l;
  CUDA_TRY(cudaMalloc(&ws->d_bar, ws->ps_bar_words * sizeof(unsigned)));
  CUDA_TRY(cudaMemset(ws->d_bar, 0, ws->ps_bar_words * sizeof(unsigned)));
  // barrier counters: L3G_PERSIST_BAR_SPREAD=n spreads the arrivals over n
  ws->ps_nsub = 1;
  if (const char* env = getenv("L3G_PERSIST_BAR_SPREAD"))
    ws->ps_nsub = std::max(1, std::min({atoi(env), (int)persist::BAR_MAX_SUB, p.grid}));
  ws->ps_on = true;
  return L3G_OK;
}



// Arguments of the persistent layer kernel for state s (its cache, RoPE
// tables and context length are captured into the step's graph).
static PersistArgs persist_args(const l3g_workspace* ws, const l3g_state* s,
                                unsigned long long* stamps) {
  const l3g_model* m = ws->m;
  PersistArgs a{};
  a.plan = ws->ps_plan;
  a.plan.ctx = s->ctx;
  a.layers = m->d_layers;
  a.nstages = ws->ps_ns;
  a.slot_bytes = ws->ps_slot;
  a.union_bytes = ws->ps_union;
  a.xq_off = ws->ps_xq_off;
  a.eps = m->hp.rms_eps;
  a.scale = (float)(1.0 / sqrt((double)m->hd));
  a.n_emb = m->hp.n_emb;
  a.n_ff = m->ff_l;
  a.hq = m->hq_l;
  a.head_dim = m->hd;
  a.group = m->group;
  a.rope_half = m->rope_half;
  a.xa = ws->x[0];
  a.xb = ws->x[1];
  a.y = ws->y;
  a.q = ws->q;
  a.attn = ws->attn;
  a.attn_d = ws->attn_d;
  a.attn_q = ws->attn_q;
  a.act = ws->act;
  a.act_d = ws->act_d;
  a.act_q = ws->act_q;
  a.part_o = ws->part_o;
  a.part_ml = ws->part_ml;
  a.rope_cos = s->rope_cos;
  a.rope_sin = s->rope_sin;
  a.io = ws->d_io;
  a.kv = state_kv(s);
  a.bar = ws->d_bar;
  a.nsub = ws->ps_nsub;
  a.fuse_quant = ws->ps_fuse ? 1 : 0;
  a.fuse_merge = ws->ps_fuse_merge ? 1 : 0;
  a.bpl = persist::barriers_per_layer(ws->ps_fuse, ws->ps_fuse_merge);
  a.res = ws->d_res;
  a.wait_ns = m->world > 1 ? WAIT_TIMEOUT_PEER_NS : WAIT_TIMEOUT_NS;
  if (ws->tp_p2p) {
    a.tp = tp_exchange(ws, 0);
  } else {
    a.tp = TpExchange{};
    a.tp.world = 1;
  }
  a.stamps = stamps;
  return a;
}

size_t persist_stamp_bytes(const l3g_workspace* ws) {
  return (size_t)persist::BARRIERS_PER_LAYER * ws->ps_plan.n_layers * ws->ps_plan.grid * 2 * 8;
}


// A cooperative launch: the driver guarantees every CTA of the grid is
// resident at once (the grid barriers between phases depend on it) or
// refuses the launch with cudaErrorCooperativeLaunchTooLarge.  No
// programmatic early launch for it: k_layers starts after k_embed ends.
cudaError_t launch_layers(const l3g_workspace* ws, const l3g_state* s,
                          unsigned long long* stamps, cudaStream_t st) {
  const l3g_model* m = ws->m;
  const PersistArgs a = persist_args(ws, s, stamps);
  int gp = 1;
  while (gp < m->group) gp <<= 1;
  void* kfn = layers_kernel(m, gp, ws->ps_fuse_merge);
  if (!kfn) return cudaErrorInvalidDeviceFunction;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ws->ps_plan.grid);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = ws->ps_smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* kargs[] = {(void*)&a};
  return cudaLaunchKernelExC(&cfg, kfn, kargs);
}

extern "C" int l3g_workspace_persistent(const l3g_workspace* ws, int32_t* on) {
  if (!ws || !on) return l3g_fail(L3G_E_INVALID, "null argument");
  *on = ws->ps_on ? 1 : 0;
  return L3G_OK;
}

extern "C" int l3g_persist_layout(const l3g_workspace* ws, int32_t* stages, int32_t* slot_bytes,
                                  int32_t* splits, int32_t* counters, int32_t* smem_bytes,
                                  int32_t* barriers_per_layer) {
  if (!ws || !stages || !slot_bytes || !splits || !counters || !smem_bytes || !barriers_per_layer)
    return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws->ps_on) return l3g_fail(L3G_E_INVALID, "the workspace does not run the persistent kernel");
  *stages = ws->ps_ns;
  *slot_bytes = ws->ps_slot;
  *splits = ws->ps_plan.splits;
  *counters = ws->ps_nsub;
  *smem_bytes = ws->ps_smem;
  *barriers_per_layer = persist::barriers_per_layer(ws->ps_fuse, ws->ps_fuse_merge);
  return L3G_OK;
}

extern "C" int l3g_persist_stamps(const l3g_workspace* ws, uint64_t* out, int64_t cap,
                                  int32_t* n_barriers, int32_t* grid) {
  if (!ws || !out || !n_barriers || !grid) return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws->ps_on) return l3g_fail(L3G_E_INVALID, "the workspace does not run the persistent kernel");
  const size_t bytes = persist_stamp_bytes(ws);
  if (kPersistStampOff * 8 + bytes > kTraceBytes)
    return l3g_fail(L3G_E_INVALID, "too many layers to stamp");
  if (cap < (int64_t)(bytes / 8)) return l3g_fail(L3G_E_INVALID, "capacity %lld < %zu", (long long)cap, bytes / 8);
  CUDA_TRY(cudaSetDevice(ws->device));
  CUDA_TRY(cudaMemcpy(out, ws->d_trace + kPersistStampOff, bytes, cudaMemcpyDeviceToHost));
  *n_barriers = persist::barriers_per_layer(ws->ps_fuse, ws->ps_fuse_merge) * ws->ps_plan.n_layers;
  *grid = ws->ps_plan.grid;
  return L3G_OK;
}

