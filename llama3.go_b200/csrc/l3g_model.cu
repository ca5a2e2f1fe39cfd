// Model upload and repack (tiled Q8_0 matrices), KV states and their
// snapshots.
#include "l3g_rt.h"

// ---------------------------------------------------------------------------
// tiled Q8_0 matrices
// ---------------------------------------------------------------------------

// Per-CTA cost of one tile on the bulk-copy path, in ns: a fixed ~250 ns per
// copy plus its bytes at ~100 GB/s (fitted on B200 with a streaming probe).
static double tile_cost_ns(int tile_bytes) { return 250.0 + tile_bytes / 100.0; }

static Q8Tiles make_tiles(int rows, int cols, int rpw) {
  const TileGeom g = tile_geometry(rows, cols, rpw, NW, TILE_TARGET);
  Q8Tiles t{};
  t.rows = rows;
  t.cols = cols;
  t.wr = g.wr;
  t.nslices = g.nslices;
  t.ck = g.ck;
  t.tile_bytes = g.tile_bytes;
  t.n_groups = g.n_groups;
  return t;
}

// Rows per warp: the layout whose busiest CTA (one CTA per SM) finishes
// first under tile_cost_ns, bounded below by the HBM time of the matrix.
// Ties (within 2%) go by the order 4, 2, 8, 1: in the fused decode step four
// rows per warp measured fastest, and one row per warp pays a cross-warp
// reduction per tile that the cost model does not see.
static Q8Tiles plan_tiles(int rows, int cols, int nsm) {
  // L3G_RPW=1|2|4|8 pins the rows per warp (a tuning knob for experiments)
  if (const char* env = getenv("L3G_RPW")) {
    const int rpw = atoi(env);
    if (rpw == 1 || rpw == 2 || rpw == 4 || rpw == 8) return make_tiles(rows, cols, rpw);
  }
  Q8Tiles best{};
  double best_t = 1e300;
  for (int rpw : {4, 2, 8, 1}) {
    const Q8Tiles t = make_tiles(rows, cols, rpw);
    const long long ntiles = (long long)t.n_groups * t.nslices;
    const long long grid = std::min<long long>(t.n_groups, nsm);
    const long long groups_per_cta = (t.n_groups + grid - 1) / grid;
    const double cta_ns = groups_per_cta * t.nslices * tile_cost_ns(t.tile_bytes);
    const double hbm_ns = (double)ntiles * t.tile_bytes / 7000.0;  // ~7 TB/s read
    const double tt = std::max(cta_ns, hbm_ns);
    if (tt < best_t * 0.98) {
      best_t = tt;
      best = t;
    }
  }
  return best;
}

// Stages: as many tiles as fit the per-CTA share (at least 2).
static void finish_plan(DevMat& m) {
  const int fixed = mv_smem_bytes(m.t.cols, 0, m.t.tile_bytes);
  m.nstages = std::max(2, std::min(MAX_STAGES, (CTA_SMEM_SHARE - fixed) / m.t.tile_bytes));
  m.smem = mv_smem_bytes(m.t.cols, m.nstages, m.t.tile_bytes);
}


// Uploads the needed source rows, repacks them into tiles on the device.
// rpw > 0 fixes the rows per warp (the persistent kernel's layout); 0 plans.
int upload_tiled(DevMat& out, const RowSrc* segs, int nseg, bool interleave2, int src_cols,
                 int blk0, int cols, int nsm, size_t* dev_bytes, int rpw) {
  int rows = 0;
  for (int i = 0; i < nseg; ++i) rows += segs[i].n;
  out.t = rpw > 0 ? make_tiles(rows, cols, rpw) : plan_tiles(rows, cols, nsm);
  finish_plan(out);
  out.bytes = (size_t)out.t.n_groups * out.t.nslices * out.t.tile_bytes;
  CUDA_TRY(cudaMalloc(&out.buf, out.bytes));
  out.t.data = out.buf;
  *dev_bytes += out.bytes;
  const size_t row_bytes = (size_t)(src_cols / 32) * 34;
  RepackArgs ra{};
  std::vector<uint8_t*> staging(nseg, nullptr);
  for (int i = 0; i < nseg; ++i) {
    const size_t nbytes = row_bytes * segs[i].n;
    CUDA_TRY(cudaMalloc(&staging[i], nbytes ? nbytes : 16));
    CUDA_TRY(cudaMemcpy(staging[i], segs[i].host + row_bytes * segs[i].row0,
                        nbytes, cudaMemcpyHostToDevice));
    ra.src[i] = staging[i];
    ra.src_row0[i] = 0;
    ra.seg_rows[i] = segs[i].n;
  }
  ra.nseg = nseg;
  ra.interleave2 = interleave2 ? 1 : 0;
  ra.src_blocks = src_cols / 32;
  ra.blk0 = blk0;
  ra.dst = out.t;
  ra.out = out.buf;
  k_repack<<<2048, 256>>>(ra);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  for (auto* p : staging) cudaFree(p);
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "repack: %s", cudaGetErrorString(e));
  return L3G_OK;
}



void free_gemm(GemmMat& g) {
  if (g.data) cudaFree(g.data);
  g = GemmMat{};
}


static const l3g_tensor* find_tensor(const l3g_tensor* ts, int n, const char* name) {
  for (int i = 0; i < n; ++i)
    if (ts[i].name && strcmp(ts[i].name, name) == 0) return &ts[i];
  return nullptr;
}

static int check_matrix(const l3g_tensor* t, const char* name, int cols, int rows) {
  if (!t) return l3g_fail(L3G_E_FORMAT, "missing tensor \"%s\"", name);
  if (t->type != L3G_TYPE_Q8_0)
    return l3g_fail(L3G_E_INVALID, "tensor \"%s\" has type %u, want Q8_0 (8)", name, t->type);
  if (t->n_dims != 2 || (int64_t)t->dims[0] != cols || (int64_t)t->dims[1] != rows)
    return l3g_fail(L3G_E_INVALID, "tensor \"%s\" dims [%llu %llu], want [%d %d]", name,
                    (unsigned long long)t->dims[0], (unsigned long long)t->dims[1], cols, rows);
  if (!t->data) return l3g_fail(L3G_E_INVALID, "tensor \"%s\" has no data", name);
  const uint64_t need = (uint64_t)rows * (cols / 32) * 34;
  if (t->nbytes && t->nbytes < need)
    return l3g_fail(L3G_E_INVALID, "tensor \"%s\" truncated", name);
  return L3G_OK;
}

// norm vectors: readVectorAnyToF32 (tensor_read.go:43-52), F32 or F16
static int upload_vector(const l3g_tensor* t, const char* name, int n, float** out,
                         size_t* dev_bytes) {
  if (!t) return l3g_fail(L3G_E_FORMAT, "missing tensor \"%s\"", name);
  std::vector<float> v(n);
  if (t->type == L3G_TYPE_F32) {
    if (t->nbytes && t->nbytes < (uint64_t)n * 4)
      return l3g_fail(L3G_E_INVALID, "tensor \"%s\" truncated", name);
    memcpy(v.data(), t->data, (size_t)n * 4);
  } else if (t->type == L3G_TYPE_F16) {
    if (t->nbytes && t->nbytes < (uint64_t)n * 2)
      return l3g_fail(L3G_E_INVALID, "tensor \"%s\" truncated", name);
    const uint16_t* h = static_cast<const uint16_t*>(t->data);
    for (int i = 0; i < n; ++i) v[i] = l3g_f16_to_f32(h[i]);
  } else {
    return l3g_fail(L3G_E_INVALID, "unsupported vector type %u for \"%s\"", t->type, name);
  }
  CUDA_TRY(cudaMalloc(out, (size_t)n * 4));
  CUDA_TRY(cudaMemcpy(*out, v.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  *dev_bytes += (size_t)n * 4;
  return L3G_OK;
}

void free_mat(DevMat& m) {
  if (m.buf) cudaFree(m.buf);
  m.buf = nullptr;
}


extern "C" void l3g_model_free(l3g_model* m) {
  if (!m) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  {
    std::lock_guard<std::mutex> lk(m->ws_mu);
    for (l3g_workspace* ws : m->workspaces) ws_detach(ws);
    m->workspaces.clear();
  }
  for (auto& L : m->layers) {
    free_mat(L.qkv);
    free_mat(L.wo);
    free_mat(L.upgate);
    free_mat(L.down);
    free_gemm(L.gqkv);
    free_gemm(L.gwo);
    free_gemm(L.gupgate);
    free_gemm(L.gdown);
    if (L.attn_norm) cudaFree(L.attn_norm);
    if (L.ffn_norm) cudaFree(L.ffn_norm);
  }
  free_mat(m->logits);
  free_gemm(m->glogits);
  if (m->d_layers) cudaFree(m->d_layers);
  if (m->out_norm) cudaFree(m->out_norm);
  if (m->emb) cudaFree(m->emb);
  if (m->comm) nccl()->CommDestroy(m->comm);
  cudaSetDevice(prev);
  delete m;
}

static int validate_hparams(const l3g_hparams& hp, int world) {
  if (hp.vocab_size <= 0 || hp.n_layers <= 0 || hp.n_emb <= 0 || hp.n_heads <= 0 ||
      hp.n_ff <= 0)
    return l3g_fail(L3G_E_FORMAT, "missing required llama.* hyperparams in gguf");
  if (hp.n_emb % hp.n_heads)
    return l3g_fail(L3G_E_INVALID, "n_emb %d not divisible by n_heads %d", hp.n_emb, hp.n_heads);
  const int hd = hp.n_emb / hp.n_heads;
  if (hd != 32 && hd != 64 && hd != 128)
    return l3g_fail(L3G_E_INVALID, "head_dim %d unsupported (32, 64 or 128)", hd);
  if (hp.n_heads_kv <= 0 || hp.n_heads % hp.n_heads_kv)
    return l3g_fail(L3G_E_INVALID, "n_heads %d not a multiple of n_heads_kv %d", hp.n_heads,
                    hp.n_heads_kv);
  if (hp.n_heads / hp.n_heads_kv > MAXG)
    return l3g_fail(L3G_E_INVALID, "GQA group %d above %d", hp.n_heads / hp.n_heads_kv, MAXG);
  if (hp.n_emb % 32 || hp.n_ff % 32)
    return l3g_fail(L3G_E_INVALID, "n_emb and n_ff must be multiples of 32");
  // the matvec prologues hold their input vector in registers
  if (hp.n_emb > 8192) return l3g_fail(L3G_E_INVALID, "n_emb %d above 8192", hp.n_emb);
  if (world >= 1 && hp.n_ff / world > 16384)
    return l3g_fail(L3G_E_INVALID, "n_ff per rank %d above 16384", hp.n_ff / world);
  if (hp.rope_dim <= 0 || hp.rope_dim > hd || hp.rope_dim % 2)
    return l3g_fail(L3G_E_INVALID, "rope_dim %d must be even and <= head_dim %d", hp.rope_dim, hd);
  if (hp.ctx_len <= 0) return l3g_fail(L3G_E_INVALID, "ctx_len %d", hp.ctx_len);
  if (world < 1) return l3g_fail(L3G_E_INVALID, "world_size %d", world);
  if (hp.n_heads % world || hp.n_heads_kv % world)
    return l3g_fail(L3G_E_INVALID, "heads %d/%d not divisible by %d ranks", hp.n_heads,
                    hp.n_heads_kv, world);
  if ((hp.n_heads / world * hd) % 32)
    return l3g_fail(L3G_E_INVALID, "per-rank attention width not a multiple of 32");
  if (hp.n_ff % (32 * world))
    return l3g_fail(L3G_E_INVALID, "n_ff %d not divisible into Q8_0 blocks over %d ranks",
                    hp.n_ff, world);
  return L3G_OK;
}

static void apply_hparam_defaults(l3g_hparams& hp) {
  if (hp.n_heads_kv == 0) hp.n_heads_kv = hp.n_heads;                       // model.go:212-214
  if (hp.rope_dim == 0 && hp.n_heads) hp.rope_dim = hp.n_emb / hp.n_heads;  // :215-217
}

extern "C" int l3g_shard_plan(const l3g_hparams* hp_in, int32_t world, int32_t rank,
                              l3g_shard* out) {
  if (!hp_in || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  l3g_hparams hp = *hp_in;
  apply_hparam_defaults(hp);
  int rc = validate_hparams(hp, world);
  if (rc) return rc;
  if (rank < 0 || rank >= world)
    return l3g_fail(L3G_E_INVALID, "rank %d outside world %d", rank, world);
  const int hd = hp.n_emb / hp.n_heads;
  const int hq = hp.n_heads / world, hkv = hp.n_heads_kv / world, ff = hp.n_ff / world;
  const int vl = (hp.vocab_size + world - 1) / world;
  l3g_shard s{};
  s.q_row0 = rank * hq * hd;
  s.q_rows = hq * hd;
  s.kv_row0 = rank * hkv * hd;
  s.kv_rows = hkv * hd;
  s.o_col0 = rank * hq * hd;
  s.o_cols = hq * hd;
  s.ff_row0 = rank * ff;
  s.ff_rows = ff;
  s.down_col0 = rank * ff;
  s.down_cols = ff;
  s.vocab_stride = vl;
  s.vocab_row0 = rank * vl;
  s.vocab_rows = std::min(hp.vocab_size, s.vocab_row0 + vl) - s.vocab_row0;
  if (s.vocab_rows < 1)
    return l3g_fail(L3G_E_INVALID, "vocab %d too small for %d ranks", hp.vocab_size, world);
  *out = s;
  return L3G_OK;
}

extern "C" int l3g_model_load(const l3g_hparams* hp_in, const l3g_tensor* ts, int32_t nt,
                              const l3g_options* opt_in, l3g_model** out) {
  if (!hp_in || !ts || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  l3g_options opt;
  if (opt_in)
    opt = *opt_in;
  else
    l3g_options_default(&opt);
  l3g_hparams hp = *hp_in;
  apply_hparam_defaults(hp);
  l3g_shard sh;
  int rc = l3g_shard_plan(&hp, opt.world_size, opt.rank, &sh);
  if (rc) return rc;
  if (opt.kv_dtype != L3G_KV_F32 && opt.kv_dtype != L3G_KV_F16)
    return l3g_fail(L3G_E_INVALID, "kv_dtype %d", opt.kv_dtype);
  if (opt.kv_dtype == L3G_KV_F16 && hp.n_emb / hp.n_heads < 64)
    return l3g_fail(L3G_E_INVALID, "f16 KV cache needs head_dim >= 64");

  int dev = opt.device;
  if (dev < 0) CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaSetDevice(dev));
  if ((rc = setup_kernels())) return rc;

  auto* m = new l3g_model();
  m->hp = hp;
  m->world = opt.world_size;
  m->rank = opt.rank;
  m->device = dev;
  m->kv_f16 = opt.kv_dtype == L3G_KV_F16;
  m->nsm = sm_count(dev);
  m->hd = hp.n_emb / hp.n_heads;
  m->hq_l = hp.n_heads / m->world;
  m->hkv_l = hp.n_heads_kv / m->world;
  m->group = hp.n_heads / hp.n_heads_kv;
  m->ff_l = hp.n_ff / m->world;
  m->v_l = sh.vocab_stride;
  m->v_off = sh.vocab_row0;
  m->rope_half = hp.rope_dim / 2;
  {
    const char* env = getenv("L3G_PERSIST");
    m->persist = env && atoi(env) == 1;
  }
  const int layer_rpw = m->persist ? 4 : 0;
  auto bail = [&](int code) {
    l3g_model_free(m);
    return code;
  };

  // RoPE inverse frequencies, NewRopeCache rope.go:20-25, divided by the
  // optional llama3 factors
  m->inv_freq.resize(m->rope_half);
  const l3g_tensor* rf = find_tensor(ts, nt, "rope_freqs.weight");
  if (rf && (rf->type != L3G_TYPE_F32 || rf->dims[0] < (uint64_t)m->rope_half))
    return bail(l3g_fail(L3G_E_INVALID, "rope_freqs.weight must be F32 [%d]", m->rope_half));
  for (int i = 0; i < m->rope_half; ++i) {
    const double e = (double)(2 * i) / (double)hp.rope_dim;
    m->inv_freq[i] = 1.0 / pow((double)hp.rope_base, e);
    if (rf) m->inv_freq[i] /= (double)static_cast<const float*>(rf->data)[i];
  }

  const int ne = hp.n_emb, hd = m->hd;
  char name[96];
  // embedding (all rows, raw, for the lookup) and output projection shard
  const l3g_tensor* emb = find_tensor(ts, nt, "token_embd.weight");
  if ((rc = check_matrix(emb, "token_embd.weight", ne, hp.vocab_size))) return bail(rc);
  const size_t emb_bytes = (size_t)hp.vocab_size * (ne / 32) * 34;
  if (cudaMalloc(&m->emb, emb_bytes) != cudaSuccess ||
      cudaMemcpy(m->emb, emb->data, emb_bytes, cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(l3g_fail(L3G_E_CUDA, "embedding upload failed"));
  m->dev_bytes += emb_bytes;
  const l3g_tensor* outp = find_tensor(ts, nt, "output.weight");
  if (!outp) outp = emb;  // tied, model.go:91-94
  else if ((rc = check_matrix(outp, "output.weight", ne, hp.vocab_size))) return bail(rc);
  {
    RowSrc seg{static_cast<const uint8_t*>(outp->data), sh.vocab_row0, sh.vocab_rows};
    if ((rc = upload_tiled(m->logits, &seg, 1, false, ne, 0, ne, m->nsm, &m->dev_bytes)))
      return bail(rc);
  }
  if ((rc = upload_vector(find_tensor(ts, nt, "output_norm.weight"), "output_norm.weight", ne,
                          &m->out_norm, &m->dev_bytes)))
    return bail(rc);

  m->layers.resize(hp.n_layers);
  const int kvdim = hp.n_heads_kv * hd;
  for (int l = 0; l < hp.n_layers; ++l) {
    LayerW& L = m->layers[l];
    auto T = [&](const char* suffix) {
      snprintf(name, sizeof name, "blk.%d.%s", l, suffix);
      return find_tensor(ts, nt, name);
    };
    auto chk = [&](const char* suffix, int cols, int rows) {
      snprintf(name, sizeof name, "blk.%d.%s", l, suffix);
      return check_matrix(find_tensor(ts, nt, name), name, cols, rows);
    };
    if ((rc = chk("attn_q.weight", ne, ne)) || (rc = chk("attn_k.weight", ne, kvdim)) ||
        (rc = chk("attn_v.weight", ne, kvdim)) || (rc = chk("attn_output.weight", ne, ne)) ||
        (rc = chk("ffn_up.weight", ne, hp.n_ff)) || (rc = chk("ffn_gate.weight", ne, hp.n_ff)) ||
        (rc = chk("ffn_down.weight", hp.n_ff, ne)))
      return bail(rc);
    const auto* wq = static_cast<const uint8_t*>(T("attn_q.weight")->data);
    const auto* wk = static_cast<const uint8_t*>(T("attn_k.weight")->data);
    const auto* wv = static_cast<const uint8_t*>(T("attn_v.weight")->data);
    const auto* wo = static_cast<const uint8_t*>(T("attn_output.weight")->data);
    const auto* wu = static_cast<const uint8_t*>(T("ffn_up.weight")->data);
    const auto* wg = static_cast<const uint8_t*>(T("ffn_gate.weight")->data);
    const auto* wd = static_cast<const uint8_t*>(T("ffn_down.weight")->data);
    // this rank's heads: q rows, k rows, v rows concatenated
    RowSrc qkv[3] = {{wq, sh.q_row0, sh.q_rows},
                     {wk, sh.kv_row0, sh.kv_rows},
                     {wv, sh.kv_row0, sh.kv_rows}};
    if ((rc = upload_tiled(L.qkv, qkv, 3, false, ne, 0, ne, m->nsm, &m->dev_bytes, layer_rpw)))
      return bail(rc);
    // Wo: all rows, this rank's head columns
    RowSrc wos{wo, 0, ne};
    if ((rc = upload_tiled(L.wo, &wos, 1, false, ne, sh.o_col0 / 32, sh.o_cols, m->nsm,
                           &m->dev_bytes, layer_rpw)))
      return bail(rc);
    // up/gate interleaved (up_i, gate_i) for this rank's FFN rows
    RowSrc ug[2] = {{wu, sh.ff_row0, sh.ff_rows}, {wg, sh.ff_row0, sh.ff_rows}};
    if ((rc = upload_tiled(L.upgate, ug, 2, true, ne, 0, ne, m->nsm, &m->dev_bytes, layer_rpw)))
      return bail(rc);
    // down: all rows, this rank's FFN columns
    RowSrc ds{wd, 0, ne};
    if ((rc = upload_tiled(L.down, &ds, 1, false, hp.n_ff, sh.down_col0 / 32, sh.down_cols,
                           m->nsm, &m->dev_bytes, layer_rpw)))
      return bail(rc);
    snprintf(name, sizeof name, "blk.%d.attn_norm.weight", l);
    if ((rc = upload_vector(find_tensor(ts, nt, name), name, ne, &L.attn_norm, &m->dev_bytes)))
      return bail(rc);
    snprintf(name, sizeof name, "blk.%d.ffn_norm.weight", l);
    if ((rc = upload_vector(find_tensor(ts, nt, name), name, ne, &L.ffn_norm, &m->dev_bytes)))
      return bail(rc);
  }

  if (m->persist) {  // the persistent kernel's table of layer pointers
    std::vector<PersistLayer> tab(hp.n_layers);
    for (int l = 0; l < hp.n_layers; ++l) {
      const LayerW& L = m->layers[l];
      tab[l].w[persist::M_QKV] = L.qkv.buf;
      tab[l].w[persist::M_WO] = L.wo.buf;
      tab[l].w[persist::M_UPGATE] = L.upgate.buf;
      tab[l].w[persist::M_DOWN] = L.down.buf;
      tab[l].attn_norm = L.attn_norm;
      tab[l].ffn_norm = L.ffn_norm;
    }
    const size_t nb = tab.size() * sizeof(PersistLayer);
    if (cudaMalloc(&m->d_layers, nb) != cudaSuccess ||
        cudaMemcpy(m->d_layers, tab.data(), nb, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(l3g_fail(L3G_E_CUDA, "layer table upload failed"));
  }

  if (m->world > 1) {
    NcclApi* api = nccl();
    if (!api->ok) return bail(l3g_fail(L3G_E_NCCL, "libnccl.so.2 not found"));
    ncclUniqueId id;
    memcpy(&id, opt.nccl_id, sizeof id);
    ncclResult_t r = api->CommInitRank(&m->comm, m->world, id, m->rank);
    if (r != ncclSuccess)
      return bail(l3g_fail(L3G_E_NCCL, "ncclCommInitRank: %s", api->GetErrorString(r)));
  }
  *out = m;
  return L3G_OK;
}

extern "C" int l3g_model_hparams(const l3g_model* m, l3g_hparams* out) {
  if (!m || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = m->hp;
  return L3G_OK;
}


static uint64_t next_serial() {
  static std::mutex mu;
  static uint64_t s = 0;
  std::lock_guard<std::mutex> g(mu);
  return ++s;
}

// ---------------------------------------------------------------------------
// paged KV cache: pools of pages, page tables
// ---------------------------------------------------------------------------
static_assert(L3G_KV_PAGE == KV_PAGE, "page size of the ABI and the kernels");
static size_t kv_row_bytes(const l3g_model* m) { return (size_t)2 * m->hd * (m->kv_f16 ? 2 : 4); }
static size_t kv_page_bytes(const l3g_model* m) { return (size_t)KV_PAGE * kv_row_bytes(m); }

static int pool_create(l3g_model* m, int n_pages, bool priv, l3g_kvpool** out) {
  *out = nullptr;
  if (n_pages <= 0) return l3g_fail(L3G_E_INVALID, "a KV pool needs at least one page, got %d", n_pages);
  auto* p = new l3g_kvpool();
  p->m = m;
  p->device = m->device;
  p->n_pages = n_pages;
  p->page_bytes = kv_page_bytes(m);
  p->priv = priv;
  const size_t bytes = p->page_bytes * (size_t)n_pages;
  cudaError_t e = cudaMalloc(&p->base, bytes);
  if (e == cudaSuccess) e = cudaMemset(p->base, 0, bytes);
  if (e != cudaSuccess) {
    if (p->base) cudaFree(p->base);
    delete p;
    cudaGetLastError();
    return l3g_fail(L3G_E_CUDA, "KV pool of %d pages (%llu bytes): %s", n_pages,
                    (unsigned long long)bytes, cudaGetErrorString(e));
  }
  if (!priv) {  // a stack: the lowest ids come out first
    p->free_pages.resize(n_pages);
    for (int i = 0; i < n_pages; ++i) p->free_pages[i] = n_pages - 1 - i;
  }
  *out = p;
  return L3G_OK;
}

static void pool_destroy(l3g_kvpool* p) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  if (p->base) cudaFree(p->base);
  cudaSetDevice(prev);
  delete p;
}

// A state leaves its pool: its pages go back on the free list; a released
// (or private) pool without states is destroyed.
static void pool_leave(l3g_kvpool* p, const std::vector<int>& pages) {
  bool destroy = false;
  {
    std::lock_guard<std::mutex> lk(p->mu);
    if (!p->priv)
      for (int id : pages)
        if (id >= 0) p->free_pages.push_back(id);
    --p->states;
    destroy = p->priv || (p->released && p->states == 0);
  }
  if (destroy) pool_destroy(p);
}

KvMap state_kv(const l3g_state* s) {
  KvMap k{};
  k.pool = s->pool->base;
  k.pages = s->d_pages;
  k.pps = s->pps;
  k.hkv = s->m->hkv_l;
  k.row_bytes = (int)kv_row_bytes(s->m);
  return k;
}

int state_map(l3g_state* s, int n_pos, cudaStream_t st) {
  const int need = std::min(s->pps, (n_pos + KV_PAGE - 1) / KV_PAGE);
  if (need <= s->mapped) return L3G_OK;
  const int heads = s->m->hp.n_layers * s->m->hkv_l;
  l3g_kvpool* p = s->pool;
  {
    std::lock_guard<std::mutex> lk(p->mu);
    const size_t want = (size_t)heads * (need - s->mapped);
    if (p->free_pages.size() < want)
      return l3g_fail(L3G_E_CTX, "KV pool exhausted: %zu free pages, %zu needed for position %d",
                      p->free_pages.size(), want, n_pos - 1);
    for (int j = s->mapped; j < need; ++j)
      for (int h = 0; h < heads; ++h) {
        s->h_pages[(size_t)h * s->pps + j] = p->free_pages.back();
        p->free_pages.pop_back();
      }
  }
  // the new entries of every (layer, kv head): one 2-D copy (pageable
  // source: staged before the call returns)
  CUDA_TRY(cudaMemcpy2DAsync(s->d_pages + s->mapped, (size_t)s->pps * sizeof(int),
                             s->h_pages.data() + s->mapped, (size_t)s->pps * sizeof(int),
                             (size_t)(need - s->mapped) * sizeof(int), (size_t)heads,
                             cudaMemcpyHostToDevice, st));
  s->mapped = need;
  return L3G_OK;
}

extern "C" int l3g_kvpool_page_bytes(const l3g_model* m, uint64_t* bytes) {
  if (!m || !bytes) return l3g_fail(L3G_E_INVALID, "null argument");
  *bytes = kv_page_bytes(m);
  return L3G_OK;
}

extern "C" int l3g_kvpool_new(l3g_model* m, int32_t n_pages, l3g_kvpool** out) {
  if (!m || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(m->device));
  return pool_create(m, n_pages, false, out);
}

extern "C" void l3g_kvpool_free(l3g_kvpool* p) {
  if (!p) return;
  bool destroy;
  {
    std::lock_guard<std::mutex> lk(p->mu);
    p->released = true;
    destroy = p->states == 0;
  }
  if (destroy) pool_destroy(p);
}

extern "C" int l3g_kvpool_free_pages(l3g_kvpool* p, int32_t* n) {
  if (!p || !n) return l3g_fail(L3G_E_INVALID, "null argument");
  std::lock_guard<std::mutex> lk(p->mu);
  *n = (int32_t)p->free_pages.size();
  return L3G_OK;
}

extern "C" void l3g_state_free(l3g_state* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  if (s->d_pages) cudaFree(s->d_pages);
  if (s->rope_cos) cudaFree(s->rope_cos);
  if (s->rope_sin) cudaFree(s->rope_sin);
  if (s->pool) pool_leave(s->pool, s->h_pages);
  delete s;
}

// A state over `pool` (nullptr: a private pool of exactly its pages, mapped
// at once, page j of (layer, kv head) h at pool page h * pps + j).
static int state_create(l3g_model* m, l3g_kvpool* pool, int32_t ctx, l3g_state** out) {
  if (!m || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  if (pool && pool->m != m) return l3g_fail(L3G_E_INVALID, "KV pool of another model");
  if (ctx <= 0) ctx = m->hp.ctx_len;  // state.go:52-57
  if (ctx > m->hp.ctx_len) ctx = m->hp.ctx_len;
  CUDA_TRY(cudaSetDevice(m->device));
  auto* s = new l3g_state();
  s->m = m;
  s->device = m->device;
  s->ctx = ctx;
  s->serial = next_serial();
  s->pps = (ctx + KV_PAGE - 1) / KV_PAGE;
  const int heads = m->hp.n_layers * m->hkv_l;
  s->h_pages.assign((size_t)heads * s->pps, -1);
  cudaError_t e = cudaMalloc(&s->d_pages, s->h_pages.size() * sizeof(int));
  if (e != cudaSuccess) {
    l3g_state_free(s);
    return l3g_fail(L3G_E_CUDA, "state allocation: %s", cudaGetErrorString(e));
  }
  if (pool) {
    {
      std::lock_guard<std::mutex> lk(pool->mu);
      if (pool->released) {
        l3g_state_free(s);
        return l3g_fail(L3G_E_INVALID, "KV pool already freed");
      }
      ++pool->states;
    }
    s->pool = pool;
    // unmapped entries point at page 0 until mapped: never read, since a
    // step maps its position's pages before it runs
    e = cudaMemset(s->d_pages, 0, s->h_pages.size() * sizeof(int));
  } else {
    l3g_kvpool* own = nullptr;
    if (int rc = pool_create(m, heads * s->pps, true, &own)) {
      l3g_state_free(s);
      return rc;
    }
    own->states = 1;
    s->pool = own;
    for (size_t i = 0; i < s->h_pages.size(); ++i) s->h_pages[i] = (int)i;
    s->mapped = s->pps;
    e = cudaMemcpy(s->d_pages, s->h_pages.data(), s->h_pages.size() * sizeof(int),
                   cudaMemcpyHostToDevice);
  }
  // RoPE tables, NewRopeCache rope.go:27-34 (f64 angles, f32 tables)
  const int half = m->rope_half;
  std::vector<float> c((size_t)ctx * half), sn((size_t)ctx * half);
  for (int p = 0; p < ctx; ++p)
    for (int i = 0; i < half; ++i) {
      const double ang = (double)p * m->inv_freq[i];
      c[(size_t)p * half + i] = (float)cos(ang);
      sn[(size_t)p * half + i] = (float)sin(ang);
    }
  const size_t tb = std::max<size_t>(4, c.size() * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->rope_cos, tb);
  if (e == cudaSuccess) e = cudaMalloc(&s->rope_sin, tb);
  if (e == cudaSuccess && !c.empty())
    e = cudaMemcpy(s->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !sn.empty())
    e = cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    l3g_state_free(s);
    return l3g_fail(L3G_E_CUDA, "state allocation: %s", cudaGetErrorString(e));
  }
  *out = s;
  return L3G_OK;
}

extern "C" int l3g_state_new(l3g_model* m, int32_t ctx, l3g_state** out) {
  return state_create(m, nullptr, ctx, out);
}

extern "C" int l3g_state_new_in_pool(l3g_model* m, l3g_kvpool* pool, int32_t ctx,
                                     l3g_state** out) {
  if (!pool) return l3g_fail(L3G_E_INVALID, "null argument");
  return state_create(m, pool, ctx, out);
}

extern "C" int l3g_state_pages(const l3g_state* s, int32_t* mapped) {
  if (!s || !mapped) return l3g_fail(L3G_E_INVALID, "null argument");
  *mapped = s->pool->priv ? 0 : s->mapped * s->m->hp.n_layers * s->m->hkv_l;
  return L3G_OK;
}

// Copies rows [pos0, pos0 + n) of (layer, kv head) between the cache and
// host memory (to_host: cache -> host), one copy per run of pages that are
// consecutive in the pool.
static int copy_rows(const l3g_state* s, int layer, int kvh, int pos0, int n, uint8_t* host,
                     bool to_host) {
  const size_t rb = kv_row_bytes(s->m);
  const size_t h = (size_t)layer * s->m->hkv_l + kvh;
  const KvMap km = state_kv(s);
  int p = pos0;
  while (p < pos0 + n) {
    const int page = s->h_pages[h * s->pps + p / KV_PAGE];
    if (page < 0) return l3g_fail(L3G_E_INVALID, "position %d of the state is not mapped", p);
    int q = std::min(pos0 + n, (p / KV_PAGE + 1) * KV_PAGE);
    while (q < pos0 + n && s->h_pages[h * s->pps + q / KV_PAGE] ==
                               page + (q / KV_PAGE - p / KV_PAGE))
      q = std::min(pos0 + n, (q / KV_PAGE + 1) * KV_PAGE);
    uint8_t* dev = s->pool->base + kv_page_byte(km, page, p);
    uint8_t* hp = host + (size_t)(p - pos0) * rb;
    if (to_host)
      CUDA_TRY(cudaMemcpy(hp, dev, (size_t)(q - p) * rb, cudaMemcpyDeviceToHost));
    else
      CUDA_TRY(cudaMemcpy(dev, hp, (size_t)(q - p) * rb, cudaMemcpyHostToDevice));
    p = q;
  }
  return L3G_OK;
}

extern "C" int l3g_state_pos(const l3g_state* s, int32_t* pos) {
  if (!s || !pos) return l3g_fail(L3G_E_INVALID, "null argument");
  *pos = s->pos;
  return L3G_OK;
}
extern "C" int l3g_state_ctx_len(const l3g_state* s, int32_t* ctx) {
  if (!s || !ctx) return l3g_fail(L3G_E_INVALID, "null argument");
  *ctx = s->ctx;
  return L3G_OK;
}
extern "C" int l3g_state_set_pos(l3g_state* s, int32_t pos) {
  if (!s) return l3g_fail(L3G_E_INVALID, "null argument");
  if (pos < 0 || pos > s->ctx) return l3g_fail(L3G_E_INVALID, "pos %d outside [0, %d]", pos, s->ctx);
  s->pos = pos;
  return L3G_OK;
}

// Snapshot layout: SnapHeader, then for each layer and local kv head the
// interleaved K|V rows of positions [0, pos) (the device layout's prefix).
struct SnapHeader {
  char magic[8];  // "L3GKV1\0\0"
  int32_t n_layers, n_emb, n_heads, n_heads_kv, world, rank, hkv_l, hd, elem_bytes, pos;
};

static bool snap_header(const l3g_state* s, SnapHeader* h) {
  const l3g_model* m = s->m;
  memset(h, 0, sizeof *h);
  memcpy(h->magic, "L3GKV1", 6);
  h->n_layers = m->hp.n_layers;
  h->n_emb = m->hp.n_emb;
  h->n_heads = m->hp.n_heads;
  h->n_heads_kv = m->hp.n_heads_kv;
  h->world = m->world;
  h->rank = m->rank;
  h->hkv_l = m->hkv_l;
  h->hd = m->hd;
  h->elem_bytes = m->kv_f16 ? 2 : 4;
  h->pos = s->pos;
  return true;
}

static size_t snap_bytes(const SnapHeader& h) {
  return sizeof(SnapHeader) +
         (size_t)h.n_layers * h.hkv_l * h.pos * 2 * h.hd * (size_t)h.elem_bytes;
}

extern "C" int l3g_state_snapshot_bytes(const l3g_state* s, uint64_t* bytes) {
  if (!s || !bytes) return l3g_fail(L3G_E_INVALID, "null argument");
  SnapHeader h;
  snap_header(s, &h);
  *bytes = snap_bytes(h);
  return L3G_OK;
}

extern "C" int l3g_state_snapshot(const l3g_state* s, void* dst, uint64_t bytes) {
  if (!s || !dst) return l3g_fail(L3G_E_INVALID, "null argument");
  SnapHeader h;
  snap_header(s, &h);
  if (bytes < snap_bytes(h))
    return l3g_fail(L3G_E_INVALID, "snapshot buffer of %llu bytes, need %llu",
                    (unsigned long long)bytes, (unsigned long long)snap_bytes(h));
  memcpy(dst, &h, sizeof h);
  if (h.pos == 0) return L3G_OK;
  CUDA_TRY(cudaSetDevice(s->device));
  CUDA_TRY(cudaDeviceSynchronize());  // steps in flight on any stream
  const size_t row = (size_t)h.pos * 2 * h.hd * h.elem_bytes;  // one (layer, kv head)
  uint8_t* out = static_cast<uint8_t*>(dst) + sizeof h;
  for (int l = 0; l < h.n_layers; ++l)
    for (int k = 0; k < h.hkv_l; ++k)
      if (int rc = copy_rows(s, l, k, 0, h.pos, out + ((size_t)l * h.hkv_l + k) * row, true))
        return rc;
  return L3G_OK;
}

extern "C" int l3g_state_restore(l3g_state* s, const void* src, uint64_t bytes) {
  if (!s || !src) return l3g_fail(L3G_E_INVALID, "null argument");
  if (bytes < sizeof(SnapHeader)) return l3g_fail(L3G_E_FORMAT, "snapshot too short");
  SnapHeader h, mine;
  memcpy(&h, src, sizeof h);
  snap_header(s, &mine);
  if (memcmp(h.magic, mine.magic, 8) != 0) return l3g_fail(L3G_E_FORMAT, "not a KV snapshot");
  if (h.n_layers != mine.n_layers || h.n_emb != mine.n_emb || h.n_heads != mine.n_heads ||
      h.n_heads_kv != mine.n_heads_kv || h.world != mine.world || h.rank != mine.rank ||
      h.hkv_l != mine.hkv_l || h.hd != mine.hd || h.elem_bytes != mine.elem_bytes)
    return l3g_fail(L3G_E_INVALID, "snapshot of another model shape, shard or KV type");
  if (h.pos < 0 || h.pos > s->ctx)
    return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  if (bytes < snap_bytes(h)) return l3g_fail(L3G_E_FORMAT, "snapshot truncated");
  if (h.pos > 0) {
    CUDA_TRY(cudaSetDevice(s->device));
    if (int rc = state_map(s, h.pos, 0)) return rc;
    CUDA_TRY(cudaDeviceSynchronize());  // the table copy and steps in flight
    const size_t row = (size_t)h.pos * 2 * h.hd * h.elem_bytes;
    uint8_t* in = const_cast<uint8_t*>(static_cast<const uint8_t*>(src)) + sizeof h;
    for (int l = 0; l < h.n_layers; ++l)
      for (int k = 0; k < h.hkv_l; ++k)
        if (int rc = copy_rows(s, l, k, 0, h.pos, in + ((size_t)l * h.hkv_l + k) * row, false))
          return rc;
  }
  s->pos = h.pos;
  return L3G_OK;
}

extern "C" int l3g_state_read_kv(const l3g_state* s, int32_t layer, int32_t pos0, int32_t npos,
                                 float* k_out, float* v_out) {
  if (!s || !k_out || !v_out) return l3g_fail(L3G_E_INVALID, "null argument");
  const l3g_model* m = s->m;
  if (layer < 0 || layer >= m->hp.n_layers || pos0 < 0 || npos < 0 || pos0 + npos > s->ctx)
    return l3g_fail(L3G_E_INVALID, "kv range out of bounds");
  if ((pos0 + npos + KV_PAGE - 1) / KV_PAGE > s->mapped)
    return l3g_fail(L3G_E_INVALID, "kv range not mapped (positions up to %d)", s->mapped * KV_PAGE);
  CUDA_TRY(cudaSetDevice(m->device));
  CUDA_TRY(cudaDeviceSynchronize());  // steps in flight on any stream
  const int hd = m->hd, nh = m->hkv_l;
  const size_t es = m->kv_f16 ? 2 : 4;
  std::vector<uint8_t> buf((size_t)npos * 2 * hd * es);
  for (int h = 0; h < nh; ++h) {
    if (int rc = copy_rows(s, layer, h, pos0, npos, buf.data(), true)) return rc;
    for (int p = 0; p < npos; ++p)
      for (int d = 0; d < hd; ++d) {
        const size_t ks = (size_t)p * 2 * hd + d, vs = ks + hd;
        const size_t dst = ((size_t)p * nh + h) * hd + d;
        if (es == 4) {
          k_out[dst] = reinterpret_cast<float*>(buf.data())[ks];
          v_out[dst] = reinterpret_cast<float*>(buf.data())[vs];
        } else {
          k_out[dst] = l3g_f16_to_f32(reinterpret_cast<uint16_t*>(buf.data())[ks]);
          v_out[dst] = l3g_f16_to_f32(reinterpret_cast<uint16_t*>(buf.data())[vs]);
        }
      }
  }
  return L3G_OK;
}

