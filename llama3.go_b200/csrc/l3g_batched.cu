// The tensor-core batched product, batched prefill and batched decode.
#include "l3g_rt.h"


// ---------------------------------------------------------------------------
// batched Q8_0 product on the tensor cores (tcgen05 kind::i8)
// ---------------------------------------------------------------------------
// K split of a product with few (row tile, token tile) tiles: the largest
// divisor of the chunk count that keeps the units within the CTA slots (SMs
// times CTAs per SM) and the partial sums within part_floats (1: no split).
static int gemm_ksplit(const GemmMat& w, int n_tok, int slots, size_t part_floats) {
  const int nt = gemm::token_tile(n_tok);
  const long long tiles = (long long)w.n_rt * ((n_tok + nt - 1) / nt);
  if (part_floats == 0 || tiles >= slots) return 1;
  const long long want = slots / tiles;
  int best = 1;
  for (int d = 2; d <= w.nk && d <= want; ++d)
    if (w.nk % d == 0 && (size_t)d * n_tok * w.rows <= part_floats) best = d;
  return best;
}
// Partial-sum floats that gemm_ksplit can ask of matrix w for up to cap tokens.
static size_t gemm_part_bound(const GemmMat& w, int cap, int nsm) {
  if (!w.data) return 0;
  // the most CTA slots any token tile gets (two per SM at 64 tokens)
  const int slots = nsm * 2;
  const long long d = std::min<long long>(w.nk, std::max(1, slots / std::max(1, w.n_rt)));
  return d > 1 ? (size_t)d * cap * w.rows : 0;
}

// One batched product out[n][r] (n < n_tok) on stream st: at most the CTAs
// that fit at once (one per SM, two at 64 tokens), work units dealt
// round-robin; with few tiles the K range is split over more CTAs (partial
// sums in part, then k_gemm_reduce).
static cudaError_t launch_gemm(const GemmMat& w, const uint8_t* act, int n_tok, float* out,
                               Result* res, unsigned long long wait_ns, int nsm,
                               cudaStream_t st, int ldo = 0, float* part = nullptr,
                               size_t part_floats = 0) {
  const int nt = gemm::token_tile(n_tok);
  const int slots = nsm * gemm::ctas_per_sm(nt);  // CTAs resident at once
  GemmArgs g{};
  g.a = w.data;
  g.b = act;
  g.out = out;
  g.rows = w.rows;
  g.ldo = ldo > 0 ? ldo : w.rows;
  g.n_tok = n_tok;
  g.nk = w.nk;
  g.n_rt = w.n_rt;
  g.n_tt = (n_tok + nt - 1) / nt;
  g.ksplit = part ? gemm_ksplit(w, n_tok, slots, part_floats) : 1;
  g.part = part;
  g.nstages = gemm::stages(nt);
  g.res = res;
  g.wait_ns = wait_ns;
  const long long units = (long long)g.n_rt * g.n_tt * g.ksplit;
  const int grid = (int)std::max<long long>(1, std::min<long long>(slots, units));
  switch (nt) {
    case 16: k_gemm_q8<16><<<grid, gemm_threads(16), gemm::smem_bytes(16), st>>>(g); break;
    case 32: k_gemm_q8<32><<<grid, gemm_threads(32), gemm::smem_bytes(32), st>>>(g); break;
    case 64: k_gemm_q8<64><<<grid, gemm_threads(64), gemm::smem_bytes(64), st>>>(g); break;
    default: k_gemm_q8<128><<<grid, gemm_threads(128), gemm::smem_bytes(128), st>>>(g); break;
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && g.ksplit > 1) {
    const long long n = (long long)n_tok * w.rows;
    k_gemm_reduce<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, g.ksplit, n_tok, w.rows,
                                                               g.ldo, out);
    e = cudaGetLastError();
  }
  return e;
}

struct l3g_gemm_matrix {
  GemmMat w;                // weight chunks, gemm::A_CHUNK bytes each
  int device = 0, nsm = 1;
  Result* d_res = nullptr;  // device error word of the kernel's bounded waits
  float* part = nullptr;    // split-K partial sums for up to 128 tokens
  size_t part_floats = 0;
};

// Kernel attributes of the batched product, once per device (kept apart from
// the decode kernels' set-up).
static int gemm_setup() {
  static int rcs[64];
  static std::once_flag onces[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return l3g_fail(L3G_E_CUDA, "gemm set-up: no current device");
  int& rc = rcs[dev];
  std::call_once(onces[dev], [&rc] {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_q8<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemm::smem_bytes(16));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_gemm_q8<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               gemm::smem_bytes(32));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_gemm_q8<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               gemm::smem_bytes(64));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_gemm_q8<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               gemm::smem_bytes(128));
#define SETPF(HD, KT)                                                                       \
  if (e == cudaSuccess)                                                                    \
  e = cudaFuncSetAttribute(k_pf_attention<HD, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           pf_attention_smem(HD))
    SETPF(32, float);
    SETPF(64, float);
    SETPF(128, float);
    SETPF(32, __half);
    SETPF(64, __half);
    SETPF(128, __half);
#undef SETPF
#define SETBD(HD, GP, KT)                                                                  \
  if (e == cudaSuccess)                                                                    \
  e = cudaFuncSetAttribute(k_bd_attention<HD, GP, KT>,                                     \
                           cudaFuncAttributeMaxDynamicSharedMemorySize,                    \
                           bd_smem_bytes(HD, (int)sizeof(KT), GP))
#define SETBD_G(HD, KT) \
  SETBD(HD, 1, KT);     \
  SETBD(HD, 2, KT);     \
  SETBD(HD, 4, KT);     \
  SETBD(HD, 8, KT)
    SETBD_G(32, float);
    SETBD_G(64, float);
    SETBD_G(128, float);
    SETBD_G(32, __half);
    SETBD_G(64, __half);
    SETBD_G(128, __half);
#undef SETBD_G
#undef SETBD
    rc = e == cudaSuccess ? L3G_OK
                          : l3g_fail(L3G_E_CUDA, "gemm kernel attributes: %s", cudaGetErrorString(e));
  });
  return rc ? l3g_fail(L3G_E_CUDA, "gemm kernel set-up failed on device %d", dev) : L3G_OK;
}

extern "C" int l3g_gemm_matrix_bytes(int32_t rows, int32_t cols, uint64_t* bytes) {
  if (!bytes) return l3g_fail(L3G_E_INVALID, "null argument");
  if (rows <= 0 || cols <= 0 || cols % 32)
    return l3g_fail(L3G_E_INVALID, "gemm: %d x %d is not a Q8_0 matrix (cols multiple of 32)",
                    rows, cols);
  *bytes = (uint64_t)gemm::row_tiles(rows) * gemm::chunks(cols) * gemm::A_CHUNK;
  return L3G_OK;
}

// Host-side repack of GGUF Q8_0 rows (34-byte blocks: fp16 d, 32 int8) into
// weight chunks; values unchanged, padding rows and blocks zero.
extern "C" int l3g_gemm_repack(const void* q8, int32_t rows, int32_t cols, void* dst,
                               uint64_t dst_bytes) {
  if (!q8 || !dst) return l3g_fail(L3G_E_INVALID, "null argument");
  uint64_t need = 0;
  if (int rc = l3g_gemm_matrix_bytes(rows, cols, &need)) return rc;
  if (dst_bytes < need)
    return l3g_fail(L3G_E_INVALID, "gemm repack needs %llu bytes, got %llu",
                    (unsigned long long)need, (unsigned long long)dst_bytes);
  using namespace gemm;
  const uint8_t* src = static_cast<const uint8_t*>(q8);
  uint8_t* out = static_cast<uint8_t*>(dst);
  std::memset(out, 0, need);
  const size_t row_bytes = (size_t)cols / QBLK * 34;
  const int nk = chunks(cols), nrt = row_tiles(rows), nblk = cols / QBLK;
  for (int rt = 0; rt < nrt; ++rt)
    for (int c = 0; c < nk; ++c) {
      uint8_t* ch = out + ((size_t)rt * nk + c) * A_CHUNK;
      for (int m = 0; m < TILE_M; ++m) {
        const int row = rt * TILE_M + m;
        if (row >= rows) break;
        for (int j = 0; j < BPC; ++j) {
          const int b = c * BPC + j;
          if (b >= nblk) break;
          const uint8_t* blk = src + (size_t)row * row_bytes + (size_t)b * 34;
          std::memcpy(ch + A_Q_BYTES + (j * TILE_M + m) * 2, blk, 2);
          std::memcpy(ch + q_offset(TILE_M, m, j * QBLK), blk + 2, 16);
          std::memcpy(ch + q_offset(TILE_M, m, j * QBLK + 16), blk + 18, 16);
        }
      }
    }
  return L3G_OK;
}

extern "C" void l3g_gemm_matrix_free(l3g_gemm_matrix* w) {
  if (!w) return;
  cudaSetDevice(w->device);
  free_gemm(w->w);
  if (w->d_res) cudaFree(w->d_res);
  if (w->part) cudaFree(w->part);
  delete w;
}

extern "C" int l3g_gemm_matrix_upload(const void* q8, int32_t rows, int32_t cols, int32_t device,
                                      l3g_gemm_matrix** out) {
  if (!q8 || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  uint64_t bytes = 0;
  if (int rc = l3g_gemm_matrix_bytes(rows, cols, &bytes)) return rc;
  int dev = device;
  if (dev < 0) CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaSetDevice(dev));
  if (int rc = gemm_setup()) return rc;
  std::vector<uint8_t> host(bytes);
  if (int rc = l3g_gemm_repack(q8, rows, cols, host.data(), bytes)) return rc;
  auto* w = new l3g_gemm_matrix();
  w->w.rows = rows;
  w->w.cols = cols;
  w->w.nk = gemm::chunks(cols);
  w->w.n_rt = gemm::row_tiles(rows);
  w->w.bytes = bytes;
  w->device = dev;
  w->nsm = sm_count(dev);
  cudaError_t e = cudaMalloc(&w->w.data, bytes);
  if (e == cudaSuccess) e = cudaMemcpy(w->w.data, host.data(), bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&w->d_res, sizeof(Result));
  if (e == cudaSuccess) e = cudaMemset(w->d_res, 0, sizeof(Result));
  // a matrix with fewer row tiles than SMs splits K over CTAs
  w->part_floats = gemm_part_bound(w->w, 128, w->nsm);
  if (e == cudaSuccess && w->part_floats) e = cudaMalloc(&w->part, w->part_floats * sizeof(float));
  if (e != cudaSuccess) {
    l3g_gemm_matrix_free(w);
    return l3g_fail(L3G_E_CUDA, "gemm matrix upload: %s", cudaGetErrorString(e));
  }
  *out = w;
  return L3G_OK;
}

extern "C" int l3g_gemm_act_bytes(int32_t n_tok, int32_t cols, uint64_t* bytes) {
  if (!bytes) return l3g_fail(L3G_E_INVALID, "null argument");
  if (n_tok <= 0 || cols <= 0 || cols % 32)
    return l3g_fail(L3G_E_INVALID, "gemm activations: n_tok=%d cols=%d", n_tok, cols);
  const int nt = gemm::token_tile(n_tok);
  *bytes = (uint64_t)((n_tok + nt - 1) / nt) * gemm::chunks(cols) * gemm::b_chunk(nt);
  return L3G_OK;
}

extern "C" int l3g_gemm_quantize(const float* x, int32_t n_tok, int32_t cols, void* act,
                                 void* stream) {
  if (!x || !act) return l3g_fail(L3G_E_INVALID, "null argument");
  uint64_t bytes = 0;
  if (int rc = l3g_gemm_act_bytes(n_tok, cols, &bytes)) return rc;
  if (((uintptr_t)x & 3) || ((uintptr_t)act & 15))
    return l3g_fail(L3G_E_INVALID, "x must be 4-byte aligned, act 16-byte");
  const int nt = gemm::token_tile(n_tok);
  const int n_pad = (n_tok + nt - 1) / nt * nt;
  const int nk = gemm::chunks(cols);
  const long long warps = (long long)n_pad * nk * gemm::BPC;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  if (blocks > INT_MAX) return l3g_fail(L3G_E_INVALID, "gemm activations too large");
  k_gemm_quantize<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      x, n_tok, cols, nt, nk, n_pad, static_cast<uint8_t*>(act));
  CUDA_TRY(cudaGetLastError());
  return L3G_OK;
}

extern "C" int l3g_gemm_q8(const l3g_gemm_matrix* w, const void* act, int32_t n_tok, float* out,
                           void* stream) {
  if (!w || !act || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  if (n_tok <= 0) return l3g_fail(L3G_E_INVALID, "n_tok=%d", n_tok);
  if (((uintptr_t)act & 15) || ((uintptr_t)out & 3))
    return l3g_fail(L3G_E_INVALID, "act must be 16-byte aligned, out 4-byte");
  CUDA_TRY(cudaSetDevice(w->device));
  if (int rc = gemm_setup()) return rc;
  CUDA_TRY(launch_gemm(w->w, static_cast<const uint8_t*>(act), n_tok, out, w->d_res,
                       WAIT_TIMEOUT_NS, w->nsm, (cudaStream_t)stream, 0, w->part,
                       w->part_floats));
  return L3G_OK;
}

extern "C" int l3g_gemm_status(const l3g_gemm_matrix* w, int32_t* err, int32_t* where) {
  if (!w || !err || !where) return l3g_fail(L3G_E_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(w->device));
  CUDA_TRY(cudaDeviceSynchronize());
  Result h{};
  CUDA_TRY(cudaMemcpy(&h, w->d_res, sizeof h, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemset(w->d_res, 0, sizeof(Result)));
  *err = h.err;
  *where = h.where;
  return L3G_OK;
}

// ---------------------------------------------------------------------------
// batched prefill
// ---------------------------------------------------------------------------
// Tokens per pass over the weights (a pass streams every layer's matrices
// once); the last pass takes the remainder.
constexpr int PF_CHUNK = 512;

static int gemm_from_tiles(const DevMat& src, GemmMat& dst, size_t* dev_bytes) {
  dst.rows = src.t.rows;
  dst.cols = src.t.cols;
  dst.nk = gemm::chunks(dst.cols);
  dst.n_rt = gemm::row_tiles(dst.rows);
  dst.bytes = (size_t)dst.n_rt * dst.nk * gemm::A_CHUNK;
  CUDA_TRY(cudaMalloc(&dst.data, dst.bytes));
  CUDA_TRY(cudaMemset(dst.data, 0, dst.bytes));
  k_gemm_from_tiles<<<2048, 256>>>(src.t, dst.data);
  CUDA_TRY(cudaGetLastError());
  *dev_bytes += dst.bytes;
  return L3G_OK;
}

// The layers' matrices as weight chunks of the batched product, built once
// per model from the resident tiles (same shard, same fused row orders).
static int ensure_gemm_weights(l3g_model* m) {
  std::lock_guard<std::mutex> lk(m->gemm_mu);
  if (m->gemm_ready) return L3G_OK;
  for (auto& L : m->layers) {
    int rc = gemm_from_tiles(L.qkv, L.gqkv, &m->dev_bytes);
    if (!rc) rc = gemm_from_tiles(L.wo, L.gwo, &m->dev_bytes);
    if (!rc) rc = gemm_from_tiles(L.upgate, L.gupgate, &m->dev_bytes);
    if (!rc) rc = gemm_from_tiles(L.down, L.gdown, &m->dev_bytes);
    if (rc) return rc;
  }
  CUDA_TRY(cudaDeviceSynchronize());
  m->gemm_ready = true;
  return L3G_OK;
}

static int ensure_prefill_buffers(l3g_workspace* ws) {
  if (ws->pf_cap) return L3G_OK;
  const l3g_model* m = ws->m;
  const int cap = PF_CHUNK;
  const int ne = m->hp.n_emb, nq = m->hq_l * m->hd, nkv = m->hkv_l * m->hd;
  const int max_cols = std::max(std::max(ne, nq), m->ff_l);
  uint64_t act_bytes = 0;
  if (int rc = l3g_gemm_act_bytes(cap, max_cols, &act_bytes)) return rc;
  cudaError_t e = cudaMalloc(&ws->pf_ids, (size_t)cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_x, (size_t)cap * ne * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_y, (size_t)cap * ne * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_qkv, (size_t)cap * (nq + 2 * nkv) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_q, (size_t)cap * nq * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_att, (size_t)cap * nq * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_ug, (size_t)cap * 2 * m->ff_l * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ws->pf_act, act_bytes);
  // padding tokens and columns of the activation chunks are never written
  if (e == cudaSuccess) e = cudaMemset(ws->pf_act, 0, act_bytes);
  size_t part = 0;
  for (const auto& L : m->layers)
    for (const GemmMat* g : {&L.gqkv, &L.gwo, &L.gupgate, &L.gdown})
      part = std::max(part, gemm_part_bound(*g, cap, m->nsm));
  if (e == cudaSuccess && part) e = cudaMalloc(&ws->pf_part, part * 4);
  ws->pf_part_floats = e == cudaSuccess ? part : 0;
  if (e != cudaSuccess)
    return l3g_fail(L3G_E_CUDA, "prefill buffers: %s", cudaGetErrorString(e));
  ws->pf_cap = cap;
  return L3G_OK;
}

template <int HD>
static cudaError_t launch_pf_attention(const l3g_model* m, const l3g_workspace* ws,
                                       const KvMap& kv, int layer, int P, int pos0,
                                       cudaStream_t st) {
  const int bq = std::max(1, 64 / m->group);
  const dim3 grid((P + bq - 1) / bq, m->hkv_l);
  const float scale = (float)(1.0 / sqrt((double)m->hd));
  if (m->kv_f16)
    k_pf_attention<HD, __half><<<grid, 256, pf_attention_smem(HD), st>>>(
        ws->pf_q, kv, layer, ws->pf_att, P, pos0, m->group, bq, m->hq_l, scale);
  else
    k_pf_attention<HD, float><<<grid, 256, pf_attention_smem(HD), st>>>(
        ws->pf_q, kv, layer, ws->pf_att, P, pos0, m->group, bq, m->hq_l, scale);
  return cudaGetLastError();
}

// One pass of P <= pf_cap tokens at positions pos0..pos0+P-1 over every
// layer.  The last layer stops after its K/V append: its attention and FFN
// outputs only feed the logits, which prefill does not compute (infer.go:250).
static int enqueue_prefill_pass(l3g_model* m, l3g_state* s, l3g_workspace* ws, int P,
                                int pos0) {
  const l3g_hparams& hp = m->hp;
  const cudaStream_t st = ws->stream;
  const int ne = hp.n_emb, hd = m->hd;
  const int nq = m->hq_l * hd, nkv = m->hkv_l * hd;
  const unsigned long long wait_ns = WAIT_TIMEOUT_NS;
  const int nt = gemm::token_tile(P);
  uint8_t* act = ws->pf_act;
  k_pf_embed<<<dim3((ne + 255) / 256, P), 256, 0, st>>>(m->emb, hp.vocab_size, ne, ws->pf_ids,
                                                        ws->pf_x, ws->d_res);
  CUDA_TRY(cudaGetLastError());
  for (int l = 0; l < hp.n_layers; ++l) {
    const LayerW& L = m->layers[l];
    const KvMap kv = state_kv(s);
    // residual (from layer l-1's down) -> RMSNorm -> act-quant, infer.go:67-73
    k_pf_rms_quant<<<P, PF_THREADS, 0, st>>>(ws->pf_x, l ? ws->pf_y : nullptr, L.attn_norm,
                                            hp.rms_eps, ne, nt, gemm::chunks(ne), act);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(launch_gemm(L.gqkv, act, P, ws->pf_qkv, ws->d_res, wait_ns, m->nsm, st, 0,
                         ws->pf_part, ws->pf_part_floats));
    {  // RoPE + KV append, infer.go:76-127
      const long long pairs = (long long)P * ((nq + 2 * nkv) / 2);
      k_pf_qkv_rope<<<(unsigned)((pairs + 255) / 256), 256, 0, st>>>(
          ws->pf_qkv, P, pos0, nq, nkv, hd, m->rope_half, s->rope_cos, s->rope_sin, ws->pf_q, kv,
          l, m->kv_f16);
      CUDA_TRY(cudaGetLastError());
    }
    if (l == hp.n_layers - 1) break;
    // attention, infer.go:130-175
    switch (hd) {
      case 32: CUDA_TRY(launch_pf_attention<32>(m, ws, kv, l, P, pos0, st)); break;
      case 64: CUDA_TRY(launch_pf_attention<64>(m, ws, kv, l, P, pos0, st)); break;
      case 128: CUDA_TRY(launch_pf_attention<128>(m, ws, kv, l, P, pos0, st)); break;
      default: return l3g_fail(L3G_E_INVALID, "batched prefill: head_dim %d", hd);
    }
    // act-quant of the attention output -> Wo, infer.go:178-187
    {
      const long long warps = (long long)((P + nt - 1) / nt * nt) * gemm::chunks(nq) * gemm::BPC;
      k_gemm_quantize<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
          ws->pf_att, P, nq, nt, gemm::chunks(nq), (P + nt - 1) / nt * nt, act);
      CUDA_TRY(cudaGetLastError());
    }
    CUDA_TRY(launch_gemm(L.gwo, act, P, ws->pf_y, ws->d_res, wait_ns, m->nsm, st, 0, ws->pf_part,
                         ws->pf_part_floats));
    if (m->world > 1)
      NCCL_TRY(nccl()->AllReduce(ws->pf_y, ws->pf_y, (size_t)P * ne, ncclFloat, ncclSum, m->comm,
                                 st));
    // residual -> RMSNorm -> act-quant -> up/gate -> SwiGLU -> act-quant,
    // infer.go:189-234
    k_pf_rms_quant<<<P, PF_THREADS, 0, st>>>(ws->pf_x, ws->pf_y, L.ffn_norm, hp.rms_eps, ne, nt,
                                            gemm::chunks(ne), act);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(launch_gemm(L.gupgate, act, P, ws->pf_ug, ws->d_res, wait_ns, m->nsm, st, 0,
                         ws->pf_part, ws->pf_part_floats));
    {
      const long long warps = (long long)P * (m->ff_l / 32);
      k_pf_swiglu_quant<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
          ws->pf_ug, P, m->ff_l, nt, gemm::chunks(m->ff_l), act);
      CUDA_TRY(cudaGetLastError());
    }
    // down, infer.go:235-246 (its residual add opens the next layer)
    CUDA_TRY(launch_gemm(L.gdown, act, P, ws->pf_y, ws->d_res, wait_ns, m->nsm, st, 0, ws->pf_part,
                         ws->pf_part_floats));
    if (m->world > 1)
      NCCL_TRY(nccl()->AllReduce(ws->pf_y, ws->pf_y, (size_t)P * ne, ncclFloat, ncclSum, m->comm,
                                 st));
  }
  return L3G_OK;
}

extern "C" int l3g_prefill_batched(l3g_model* m, l3g_state* s, l3g_workspace* ws,
                                   const int32_t* tokens, int32_t n) {
  if (!m || !s) return l3g_fail(L3G_E_INVALID, "null argument");
  if (!ws) return l3g_fail(L3G_E_INVALID, "workspace is nil");
  if (n > 0 && !tokens) return l3g_fail(L3G_E_INVALID, "null argument");
  if (s->m != m || ws->m != m)
    return l3g_fail(L3G_E_INVALID, "state or workspace belongs to another model");
  if (n <= 0) return L3G_OK;
  if (ws->ctx < s->ctx)
    return l3g_fail(L3G_E_INVALID, "workspace ctxLen=%d < state ctxLen=%d", ws->ctx, s->ctx);
  if ((long long)s->pos + n > s->ctx)
    return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->hp.vocab_size)
      return l3g_fail(L3G_E_TOKEN, "token out of range: %d", tokens[i]);
  if (m->hp.n_emb > PF_THREADS * 4 * PF_VK || m->hp.n_emb % 32)
    return l3g_fail(L3G_E_INVALID, "batched prefill: n_emb %d", m->hp.n_emb);
  CUDA_TRY(cudaSetDevice(m->device));
  if (int rc = gemm_setup()) return rc;
  if (int rc = ensure_gemm_weights(m)) return rc;
  if (int rc = ensure_prefill_buffers(ws)) return rc;
  if (int rc = state_map(s, s->pos + n, ws->stream)) return rc;
  ws->logits_valid = false;
  for (int c0 = 0; c0 < n; c0 += ws->pf_cap) {
    const int P = std::min(ws->pf_cap, n - c0);
    CUDA_TRY(cudaMemcpyAsync(ws->pf_ids, tokens + c0, (size_t)P * 4, cudaMemcpyHostToDevice,
                             ws->stream));
    if (int rc = enqueue_prefill_pass(m, s, ws, P, s->pos)) return rc;
    CUDA_TRY(cudaMemcpyAsync(ws->h_res, ws->d_res, sizeof(Result), cudaMemcpyDeviceToHost,
                             ws->stream));
    CUDA_TRY(cudaStreamSynchronize(ws->stream));
    if (ws->h_res->err) {
      const int code = ws->h_res->err, where = ws->h_res->where;
      ws_clear_device_error(ws);
      return l3g_fail(L3G_E_DEVICE, "device check failed: code %d at site %d (%s)", code, where,
                      code == ERR_TIMEOUT ? "bounded wait ran out" : "bad input");
    }
    s->pos += P;
  }
  return L3G_OK;
}

// ---------------------------------------------------------------------------
// batched decode
// ---------------------------------------------------------------------------
struct l3g_batch {
  l3g_model* m = nullptr;
  int device = 0, cap = 0, max_splits = 0, tk_chunks = 0;
  cudaStream_t stream = nullptr;
  SeqInfo* h_seq = nullptr;  // pinned [cap]
  SeqInfo* d_seq = nullptr;
  Result* h_out = nullptr;   // pinned [cap]: sampled token and its logit
  Result* d_out = nullptr;
  Result* h_res = nullptr;   // pinned: error word
  Result* d_res = nullptr;
  float* x = nullptr;        // [cap][n_emb]
  float* y = nullptr;        // [cap][n_emb]
  float* qkv = nullptr;      // [cap][qkv rows]
  float* q = nullptr;        // [cap][local q heads * hd]
  float* att = nullptr;      // [cap][local q heads * hd]
  float* ug = nullptr;       // [cap][2 * local n_ff]
  float* logits = nullptr;   // [cap][v_l], columns past the shard's rows -inf
  float* logits_full = nullptr;  // [world][cap][v_l] (world > 1)
  float* part_o = nullptr;   // [cap][local q heads][max_splits][hd]
  float* part_ml = nullptr;  // [cap][local q heads][max_splits][2]
  uint8_t* act = nullptr;
  float* part = nullptr;         // split-K partial sums of the product
  size_t part_floats = 0;
  uint64_t* tk_part = nullptr;  // [cap][tk_chunks][MAX_TOPK]
  int* tk_ids = nullptr;        // [cap][MAX_TOPK]
  float* tk_logits = nullptr;
};

extern "C" void l3g_batch_free(l3g_batch* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  void* d[] = {b->d_seq, b->d_out, b->d_res, b->x, b->y, b->qkv, b->q, b->att, b->ug,
               b->logits, b->logits_full, b->part_o, b->part_ml, b->act, b->tk_part,
               b->tk_ids, b->tk_logits, b->part};
  for (void* p : d)
    if (p) cudaFree(p);
  void* h[] = {b->h_seq, b->h_out, b->h_res};
  for (void* p : h)
    if (p) cudaFreeHost(p);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

extern "C" int l3g_batch_new(l3g_model* m, int32_t max_seqs, l3g_batch** out) {
  if (!m || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  if (max_seqs <= 0 || max_seqs > L3G_BATCH_MAX)
    return l3g_fail(L3G_E_INVALID, "max_seqs=%d outside [1, %d]", max_seqs, L3G_BATCH_MAX);
  if (m->hp.n_emb > PF_THREADS * 4 * PF_VK || m->hd > 128 || (m->hd != 32 && m->hd != 64 &&
                                                              m->hd != 128))
    return l3g_fail(L3G_E_INVALID, "batched decode: n_emb %d, head_dim %d", m->hp.n_emb, m->hd);
  CUDA_TRY(cudaSetDevice(m->device));
  if (int rc = gemm_setup()) return rc;
  if (int rc = ensure_gemm_weights(m)) return rc;
  {
    std::lock_guard<std::mutex> lk(m->gemm_mu);
    if (!m->glogits.data) {
      size_t bytes = 0;
      if (int rc = gemm_from_tiles(m->logits, m->glogits, &bytes)) return rc;
      CUDA_TRY(cudaDeviceSynchronize());
      m->dev_bytes += bytes;
    }
  }
  auto* b = new l3g_batch();
  b->m = m;
  b->device = m->device;
  b->cap = max_seqs;
  b->max_splits = (m->hp.ctx_len + BD_SPLIT - 1) / BD_SPLIT;
  b->tk_chunks = (m->hp.vocab_size + TOPK_CHUNK - 1) / TOPK_CHUNK;
  const size_t cap = (size_t)max_seqs;
  const int ne = m->hp.n_emb, nq = m->hq_l * m->hd, nkv = m->hkv_l * m->hd;
  const int max_cols = std::max(std::max(ne, nq), m->ff_l);
  uint64_t act_bytes = 0;
  if (int rc = l3g_gemm_act_bytes(max_seqs, max_cols, &act_bytes)) {
    l3g_batch_free(b);
    return rc;
  }
  cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMallocHost(&b->h_seq, cap * sizeof(SeqInfo));
  if (e == cudaSuccess) e = cudaMallocHost(&b->h_out, cap * sizeof(Result));
  if (e == cudaSuccess) e = cudaMallocHost(&b->h_res, sizeof(Result));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_seq, cap * sizeof(SeqInfo));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_out, cap * sizeof(Result));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_res, sizeof(Result));
  if (e == cudaSuccess) e = cudaMemset(b->d_res, 0, sizeof(Result));
  if (e == cudaSuccess) e = cudaMalloc(&b->x, cap * ne * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->y, cap * ne * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->qkv, cap * (nq + 2 * nkv) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->q, cap * nq * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->att, cap * nq * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->ug, cap * 2 * m->ff_l * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->logits, cap * m->v_l * 4);
  if (e == cudaSuccess && m->world > 1)
    e = cudaMalloc(&b->logits_full, cap * m->v_l * m->world * 4);
  if (e == cudaSuccess)
    e = cudaMalloc(&b->part_o, cap * m->hq_l * b->max_splits * m->hd * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->part_ml, cap * m->hq_l * b->max_splits * 2 * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->act, act_bytes);
  if (e == cudaSuccess) e = cudaMemset(b->act, 0, act_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&b->tk_part, cap * b->tk_chunks * MAX_TOPK * 8);
  if (e == cudaSuccess) e = cudaMalloc(&b->tk_ids, cap * MAX_TOPK * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->tk_logits, cap * MAX_TOPK * 4);
  if (e == cudaSuccess) {
    size_t part = gemm_part_bound(m->glogits, max_seqs, m->nsm);
    for (const auto& L : m->layers)
      for (const GemmMat* g : {&L.gqkv, &L.gwo, &L.gupgate, &L.gdown})
        part = std::max(part, gemm_part_bound(*g, max_seqs, m->nsm));
    if (part) e = cudaMalloc(&b->part, part * 4);
    b->part_floats = e == cudaSuccess ? part : 0;
  }
  if (e == cudaSuccess) {  // the shard's padding columns (past its vocabulary rows) stay -inf
    std::vector<float> ninf(cap * m->v_l, -INFINITY);
    e = cudaMemcpy(b->logits, ninf.data(), ninf.size() * 4, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    l3g_batch_free(b);
    return l3g_fail(L3G_E_CUDA, "batch allocation: %s", cudaGetErrorString(e));
  }
  *out = b;
  return L3G_OK;
}

extern "C" int l3g_batch_step(l3g_batch* b, l3g_state* const* states, int32_t n,
                              const int32_t* tokens, int32_t top_k, float temperature,
                              const uint64_t* seeds, int32_t* next_tokens, float* logits_out) {
  if (!b || !states || !tokens || !seeds || !next_tokens)
    return l3g_fail(L3G_E_INVALID, "null argument");
  l3g_model* m = b->m;
  if (n <= 0 || n > b->cap) return l3g_fail(L3G_E_INVALID, "n=%d outside [1, %d]", n, b->cap);
  if (top_k <= 0) top_k = 40;  // infer.go:279-281
  if (top_k > MAX_TOPK) return l3g_fail(L3G_E_INVALID, "top_k %d above %d", top_k, MAX_TOPK);
  if (top_k > m->hp.vocab_size) top_k = m->hp.vocab_size;
  if (temperature <= 0.0f) temperature = 0.8f;  // sampling.go:20-22
  int max_pos = 0;
  for (int i = 0; i < n; ++i) {
    l3g_state* s = states[i];
    if (!s) return l3g_fail(L3G_E_INVALID, "null state %d", i);
    if (s->m != m) return l3g_fail(L3G_E_INVALID, "state %d belongs to another model", i);
    for (int j = 0; j < i; ++j)
      if (states[j] == s) return l3g_fail(L3G_E_INVALID, "state %d appears twice", i);
    if (s->pos >= s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
    if (tokens[i] < 0 || tokens[i] >= m->hp.vocab_size)
      return l3g_fail(L3G_E_TOKEN, "token out of range: %d", tokens[i]);
    SeqInfo& q = b->h_seq[i];
    q = SeqInfo{};
    q.kv_pool = s->pool->base;
    q.kv_pages = s->d_pages;
    q.kv_pps = s->pps;
    q.rope_cos = s->rope_cos;
    q.rope_sin = s->rope_sin;
    q.ctx = s->ctx;
    q.pos = s->pos;
    q.token = tokens[i];
    q.seed = seeds[i];
    q.temperature = temperature;
    max_pos = std::max(max_pos, s->pos);
  }
  CUDA_TRY(cudaSetDevice(m->device));
  const l3g_hparams& hp = m->hp;
  const cudaStream_t st = b->stream;
  const int ne = hp.n_emb, hd = m->hd;
  const int nq = m->hq_l * hd, nkv = m->hkv_l * hd;
  const unsigned long long wait_ns = m->world > 1 ? WAIT_TIMEOUT_PEER_NS : WAIT_TIMEOUT_NS;
  const int nt = gemm::token_tile(n);
  const int n_pad = (n + nt - 1) / nt * nt;
  // split length: a few waves of CTAs over every session's positions (two
  // CTAs per SM), long splits for long sessions, at least BD_SPLIT
  long long total = 0;
  for (int i = 0; i < n; ++i) total += states[i]->pos + 1;
  const long long target = 8LL * m->nsm;
  int split_len = (int)((total * m->hkv_l + target - 1) / target);
  // L3G_BD_SPLIT=n fixes it (a multiple of BD_SPLIT; for tests and sweeps)
  if (const char* env = getenv("L3G_BD_SPLIT")) split_len = atoi(env);
  split_len = std::min(16 * BD_SPLIT, std::max(BD_SPLIT, (split_len + BD_SPLIT - 1) / BD_SPLIT * BD_SPLIT));
  const int splits = (max_pos + 1 + split_len - 1) / split_len;
  const float scale = (float)(1.0 / sqrt((double)hd));
  for (int i = 0; i < n; ++i)  // each session's page for this step's position
    if (int rc = state_map(states[i], states[i]->pos + 1, st)) return rc;
  CUDA_TRY(cudaMemcpyAsync(b->d_seq, b->h_seq, (size_t)n * sizeof(SeqInfo),
                           cudaMemcpyHostToDevice, st));
  k_bd_embed<<<dim3((ne + 255) / 256, n), 256, 0, st>>>(m->emb, hp.vocab_size, ne, b->d_seq, b->x,
                                                        b->d_res);
  CUDA_TRY(cudaGetLastError());
  for (int l = 0; l < hp.n_layers; ++l) {
    const LayerW& L = m->layers[l];
    k_pf_rms_quant<<<n, PF_THREADS, 0, st>>>(b->x, l ? b->y : nullptr, L.attn_norm, hp.rms_eps,
                                            ne, nt, gemm::chunks(ne), b->act);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(launch_gemm(L.gqkv, b->act, n, b->qkv, b->d_res, wait_ns, m->nsm, st, 0, b->part,
                         b->part_floats));
    {
      const long long pairs = (long long)n * ((nq + 2 * nkv) / 2);
      k_bd_qkv_rope<<<(unsigned)((pairs + 255) / 256), 256, 0, st>>>(
          b->qkv, n, b->d_seq, l, nq, nkv, hd, m->rope_half, b->q, m->kv_f16);
      CUDA_TRY(cudaGetLastError());
    }
    {
      const dim3 grid(splits, m->hkv_l, n);
      const int gp = m->group <= 1 ? 1 : m->group <= 2 ? 2 : m->group <= 4 ? 4 : 8;
#define BDATT(HD, GP)                                                                         \
  if (m->kv_f16)                                                                             \
    k_bd_attention<HD, GP, __half><<<grid, BD_THREADS, bd_smem_bytes(HD, 2, GP), st>>>(      \
        b->q, b->d_seq, l, m->group, m->hq_l, scale, b->part_o, b->part_ml, b->max_splits,     \
        split_len, b->d_res, wait_ns);                                                        \
  else                                                                                       \
    k_bd_attention<HD, GP, float><<<grid, BD_THREADS, bd_smem_bytes(HD, 4, GP), st>>>(       \
        b->q, b->d_seq, l, m->group, m->hq_l, scale, b->part_o, b->part_ml, b->max_splits,     \
        split_len, b->d_res, wait_ns)
#define BDATT_G(HD)          \
  if (gp == 1) {             \
    BDATT(HD, 1);            \
  } else if (gp == 2) {      \
    BDATT(HD, 2);            \
  } else if (gp == 4) {      \
    BDATT(HD, 4);            \
  } else {                   \
    BDATT(HD, 8);            \
  }
      if (hd == 32) {
        BDATT_G(32)
      } else if (hd == 64) {
        BDATT_G(64)
      } else {
        BDATT_G(128)
      }
#undef BDATT_G
#undef BDATT
      CUDA_TRY(cudaGetLastError());
      k_bd_merge<<<dim3(m->hq_l, n), 128, 0, st>>>(b->part_o, b->part_ml, b->d_seq, m->hq_l, hd,
                                                   b->max_splits, split_len, b->att);
      CUDA_TRY(cudaGetLastError());
    }
    {
      const long long warps = (long long)n_pad * gemm::chunks(nq) * gemm::BPC;
      k_gemm_quantize<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
          b->att, n, nq, nt, gemm::chunks(nq), n_pad, b->act);
      CUDA_TRY(cudaGetLastError());
    }
    CUDA_TRY(launch_gemm(L.gwo, b->act, n, b->y, b->d_res, wait_ns, m->nsm, st, 0, b->part,
                         b->part_floats));
    if (m->world > 1)
      NCCL_TRY(nccl()->AllReduce(b->y, b->y, (size_t)n * ne, ncclFloat, ncclSum, m->comm, st));
    k_pf_rms_quant<<<n, PF_THREADS, 0, st>>>(b->x, b->y, L.ffn_norm, hp.rms_eps, ne, nt,
                                            gemm::chunks(ne), b->act);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(launch_gemm(L.gupgate, b->act, n, b->ug, b->d_res, wait_ns, m->nsm, st, 0, b->part,
                         b->part_floats));
    {
      const long long warps = (long long)n * (m->ff_l / 32);
      k_pf_swiglu_quant<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
          b->ug, n, m->ff_l, nt, gemm::chunks(m->ff_l), b->act);
      CUDA_TRY(cudaGetLastError());
    }
    CUDA_TRY(launch_gemm(L.gdown, b->act, n, b->y, b->d_res, wait_ns, m->nsm, st, 0, b->part,
                         b->part_floats));
    if (m->world > 1)
      NCCL_TRY(nccl()->AllReduce(b->y, b->y, (size_t)n * ne, ncclFloat, ncclSum, m->comm, st));
  }
  // residual -> final RMSNorm -> act-quant -> logits shard, infer.go:250-260
  k_pf_rms_quant<<<n, PF_THREADS, 0, st>>>(b->x, b->y, m->out_norm, hp.rms_eps, ne, nt,
                                          gemm::chunks(ne), b->act);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(launch_gemm(m->glogits, b->act, n, b->logits, b->d_res, wait_ns, m->nsm, st, m->v_l,
                         b->part, b->part_floats));
  const float* lg = b->logits;
  if (m->world > 1) {
    NCCL_TRY(nccl()->AllGather(b->logits, b->logits_full, (size_t)n * m->v_l, ncclFloat, m->comm,
                               st));
    lg = b->logits_full;
  }
  // top-K and SampleTopK per sequence
  k_bd_topk_partial<<<dim3(b->tk_chunks, n), 256, 0, st>>>(lg, n, m->v_l, hp.vocab_size, top_k,
                                                          b->tk_part);
  CUDA_TRY(cudaGetLastError());
  {
    const int count = b->tk_chunks * top_k;
    int cap2 = 1;
    while (cap2 < count) cap2 <<= 1;
    k_bd_topk_final<<<n, 256, (size_t)cap2 * 8, st>>>(b->tk_part, count, cap2, top_k, b->tk_ids,
                                                     b->tk_logits);
    CUDA_TRY(cudaGetLastError());
  }
  k_bd_sample<<<n, 32, 0, st>>>(b->tk_ids, b->tk_logits, top_k, b->d_seq, b->d_out);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaMemcpyAsync(b->h_out, b->d_out, (size_t)n * sizeof(Result), cudaMemcpyDeviceToHost,
                           st));
  CUDA_TRY(cudaMemcpyAsync(b->h_res, b->d_res, sizeof(Result), cudaMemcpyDeviceToHost, st));
  if (logits_out) {  // [n][vocab]: the shards side by side
    for (int r = 0; r < m->world; ++r) {
      const int rows = std::min(m->v_l, hp.vocab_size - r * m->v_l);
      if (rows <= 0) break;
      CUDA_TRY(cudaMemcpy2DAsync(logits_out + (size_t)r * m->v_l, (size_t)hp.vocab_size * 4,
                                 lg + (size_t)r * n * m->v_l, (size_t)m->v_l * 4,
                                 (size_t)rows * 4, n, cudaMemcpyDeviceToHost, st));
    }
  }
  CUDA_TRY(cudaStreamSynchronize(st));
  if (b->h_res->err) {
    const int code = b->h_res->err, where = b->h_res->where;
    cudaMemset(b->d_res, 0, sizeof(Result));
    return l3g_fail(L3G_E_DEVICE, "device check failed: code %d at site %d (%s)", code, where,
                    code == ERR_TIMEOUT ? "bounded wait ran out" : "bad input");
  }
  for (int i = 0; i < n; ++i) {
    next_tokens[i] = b->h_out[i].token;
    states[i]->pos++;
  }
  return L3G_OK;
}
