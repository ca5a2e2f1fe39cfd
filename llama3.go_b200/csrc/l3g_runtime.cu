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
#include <dlfcn.h>
#include <unistd.h>
#include <nccl.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "l3g.h"
#include "l3g_internal.h"
#include "l3g_kernels.cuh"

using namespace l3g;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local std::string g_err;

int l3g_fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CUDA_TRY(expr)                                                     \
  do {                                                                     \
    cudaError_t e_ = (expr);                                               \
    if (e_ != cudaSuccess)                                                 \
      return l3g_fail(L3G_E_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

extern "C" const char* l3g_last_error(void) { return g_err.c_str(); }
extern "C" int l3g_version(void) { return L3G_VERSION; }

extern "C" int l3g_device_count(int32_t* n) {
  int c = 0;
  CUDA_TRY(cudaGetDeviceCount(&c));
  if (n) *n = c;
  return L3G_OK;
}

extern "C" void l3g_options_default(l3g_options* opt) {
  if (!opt) return;
  memset(opt, 0, sizeof *opt);
  opt->world_size = 1;
  opt->rank = 0;
  opt->device = -1;
  opt->kv_dtype = L3G_KV_F32;
}

// ---------------------------------------------------------------------------
// NCCL, bound at run time (the process may already hold torch's copy)
// ---------------------------------------------------------------------------
struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t,
                            ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t,
                            ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
    api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
    api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
    api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
    api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce &&
             api.AllGather && api.CommDestroy && api.GetErrorString;
  });
  return &api;
}

#define NCCL_TRY(expr)                                                      \
  do {                                                                      \
    ncclResult_t r_ = (expr);                                               \
    if (r_ != ncclSuccess)                                                  \
      return l3g_fail(L3G_E_NCCL, "%s: %s", #expr, nccl()->GetErrorString(r_)); \
  } while (0)

extern "C" int l3g_nccl_unique_id(uint8_t out[128]) {
  NcclApi* api = nccl();
  if (!api->ok) return l3g_fail(L3G_E_NCCL, "libnccl.so.2 not found");
  ncclUniqueId id;
  NCCL_TRY(api->GetUniqueId(&id));
  static_assert(sizeof(id) == 128, "ncclUniqueId size");
  memcpy(out, &id, 128);
  return L3G_OK;
}

// ---------------------------------------------------------------------------
// kernel set-up
// ---------------------------------------------------------------------------
static int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

// Dynamic shared memory may take what static shared memory leaves of the
// per-block opt-in limit.
template <typename K>
static cudaError_t set_max_shared(K k, int limit) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, k);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             limit - (int)fa.sharedSizeBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  return e;
}

// Kernel attributes belong to the device (context) they were set on: once
// per device, with that device current.
static int setup_kernels() {
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

// ---------------------------------------------------------------------------
// tiled Q8_0 matrices
// ---------------------------------------------------------------------------
struct DevMat {
  Q8Tiles t{};
  uint8_t* buf = nullptr;
  size_t bytes = 0;
  int nstages = 2;
  int smem = 0;
};

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

struct RowSrc {         // rows [row0, row0+n) of a host GGUF Q8_0 tensor
  const uint8_t* host;
  int row0, n;
};

// Uploads the needed source rows, repacks them into tiles on the device.
// rpw > 0 fixes the rows per warp (the persistent kernel's layout); 0 plans.
static int upload_tiled(DevMat& out, const RowSrc* segs, int nseg,
                        bool interleave2, int src_cols, int blk0, int cols,
                        int nsm, size_t* dev_bytes, int rpw = 0) {
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

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
// A matrix in the batched product's weight chunks (l3g_gemm_layout.h).
struct GemmMat {
  uint8_t* data = nullptr;
  int rows = 0, cols = 0, nk = 0, n_rt = 0;
  size_t bytes = 0;
};

static void free_gemm(GemmMat& g) {
  if (g.data) cudaFree(g.data);
  g = GemmMat{};
}

struct LayerW {
  DevMat qkv, wo, upgate, down;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  // the same matrices as weight chunks of the batched product (built on
  // the first batched prefill)
  GemmMat gqkv, gwo, gupgate, gdown;
};

struct l3g_model {
  l3g_hparams hp{};
  int world = 1, rank = 0, device = 0, kv_f16 = 0, nsm = 1;
  // live workspaces: their captured step graphs hold NCCL calls on `comm`,
  // so they are released before the communicator is destroyed
  std::mutex ws_mu;
  std::vector<l3g_workspace*> workspaces;
  int hd = 0, hq_l = 0, hkv_l = 0, group = 1, ff_l = 0, v_l = 0, v_off = 0;
  int rope_half = 0;
  std::vector<double> inv_freq;
  std::vector<LayerW> layers;
  DevMat logits;
  float* out_norm = nullptr;
  uint8_t* emb = nullptr;  // raw GGUF Q8_0 token_embd (all rows)
  ncclComm_t comm = nullptr;
  size_t dev_bytes = 0;
  std::mutex gemm_mu;       // guards the lazy build of the layers' GemmMat
  bool gemm_ready = false;
  GemmMat glogits;          // logits shard as weight chunks (batched decode)
  // persistent layer kernel (L3G_PERSIST=1 at load): layer matrices tiled
  // with four rows per warp, and their pointers in a device table
  bool persist = false;
  PersistLayer* d_layers = nullptr;
};

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

static void free_mat(DevMat& m) {
  if (m.buf) cudaFree(m.buf);
  m.buf = nullptr;
}

static void ws_detach(l3g_workspace* ws);  // releases its graphs, forgets the model

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

// ---------------------------------------------------------------------------
// state
// ---------------------------------------------------------------------------
struct l3g_state {
  l3g_model* m = nullptr;
  int device = 0;
  int ctx = 0, pos = 0;
  void* kv = nullptr;      // [layer][local kv head][ctx][K hd | V hd]
  size_t layer_elems = 0;  // per layer: local kv heads * ctx * 2 * hd
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  uint64_t serial = 0;
};

static uint64_t next_serial() {
  static std::mutex mu;
  static uint64_t s = 0;
  std::lock_guard<std::mutex> g(mu);
  return ++s;
}

extern "C" void l3g_state_free(l3g_state* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  if (s->kv) cudaFree(s->kv);
  if (s->rope_cos) cudaFree(s->rope_cos);
  if (s->rope_sin) cudaFree(s->rope_sin);
  delete s;
}

extern "C" int l3g_state_new(l3g_model* m, int32_t ctx, l3g_state** out) {
  if (!m || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  if (ctx <= 0) ctx = m->hp.ctx_len;  // state.go:52-57
  if (ctx > m->hp.ctx_len) ctx = m->hp.ctx_len;
  CUDA_TRY(cudaSetDevice(m->device));
  auto* s = new l3g_state();
  s->m = m;
  s->device = m->device;
  s->ctx = ctx;
  s->serial = next_serial();
  s->layer_elems = (size_t)m->hkv_l * ctx * 2 * m->hd;
  const size_t es = m->kv_f16 ? 2 : 4;
  const size_t kvb = s->layer_elems * m->hp.n_layers * es;
  cudaError_t e = cudaMalloc(&s->kv, kvb);
  if (e == cudaSuccess) e = cudaMemset(s->kv, 0, kvb);
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
  const size_t row = (size_t)h.pos * 2 * h.hd * h.elem_bytes;     // one (layer, kv head)
  const size_t pitch = (size_t)s->ctx * 2 * h.hd * h.elem_bytes;  // its slot in the cache
  CUDA_TRY(cudaMemcpy2D(static_cast<uint8_t*>(dst) + sizeof h, row, s->kv, pitch, row,
                        (size_t)h.n_layers * h.hkv_l, cudaMemcpyDeviceToHost));
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
    const size_t row = (size_t)h.pos * 2 * h.hd * h.elem_bytes;
    const size_t pitch = (size_t)s->ctx * 2 * h.hd * h.elem_bytes;
    CUDA_TRY(cudaMemcpy2D(s->kv, pitch, static_cast<const uint8_t*>(src) + sizeof h, row, row,
                          (size_t)h.n_layers * h.hkv_l, cudaMemcpyHostToDevice));
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
  CUDA_TRY(cudaSetDevice(m->device));
  const int hd = m->hd, nh = m->hkv_l;
  const size_t es = m->kv_f16 ? 2 : 4;
  std::vector<uint8_t> buf((size_t)npos * 2 * hd * es);
  for (int h = 0; h < nh; ++h) {
    const size_t off =
        ((size_t)layer * s->layer_elems + ((size_t)h * s->ctx + pos0) * 2 * hd) * es;
    CUDA_TRY(cudaMemcpy(buf.data(), static_cast<uint8_t*>(s->kv) + off, buf.size(),
                        cudaMemcpyDeviceToHost));
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

// ---------------------------------------------------------------------------
// workspace and the step graphs
// ---------------------------------------------------------------------------
// V_GREEDY_DEV: the token and position come from the previous replay's
// argmax on the device (k_advance), no host copies inside the graph.
// V_TRACE: V_GREEDY_DEV with the device timeline recorded.
enum Variant {
  V_PREFILL = 0, V_ARGMAX = 1, V_LOGITS = 2, V_TOPK = 3, V_GREEDY_DEV = 4, V_TRACE = 5,
  V_SAMPLE = 6,      // top-K + device sampler, token to the host
  V_SAMPLE_DEV = 7   // top-K + device sampler, token fed to the next step
};
constexpr int kTraceCap = 256;  // traced launches per step
constexpr size_t kTraceBytes = (size_t)kTraceCap * TRACE_CTAS * 8 * 8;

struct StepGraph {
  int variant, k;
  uint64_t state_serial;
  cudaGraphExec_t exec;
};

struct l3g_workspace {
  l3g_model* m = nullptr;
  int device = 0;
  int ctx = 0, topk = 40;
  cudaStream_t stream = nullptr;
  int* d_io = nullptr;
  int* h_io = nullptr;       // pinned {token, pos, 0, 0}
  Result* d_res = nullptr;
  Result* h_res = nullptr;   // pinned
  Result* d_gather = nullptr;  // [world] per-rank argmax results
  float* x[2] = {nullptr, nullptr};
  float* y = nullptr;
  float* q = nullptr;
  float* attn = nullptr;
  float* act = nullptr;
  float* attn_d = nullptr;     // attention output, Q8_0-quantized by the merge
  int8_t* attn_q = nullptr;
  float* act_d = nullptr;      // SwiGLU output, Q8_0-quantized once per step
  int8_t* act_q = nullptr;
  float* logits = nullptr;     // [world * v_l]: local shard first, gathered when TP
  float* logits_full = nullptr;
  float* h_logits = nullptr;   // pinned [vocab]
  float* part_o = nullptr;
  float* part_ml = nullptr;
  unsigned* att_cnt = nullptr;
  float* am_val = nullptr;
  int* am_idx = nullptr;
  unsigned* am_cnt = nullptr;
  uint64_t* tk_part = nullptr;
  int* d_tk_ids = nullptr;
  float* d_tk_logits = nullptr;
  int* h_tk_ids = nullptr;
  float* h_tk_logits = nullptr;
  int n_splits = 1, att_P = 16, att_ns = 3, att_stage = 0, att_smem = 0, att_gp = 1;
  int att_cluster = 0;         // > 0: the splits of a kv head form one cluster
  unsigned* d_step = nullptr;  // steps run (advanced by k_embed)
  SampleParams* h_samp = nullptr;  // pinned: the sampler's temperature, seed, draw index
  SampleParams* d_samp = nullptr;
  uint64_t draws = 0;              // sampler draws made with this workspace
  int* d_sync = nullptr;       // operand of the ranks' line-up after a capture
  // tensor parallel exchange over peer memory (world > 1 and IPC available)
  bool tp_p2p = false;
  unsigned long long* tp_recv = nullptr;               // [2][world][n_emb] {value, epoch}
  unsigned long long* tp_peer_recv[MAX_WORLD] = {};    // every rank's (self: own)
  bool tp_peer_same_process[MAX_WORLD] = {};            // mapped without IPC
  int tk_chunks = 0;
  int* d_tokens = nullptr;     // [ctx] tokens of a device-fed greedy run
  int kernels = 0;             // kernel launches counted during a capture
  int kernels_greedy = 0;      // ... of the greedy variant
  bool profiling = false;      // record an event after every kernel
  std::vector<int> prof_kind;
  std::vector<cudaEvent_t> prof_ev;
  unsigned long long* d_trace = nullptr;  // [kernels][2][8] timeline stamps
  std::vector<int> trace_kinds;            // kind of each traced launch
  std::vector<int> trace_kinds_graph;      // ... as captured in the V_TRACE graph
  std::vector<StepGraph> graphs;
  bool logits_valid = false;
  // batched prefill buffers for up to pf_cap tokens (allocated on first use)
  int pf_cap = 0;
  int* pf_ids = nullptr;
  float* pf_x = nullptr;    // [pf_cap][n_emb] residual stream
  float* pf_y = nullptr;    // [pf_cap][n_emb] Wo / down output
  float* pf_qkv = nullptr;  // [pf_cap][qkv rows]
  float* pf_q = nullptr;    // [pf_cap][local q heads * hd] roped queries
  float* pf_att = nullptr;  // [pf_cap][local q heads * hd] attention output
  float* pf_ug = nullptr;   // [pf_cap][2 * local n_ff] interleaved up/gate
  uint8_t* pf_act = nullptr;  // activation chunks of the batched product
  float* pf_part = nullptr;   // split-K partial sums of the product
  size_t pf_part_floats = 0;
  // persistent layer kernel (model->persist, see persist_setup)
  bool ps_on = false;
  persist::Plan ps_plan{};     // ctx is the state's, filled per capture
  int ps_ns = 0, ps_slot = 0, ps_union = 0, ps_xq_off = 0, ps_smem = 0, ps_nsub = 1;
  bool ps_fuse = false;        // SwiGLU act-quant fused into the up/gate phase
  bool ps_fuse_merge = false;  // split merge fused into the attention phase
  int ps_bar_words = 0;        // words of d_bar that k_embed zeroes
  unsigned* d_bar = nullptr;   // grid-barrier counters and abort word (persist::BAR_*)
  // the top-K path's fastExp attention (l3g_workspace_set_topk_fast_exp):
  // scores [local q heads][ctx], per-split max / sum [kv heads][splits][group],
  // per-split sum of e * V [kv heads][splits][group][hd]
  bool topk_fast = false;
  int attf_splits = 0;
  float* attf_scores = nullptr;
  float* attf_pmax = nullptr;
  float* attf_psum = nullptr;
  float* attf_po = nullptr;
};

static void ws_release(l3g_workspace* ws) {
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

static void ws_detach(l3g_workspace* ws) {
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

// Tensor-parallel exchange buffer: a receive buffer [2][world][n_emb] of
// {value, epoch} words per rank (zero: no epoch yet), mapped into every other
// rank's address space with CUDA IPC (ranks in other processes) or reached
// through unified addressing with peer access (ranks that are threads of the
// same process); the handles and pointers travel over the model's NCCL
// communicator.  All ranks agree (an NCCL min) on whether every mapping
// succeeded; otherwise the step uses NCCL allreduces instead.  L3G_TP_NCCL=1
// forces the NCCL path.  Collective: every rank creates its workspaces in
// the same order.
static int tp_setup(l3g_workspace* ws) {
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
static int persist_setup(l3g_workspace* ws) {
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
  // K|V rows of P positions, one ~32 KB bulk copy; three stages in flight
  ws->att_P = std::max(NW, (int)(32768 / (2 * hd * es)));
  ws->att_stage = 2 * ws->att_P * hd * (int)es;
  ws->att_ns = 3;
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
  DM(ws->att_cnt, (size_t)m->hkv_l * 2 * 4);  // arrivals, departures
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
  if (e == cudaSuccess) e = cudaMemset(ws->att_cnt, 0, (size_t)m->hkv_l * 2 * 4);
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

// Enqueues one decode step on ws->stream (captured into a graph).
// Exchange descriptor of reduction phase `phase` (2 * layer + 0 after Wo,
// + 1 after down) for this rank.
static TpExchange tp_exchange(const l3g_workspace* ws, int phase) {
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
  a.kv = static_cast<uint8_t*>(s->kv);
  a.kv_layer_bytes = s->layer_elems * (m->kv_f16 ? 2 : 4);
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

// The persistent kernel's barrier stamps of a traced step live in the trace
// buffer after the first kPersistStampSlot launches' per-CTA stamps (the
// step's other kernels stamp there), [barrier][cta]{arrival, release}.
constexpr size_t kPersistStampSlot = 16;
constexpr size_t kPersistStampOff = kPersistStampSlot * TRACE_CTAS * 8;  // in 64-bit words
static size_t persist_stamp_bytes(const l3g_workspace* ws) {
  return (size_t)persist::BARRIERS_PER_LAYER * ws->ps_plan.n_layers * ws->ps_plan.grid * 2 * 8;
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
    const PersistArgs a = persist_args(ws, s, stamps);
    int gp = 1;
    while (gp < m->group) gp <<= 1;
    void* kfn = layers_kernel(m, gp, ws->ps_fuse_merge);
    if (!kfn) return l3g_fail(L3G_E_INVALID, "no persistent layer kernel for this shape");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ws->ps_plan.grid);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = ws->ps_smem;
    cfg.stream = st;
    // A cooperative launch: the driver guarantees every CTA of the grid is
    // resident at once (the grid barriers between phases depend on it) or
    // refuses the launch with cudaErrorCooperativeLaunchTooLarge.  No
    // programmatic early launch for it: k_layers starts after k_embed ends.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* kargs[] = {(void*)&a};
    KL(L3G_K_LAYERS, cudaLaunchKernelExC(&cfg, kfn, kargs));
  }
  // the per-kernel step (skipped when the persistent kernel ran the layers)
  for (int l = 0; !persistent && l < hp.n_layers; ++l) {
    const LayerW& L = m->layers[l];
    uint8_t* kv = static_cast<uint8_t*>(s->kv) + (size_t)l * s->layer_elems * es;
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
      a.ctx = s->ctx;
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
      a.ctx = s->ctx;
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
  ws->h_io[0] = token;
  ws->h_io[1] = s->pos;
  ws->h_io[2] = 0;
  ws->h_io[3] = 0;
  CUDA_TRY(cudaGraphLaunch(exec, ws->stream));
  CUDA_TRY(cudaStreamSynchronize(ws->stream));
  if (ws->h_res->err) {
    const int code = ws->h_res->err, where = ws->h_res->where;
    cudaMemset(ws->d_res, 0, sizeof(Result));
    // an aborted kernel may have left its last-CTA counters mid-count
    cudaMemset(ws->att_cnt, 0, (size_t)m->hkv_l * 2 * 4);
    cudaMemset(ws->am_cnt, 0, 4);
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
    cudaMemset(ws->d_res, 0, sizeof(Result));
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
    cudaMemset(ws->d_res, 0, sizeof(Result));
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
    cudaMemset(ws->d_res, 0, sizeof(Result));
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
    cudaMemset(ws->d_res, 0, sizeof(Result));
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

// ---------------------------------------------------------------------------
// batched Q8_0 product on the tensor cores (tcgen05 kind::i8)
// ---------------------------------------------------------------------------
// One batched product out[n][r] (n < n_tok) on stream st: one CTA per SM at
// most, tiles dealt round-robin.
// K split of a product with few (row tile, token tile) tiles: the largest
// divisor of the chunk count that keeps the units within the SM count and
// the partial sums within part_floats (1: no split).
static int gemm_ksplit(const GemmMat& w, int n_tok, int nsm, size_t part_floats) {
  const int nt = gemm::token_tile(n_tok);
  const long long tiles = (long long)w.n_rt * ((n_tok + nt - 1) / nt);
  if (part_floats == 0 || tiles >= nsm) return 1;
  const long long want = nsm / tiles;
  int best = 1;
  for (int d = 2; d <= w.nk && d <= want; ++d)
    if (w.nk % d == 0 && (size_t)d * n_tok * w.rows <= part_floats) best = d;
  return best;
}
// Partial-sum floats that gemm_ksplit can ask of matrix w for up to cap tokens.
static size_t gemm_part_bound(const GemmMat& w, int cap, int nsm) {
  if (!w.data) return 0;
  const long long d = std::min<long long>(w.nk, std::max(1, nsm / std::max(1, w.n_rt)));
  return d > 1 ? (size_t)d * cap * w.rows : 0;
}

// One batched product out[n][r] (n < n_tok) on stream st: one CTA per SM at
// most, work units dealt round-robin; with few tiles the K range is split
// over more CTAs (partial sums in part, then k_gemm_reduce).
static cudaError_t launch_gemm(const GemmMat& w, const uint8_t* act, int n_tok, float* out,
                               Result* res, unsigned long long wait_ns, int nsm,
                               cudaStream_t st, int ldo = 0, float* part = nullptr,
                               size_t part_floats = 0) {
  const int nt = gemm::token_tile(n_tok);
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
  g.ksplit = part ? gemm_ksplit(w, n_tok, nsm, part_floats) : 1;
  g.part = part;
  g.nstages = gemm::stages(nt);
  g.res = res;
  g.wait_ns = wait_ns;
  const long long units = (long long)g.n_rt * g.n_tt * g.ksplit;
  const int grid = (int)std::max<long long>(1, std::min<long long>(nsm, units));
  switch (nt) {
    case 16: k_gemm_q8<16><<<grid, GEMM_THREADS, gemm::smem_bytes(16), st>>>(g); break;
    case 32: k_gemm_q8<32><<<grid, GEMM_THREADS, gemm::smem_bytes(32), st>>>(g); break;
    case 64: k_gemm_q8<64><<<grid, GEMM_THREADS, gemm::smem_bytes(64), st>>>(g); break;
    default: k_gemm_q8<128><<<grid, GEMM_THREADS, gemm::smem_bytes(128), st>>>(g); break;
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
                       WAIT_TIMEOUT_NS, w->nsm, (cudaStream_t)stream));
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
                                       const void* kv, int P, int pos0, int ctx,
                                       cudaStream_t st) {
  const int bq = std::max(1, 64 / m->group);
  const dim3 grid((P + bq - 1) / bq, m->hkv_l);
  const float scale = (float)(1.0 / sqrt((double)m->hd));
  if (m->kv_f16)
    k_pf_attention<HD, __half><<<grid, 256, pf_attention_smem(HD), st>>>(
        ws->pf_q, kv, ws->pf_att, P, pos0, ctx, m->group, bq, m->hq_l, scale);
  else
    k_pf_attention<HD, float><<<grid, 256, pf_attention_smem(HD), st>>>(
        ws->pf_q, kv, ws->pf_att, P, pos0, ctx, m->group, bq, m->hq_l, scale);
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
  const size_t es = m->kv_f16 ? 2 : 4;
  const unsigned long long wait_ns = WAIT_TIMEOUT_NS;
  const int nt = gemm::token_tile(P);
  uint8_t* act = ws->pf_act;
  k_pf_embed<<<dim3((ne + 255) / 256, P), 256, 0, st>>>(m->emb, hp.vocab_size, ne, ws->pf_ids,
                                                        ws->pf_x, ws->d_res);
  CUDA_TRY(cudaGetLastError());
  for (int l = 0; l < hp.n_layers; ++l) {
    const LayerW& L = m->layers[l];
    uint8_t* kv = static_cast<uint8_t*>(s->kv) + (size_t)l * s->layer_elems * es;
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
          s->ctx, m->kv_f16);
      CUDA_TRY(cudaGetLastError());
    }
    if (l == hp.n_layers - 1) break;
    // attention, infer.go:130-175
    switch (hd) {
      case 32: CUDA_TRY(launch_pf_attention<32>(m, ws, kv, P, pos0, s->ctx, st)); break;
      case 64: CUDA_TRY(launch_pf_attention<64>(m, ws, kv, P, pos0, s->ctx, st)); break;
      case 128: CUDA_TRY(launch_pf_attention<128>(m, ws, kv, P, pos0, s->ctx, st)); break;
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
      cudaMemset(ws->d_res, 0, sizeof(Result));
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
  const size_t es = m->kv_f16 ? 2 : 4;
  int max_pos = 0;
  for (int i = 0; i < n; ++i) {
    const l3g_state* s = states[i];
    if (!s) return l3g_fail(L3G_E_INVALID, "null state %d", i);
    if (s->m != m) return l3g_fail(L3G_E_INVALID, "state %d belongs to another model", i);
    for (int j = 0; j < i; ++j)
      if (states[j] == s) return l3g_fail(L3G_E_INVALID, "state %d appears twice", i);
    if (s->pos >= s->ctx) return l3g_fail(L3G_E_CTX, "context length exceeded (%d)", s->ctx);
    if (tokens[i] < 0 || tokens[i] >= m->hp.vocab_size)
      return l3g_fail(L3G_E_TOKEN, "token out of range: %d", tokens[i]);
    SeqInfo& q = b->h_seq[i];
    q = SeqInfo{};
    q.kv = s->kv;
    q.rope_cos = s->rope_cos;
    q.rope_sin = s->rope_sin;
    q.layer_bytes = (long long)(s->layer_elems * es);
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
  const int splits = (max_pos + 1 + BD_SPLIT - 1) / BD_SPLIT;
  const float scale = (float)(1.0 / sqrt((double)hd));
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
        b->d_res, wait_ns);                                                                   \
  else                                                                                       \
    k_bd_attention<HD, GP, float><<<grid, BD_THREADS, bd_smem_bytes(HD, 4, GP), st>>>(       \
        b->q, b->d_seq, l, m->group, m->hq_l, scale, b->part_o, b->part_ml, b->max_splits,     \
        b->d_res, wait_ns)
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
                                                   b->max_splits, b->att);
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

// ---------------------------------------------------------------------------
// failure-detection self test
// ---------------------------------------------------------------------------
extern "C" int l3g_selftest_bounded_wait(int32_t device, int32_t timeout_us, int32_t* status) {
  if (!status) return l3g_fail(L3G_E_INVALID, "null argument");
  if (timeout_us <= 0 || timeout_us > 1000000)
    return l3g_fail(L3G_E_INVALID, "timeout_us must be in (0, 1e6]");
  int dev = device;
  if (dev < 0) CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaSetDevice(dev));
  Result* d = nullptr;
  CUDA_TRY(cudaMalloc(&d, sizeof(Result)));
  cudaMemset(d, 0, sizeof(Result));
  k_selftest_wait<<<1, 32>>>(d, (unsigned long long)timeout_us * 1000ull);
  cudaError_t e = cudaDeviceSynchronize();
  Result h{};
  if (e == cudaSuccess) e = cudaMemcpy(&h, d, sizeof h, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "selftest: %s", cudaGetErrorString(e));
  *status = h.err == ERR_TIMEOUT ? L3G_E_DEVICE : (h.err ? -100 - h.err : L3G_OK);
  return L3G_OK;
}
