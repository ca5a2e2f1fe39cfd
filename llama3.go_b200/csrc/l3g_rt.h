// Host runtime of libl3g, shared by its translation units (not part of the
// public ABI): the handle types behind include/l3g.h (model, state,
// workspace), the error and CUDA helpers, and the functions one unit
// provides to another.
//
// Units: l3g_api.cu (errors, options, NCCL binding, self test),
// l3g_model.cu (model upload and repack, KV states, snapshots),
// l3g_tp.cu (tensor-parallel exchange set-up), l3g_step.cu (workspaces,
// the per-step graphs and every per-token entry, the matrix entries),
// l3g_persist_host.cu (the persistent layer kernel), l3g_batched.cu (the
// tensor-core product, batched prefill, batched decode).  A kernel is set
// up (attributes) and launched in the same unit: each unit is its own
// device module.
#pragma once

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

#define CUDA_TRY(expr)                                                     \
  do {                                                                     \
    cudaError_t e_ = (expr);                                               \
    if (e_ != cudaSuccess)                                                 \
      return l3g_fail(L3G_E_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

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
NcclApi* nccl();

#define NCCL_TRY(expr)                                                      \
  do {                                                                      \
    ncclResult_t r_ = (expr);                                               \
    if (r_ != ncclSuccess)                                                  \
      return l3g_fail(L3G_E_NCCL, "%s: %s", #expr, nccl()->GetErrorString(r_)); \
  } while (0)

int sm_count(int dev);
// Sets the kernels' attributes of the per-token step (l3g_step.cu), once
// per device, with that device current.
int setup_kernels();

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

struct DevMat {
  Q8Tiles t{};
  uint8_t* buf = nullptr;
  size_t bytes = 0;
  int nstages = 2;
  int smem = 0;
};

// model
// ---------------------------------------------------------------------------
// A matrix in the batched product's weight chunks (l3g_gemm_layout.h).
struct GemmMat {
  uint8_t* data = nullptr;
  int rows = 0, cols = 0, nk = 0, n_rt = 0;
  size_t bytes = 0;
};

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

// ---------------------------------------------------------------------------
// state
// ---------------------------------------------------------------------------
// A pool of KV pages: one device allocation of n_pages pages, each KV_PAGE
// K|V rows of one (layer, kv head) of its model.  States take pages as their
// position grows and give them back when freed.  A state made by
// l3g_state_new has a private pool holding exactly its pages (freed with
// it); l3g_kvpool_new makes a pool several states share.
struct l3g_kvpool {
  l3g_model* m = nullptr;
  int device = 0;
  uint8_t* base = nullptr;
  int n_pages = 0;
  size_t page_bytes = 0;
  std::mutex mu;
  std::vector<int> free_pages;  // a stack of free page ids
  int states = 0;               // states holding pages of it
  bool released = false;        // its owner freed it: destroyed with its last state
  bool priv = false;            // a state's private pool
};

struct l3g_state {
  l3g_model* m = nullptr;
  int device = 0;
  int ctx = 0, pos = 0;
  l3g_kvpool* pool = nullptr;  // where its pages live
  int pps = 0;                 // pages per (layer, kv head): ceil(ctx / KV_PAGE)
  int* d_pages = nullptr;      // page table [n_layers * local kv heads][pps] (device)
  std::vector<int> h_pages;    // its host copy; -1: not mapped
  int mapped = 0;              // logical pages [0, mapped) of every (layer, kv head) mapped
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  uint64_t serial = 0;
};
// The device view of a state's cache.
KvMap state_kv(const l3g_state* s);  // l3g_model.cu
// Maps pages for positions [0, n_pos) of every (layer, kv head), taking
// them from the state's pool, and copies the new table entries to the
// device on stream st (ordered before the kernels that use them).
int state_map(l3g_state* s, int n_pos, cudaStream_t st);  // l3g_model.cu

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
  int att_cnt_n = 0;  // entries of att_cnt
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

// provided by one unit to the others
struct RowSrc {         // rows [row0, row0+n) of a host GGUF Q8_0 tensor
  const uint8_t* host;
  int row0, n;
};
// Uploads the needed source rows, repacks them into tiles on the device.
// rpw > 0 fixes the rows per warp (the persistent kernel's layout); 0 plans.
int upload_tiled(DevMat& out, const RowSrc* segs, int nseg, bool interleave2, int src_cols,
                 int blk0, int cols, int nsm, size_t* dev_bytes, int rpw = 0);  // l3g_model.cu
void free_mat(DevMat& m);                             // l3g_model.cu
void free_gemm(GemmMat& g);                           // l3g_model.cu
void ws_release(l3g_workspace* ws);
// After a step reported a device error: clears the result word and every
// last-arriver counter an aborted kernel may have left mid-count.
void ws_clear_device_error(l3g_workspace* ws);                   // l3g_step.cu
void ws_detach(l3g_workspace* ws);                    // l3g_step.cu: releases its graphs, forgets the model
int tp_setup(l3g_workspace* ws);                      // l3g_tp.cu
TpExchange tp_exchange(const l3g_workspace* ws, int phase);  // l3g_tp.cu
int persist_setup(l3g_workspace* ws);                 // l3g_persist_host.cu
size_t persist_stamp_bytes(const l3g_workspace* ws);  // l3g_persist_host.cu
// Enqueues the persistent layer kernel (every layer of a step) on st.
cudaError_t launch_layers(const l3g_workspace* ws, const l3g_state* s,
                          unsigned long long* stamps, cudaStream_t st);  // l3g_persist_host.cu
// The persistent kernel's barrier stamps of a traced step live in the trace
// buffer after the first kPersistStampSlot launches' per-CTA stamps (the
// step's other kernels stamp there), [barrier][cta]{arrival, release}.
constexpr size_t kPersistStampSlot = 16;
constexpr size_t kPersistStampOff = kPersistStampSlot * TRACE_CTAS * 8;  // in 64-bit words

