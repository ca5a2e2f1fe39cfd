/*
 * l3g.h -- C ABI of libl3g.so, the B200 (sm_100a) decode library for
 * llama3.go.  Plain pointers and sizes only, so a cgo shim (build tag
 * "cuda") can replace:
 *   - the cgo SIMD kernels   internal/llama/simd.h:7-9 (matvec_q8_c,
 *     dot_product), bound in matvec_cgo.go:14-30 and dot_cgo.go:16-22;
 *   - the goroutine pool     internal/llama/workers.go:21-116
 *     (WorkerPool.Run / ParallelFor), held as Model.Pool (model.go:52);
 *   - the per-token forward  internal/llama/infer.go:21-267 and :269-511.
 * The Go Model / State / Workspace / Sampler API stays; each of its calls maps
 * onto one entry point below.
 *
 * Conventions
 *   - Every function returns an int status: L3G_OK (0) or a negative code;
 *     l3g_last_error() returns the message of the calling thread's last
 *     failure.  Messages reuse the reference's wording where one exists
 *     (e.g. "context length exceeded (%d)", infer.go:23).
 *   - Host pointers unless a parameter says "device".  The library owns all
 *     device memory; it keeps no caller pointer after a call returns.
 *   - A state / workspace is used by one host thread at a time (as the
 *     reference's Workspace, workspace.go:3-4).
 *   - Tensor-parallel runs use one process (or thread) per GPU; ranks pass
 *     the same l3g_options.nccl_id, obtained on rank 0 from
 *     l3g_nccl_unique_id() and shared by the caller.
 */
#ifndef L3G_H
#define L3G_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define L3G_VERSION 1

/* status codes */
#define L3G_OK 0
#define L3G_E_INVALID (-1) /* bad argument, shape or tensor type          */
#define L3G_E_CUDA (-2)    /* CUDA runtime error                          */
#define L3G_E_NCCL (-3)    /* NCCL missing or failed                      */
#define L3G_E_CTX (-4)     /* context length exceeded, infer.go:22-24     */
#define L3G_E_TOKEN (-5)   /* token out of range, infer.go:514-516        */
#define L3G_E_FORMAT (-6)  /* GGUF parse / missing tensor or hyperparam   */
#define L3G_E_DEVICE (-7)  /* a kernel's own check failed (bounded wait
                              ran out, index out of range): see message  */

/* ggml tensor type ids, internal/llama/q8_0.go:7-11 */
#define L3G_TYPE_F32 0
#define L3G_TYPE_F16 1
#define L3G_TYPE_Q8_0 8

/* KV cache element type */
#define L3G_KV_F32 0 /* the reference's layout type (state.go:8-9)      */
#define L3G_KV_F16 1 /* half the KV bytes per token                      */

typedef struct l3g_model l3g_model;
typedef struct l3g_state l3g_state;
typedef struct l3g_workspace l3g_workspace;
typedef struct l3g_matrix l3g_matrix;
typedef struct l3g_gemm_matrix l3g_gemm_matrix;
typedef struct l3g_batch l3g_batch;

/* HyperParams, internal/llama/model.go:10-21.  llama3 RoPE frequency scaling,
 * absent from the reference (rope.go:15-37), is taken from an optional f32
 * tensor "rope_freqs.weight" of rope_dim/2 divisors (llama.cpp's
 * convention); without it the tables are exactly the reference's. */
typedef struct {
  int32_t vocab_size;
  int32_t n_layers;
  int32_t n_emb;
  int32_t n_heads;
  int32_t n_heads_kv;
  int32_t n_ff;
  int32_t rope_dim;
  int32_t ctx_len;
  float rms_eps;
  float rope_base;
} l3g_hparams;

/* One tensor of the model file: gguf.TensorInfo + Tensor.Data
 * (internal/gguf/gguf.go:47-53, internal/llama/tensor.go:9-12).  dims are
 * ne0-first ([cols, rows] for matrices).  data points at the tensor's first
 * byte (e.g. into the mmapped GGUF); nbytes may be 0 (then derived). */
typedef struct {
  const char *name;
  uint32_t type;
  uint32_t n_dims;
  uint64_t dims[4];
  const void *data;
  uint64_t nbytes;
} l3g_tensor;

/* Placement of a model: single GPU or tensor-parallel rank. */
typedef struct {
  int32_t world_size; /* 1 = single GPU                                   */
  int32_t rank;       /* 0 .. world_size-1                                */
  int32_t device;     /* CUDA device ordinal, -1 = the current device      */
  int32_t kv_dtype;   /* L3G_KV_F32 or L3G_KV_F16                         */
  uint8_t nccl_id[128]; /* ncclUniqueId shared by all ranks (world > 1)   */
} l3g_options;

/* TopKItem, internal/llama/topk.go:5-8 */
typedef struct {
  int32_t id;
  float logit;
} l3g_topk_item;

/* ---- library ----------------------------------------------------------- */
const char *l3g_last_error(void);
int l3g_version(void);
int l3g_device_count(int32_t *n);
/* ncclGetUniqueId for rank 0 of a tensor-parallel group. */
int l3g_nccl_unique_id(uint8_t out[128]);
void l3g_options_default(l3g_options *opt);

/* Tensor-parallel shard of one rank (the reference has no parallelism beyond
 * its goroutine pool, workers.go:88-116; this is the split the library uses):
 * attention by heads, FFN by rows, Wo / down by the matching columns, logits
 * by vocab rows.  Row / column ranges are [start, start + count). */
typedef struct {
  int32_t q_row0, q_rows;         /* rows of attn_q                       */
  int32_t kv_row0, kv_rows;       /* rows of attn_k and attn_v            */
  int32_t o_col0, o_cols;         /* columns of attn_output               */
  int32_t ff_row0, ff_rows;       /* rows of ffn_up and ffn_gate          */
  int32_t down_col0, down_cols;   /* columns of ffn_down                  */
  int32_t vocab_row0, vocab_rows; /* rows of output.weight (or tied emb)  */
  int32_t vocab_stride;           /* rows per rank before the last shard  */
} l3g_shard;
/* Host-only: validates hp for world_size ranks and fills this rank's shard. */
int l3g_shard_plan(const l3g_hparams *hp, int32_t world_size, int32_t rank,
                   l3g_shard *out);

/* ---- model: LoadModel (model.go:55-156), Close (model.go:158-166) ------- */
/* Uploads the Q8_0 blocks once (values unchanged, repacked into 16-byte
 * aligned tiles) plus f32 norms; keeps no host pointer.  Tensor names as
 * model.go:83-138; output.weight optional (tied, model.go:91-94). */
int l3g_model_load(const l3g_hparams *hp, const l3g_tensor *tensors,
                   int32_t n_tensors, const l3g_options *opt,
                   l3g_model **out);
/* Same, parsing the GGUF file itself (gguf.go:64-234, readHyperParams
 * model.go:168-219). */
int l3g_model_load_gguf(const char *path, const l3g_options *opt,
                        l3g_model **out);
int l3g_model_hparams(const l3g_model *m, l3g_hparams *out);
void l3g_model_free(l3g_model *m);

/* ---- state: NewState (state.go:51-64), KV cache in HBM ------------------ */
/* The KV cache is paged.  The reference's KVCache (state.go:3-23) is one
 * contiguous [layer][pos][kv head][hd] block per State.  Here a page holds
 * L3G_KV_PAGE consecutive positions (K | V rows) of one (layer, kv head),
 * and each state has a page table from (layer, kv head, position /
 * L3G_KV_PAGE) to pages of a pool; attention and the KV append go through
 * that table.  l3g_state_new gives the state a private pool with every page
 * of its context mapped at once (ctx_len rounded up to L3G_KV_PAGE). */
#define L3G_KV_PAGE 256
int l3g_state_new(l3g_model *m, int32_t ctx_len, l3g_state **out);
/* A pool of n_pages pages shared by many states (a server's sessions):
 * l3g_state_new_in_pool makes a state that takes pages from it as its
 * position grows (before each step, for the positions the step writes) and
 * returns them when freed; a step that finds no free page fails with
 * L3G_E_CTX ("KV pool exhausted").  l3g_kvpool_page_bytes gives a page's
 * size for the model, to size the pool; l3g_kvpool_free_pages counts the
 * free ones; l3g_state_pages counts the pages a pooled state holds (0 for a
 * private pool).  The pool must be freed after the model's workspaces and
 * before the model; freeing it while states still hold pages defers its
 * release to the last of them. */
typedef struct l3g_kvpool l3g_kvpool;
int l3g_kvpool_page_bytes(const l3g_model *m, uint64_t *bytes);
int l3g_kvpool_new(l3g_model *m, int32_t n_pages, l3g_kvpool **out);
void l3g_kvpool_free(l3g_kvpool *p);
int l3g_kvpool_free_pages(l3g_kvpool *p, int32_t *n);
int l3g_state_new_in_pool(l3g_model *m, l3g_kvpool *pool, int32_t ctx_len,
                          l3g_state **out);
int l3g_state_pages(const l3g_state *s, int32_t *mapped);
int l3g_state_pos(const l3g_state *s, int32_t *pos);
int l3g_state_ctx_len(const l3g_state *s, int32_t *ctx_len);
/* Moves the write position (0 <= pos <= ctx): rewinds a session for reuse
 * (the REPL's /reset, main.go:120-122) without reallocating. */
int l3g_state_set_pos(l3g_state *s, int32_t pos);
/* Session snapshot (a KV-cache checkpoint; no counterpart in the reference,
 * whose State lives in Go memory and is rebuilt by ingesting the prompt
 * again, main.go:120-122 and :276-286).  A snapshot holds the position and
 * this rank's KV rows of positions [0, pos) plus a header (model shape,
 * shard, KV element type), in host memory.  _bytes gives its size; restore
 * loads it into a state of the same model shape and shard whose context
 * length is at least the snapshot's position, and sets that position. */
int l3g_state_snapshot_bytes(const l3g_state *s, uint64_t *bytes);
int l3g_state_snapshot(const l3g_state *s, void *dst, uint64_t bytes);
int l3g_state_restore(l3g_state *s, const void *src, uint64_t bytes);
void l3g_state_free(l3g_state *s);

/* ---- workspace: NewWorkspace (workspace.go:35-69) ------------------------ */
/* Device activations, scratch, stream and the captured per-step CUDA graphs.
 * ctx_len <= 0 or > model ctx is clamped like workspace.go:36-41; top_k <= 0
 * means 40 (workspace.go:42-44). */
int l3g_workspace_new(l3g_model *m, int32_t ctx_len, int32_t top_k,
                      l3g_workspace **out);
void l3g_workspace_free(l3g_workspace *ws);

/* ---- per-token forward ---------------------------------------------------- */
/* ForwardIntoWorkspace, infer.go:21-267: one token through all layers; fills
 * logits_out[vocab] (host) when non-NULL, otherwise skips the logits matvec
 * like infer.go:250 (prefill).  Advances the state's position. */
int l3g_forward(l3g_model *m, l3g_state *s, l3g_workspace *ws, int32_t token,
                float *logits_out);
/* ForwardTopKIntoWorkspace, infer.go:269-511: the top_k largest logits
 * (top_k <= 0 means 40, at most 64), sorted by descending logit, ties by
 * lower id.  *n_items receives the count. */
int l3g_forward_topk(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                     int32_t token, int32_t top_k, l3g_topk_item *items,
                     int32_t *n_items);
/* The attention softmax of ForwardTopKIntoWorkspace exactly as the reference
 * computes it (infer.go:376-423): weights fastExp(score - max) with max over
 * all positions (infer.go:404,520-525) instead of the exact exp of
 * ForwardIntoWorkspace (infer.go:130-175).  With on = 1 the top-K and sampled
 * calls of this workspace (l3g_forward_topk, l3g_forward_sample,
 * l3g_decode_sample) run that attention, so their items are the reference
 * top-K path's; l3g_forward, l3g_forward_argmax, l3g_decode_greedy and
 * l3g_prefill keep the exact exp, as the reference's full path does.  Off
 * (the exact exp everywhere) by default.  The first call with on = 1
 * allocates the pass's scratch (scores of every local query head over the
 * workspace's context), so make it before any stream capture. */
int l3g_workspace_set_topk_fast_exp(l3g_workspace *ws, int32_t on);
/* Greedy decode step: argmax (lowest id on ties) of the logits that
 * l3g_forward would return, computed on the device. */
int l3g_forward_argmax(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                       int32_t token, int32_t *next_token, float *max_logit);
/* ingest, cmd/go-llama-chat/main.go:276-286: l3g_forward without logits for
 * each token in turn. */
int l3g_prefill(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                const int32_t *tokens, int32_t n);
/* The same ingest as l3g_prefill (KV entries of positions pos..pos+n-1,
 * position advanced by n, no logits), computed up to 512 tokens at a time:
 * every projection as one batched Q8_0 product on the tensor cores
 * (l3g_gemm_q8) over the tokens of the pass, causal attention of the pass's
 * positions over the cache, and the last layer cut after its K/V append
 * (its attention and FFN outputs feed only the logits).  The reference
 * ingests one token per ForwardIntoWorkspace (main.go:276-286); per token the
 * arithmetic is the same (quantized activations, int32 block sums), with
 * fp32 sums in another order. */
int l3g_prefill_batched(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                        const int32_t *tokens, int32_t n);
/* The decode loop of cmd/go-llama-chat/main.go:141-165 with a greedy
 * sampler: n steps, each fed the previous step's argmax, replayed back to
 * back on the device with no host round trip in between.  out_tokens[i]
 * (host, n entries) is the argmax after step i; device_ms (nullable)
 * receives the device time of the n steps (CUDA events on the workspace's
 * stream).  Advances the position by n. */
int l3g_decode_greedy(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                      int32_t first_token, int32_t n, int32_t *out_tokens,
                      float *device_ms);
/* ForwardTopKIntoWorkspace (infer.go:269-511) followed by Sampler.SampleTopK
 * (sampling.go:103-143) on the device: float64 temperature softmax over the
 * top-K items, cumulative pick with a uniform draw from Philox4x32-10 keyed
 * by `seed` and counted by the workspace's draw index (the reference draws
 * from Go's math/rand, whose stream is not reproduced).  temperature <= 0
 * means 0.8 and top_k <= 0 the workspace's top-K, as NewSampler
 * (sampling.go:19-30).  Advances the position. */
int l3g_forward_sample(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                       int32_t token, int32_t top_k, float temperature,
                       uint64_t seed, int32_t *next);
/* The sampled decode loop on the device (n steps: step i ingests a token and
 * samples out_tokens[i], which step i+1 ingests; one host synchronization),
 * then the chat loop's stop rule (cmd/go-llama-chat/main.go:146-150):
 * *n_out counts the samples up to and including the first of stop_ids (n if
 * none).  The position covers the ingested tokens through the stop token's
 * own ingestion when the loop ran it (*n_out + 1 steps), else all n steps
 * (a stop token sampled last is not yet ingested: the caller ingests it, as
 * main.go:148 does). */
int l3g_decode_sample(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                      int32_t first_token, int32_t n, int32_t top_k,
                      float temperature, uint64_t seed, const int32_t *stop_ids,
                      int32_t n_stop, int32_t *out_tokens, int32_t *n_out,
                      float *device_ms);
/* Kernels of this library one step launches (greedy variant), for launch
 * accounting. */
int l3g_workspace_kernels_per_step(l3g_workspace *ws, int32_t *n);
/* Attention layout the workspace chose: splits per kv head, and the cluster
 * size when the splits of a kv head merge as one thread-block cluster (0:
 * they merge through global memory).  Inspection only; no reference
 * counterpart (the reference attends on one goroutine, infer.go:130-175). */
int l3g_workspace_attention_layout(const l3g_workspace *ws, int32_t *splits,
                                   int32_t *cluster);
/* Tensor-parallel reduction the workspace uses: 1 when the Wo / down partial
 * sums travel over peer memory (CUDA IPC mappings, pushed by the producing
 * matvec and summed by the next kernel), 0 for NCCL allreduces (or a single
 * GPU).  Inspection only; no reference counterpart (the reference is one
 * process on one CPU). */
int l3g_workspace_tp_p2p(const l3g_workspace *ws, int32_t *p2p);

/* Profiling (the device counterpart of the chat CLI's -cpuprofile,
 * cmd/go-llama-chat/main.go:35-54): runs one greedy step eagerly, each kernel
 * serialized and bracketed by CUDA events, and reports per launch its kind
 * (L3G_K_*) and device time in microseconds.  Advances the position like a
 * step.  *n is the capacity on entry and the count on return. */
#define L3G_K_EMBED 0
#define L3G_K_QKV 1
#define L3G_K_ATTN 2
#define L3G_K_WO 3
#define L3G_K_UPGATE 4
#define L3G_K_DOWN 5
#define L3G_K_LOGITS 6
#define L3G_K_OTHER 7
#define L3G_K_ACT_QUANT 8 /* act-quant of the SwiGLU output for down     */
#define L3G_K_LAYERS 9    /* every layer in one persistent launch         */
int l3g_profile_step(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                     int32_t token, int32_t *kinds, float *us, int32_t *n);
/* Device timeline of one greedy step replayed as its CUDA graph (kernels
 * overlapping as in production): for each launch i, kinds[i] (L3G_K_*) and
 * stamps[(i * L3G_TRACE_CTAS + cta) * 8 + e] = %globaltimer (ns) of CTA cta
 * at e = {entry, dependency wait done, prologue done, tile loop done, exit};
 * zero where a launch or CTA records nothing.  Advances the position by one.
 * *n is the capacity in launches on entry and the count on return. */
#define L3G_TRACE_CTAS 256
int l3g_trace_step(l3g_model *m, l3g_state *s, l3g_workspace *ws,
                   int32_t token, uint64_t *stamps, int32_t *kinds,
                   int32_t *n);

/* Persistent layer kernel (opt-in: L3G_PERSIST=1 in the environment when the
 * model is loaded).  It replaces the per-layer launches of a step, i.e. the
 * per-row-chunk matvec calls and the goroutine fork-join of
 * ForwardIntoWorkspace's layer loop (infer.go:56-246, workers.go:98-112),
 * with one launch of one CTA per SM whose layer phases are separated by grid
 * barriers.  *on = 1 when this workspace's steps use it.  Inspection only. */
int l3g_workspace_persistent(const l3g_workspace *ws, int32_t *on);
/* The persistent kernel's layout on this workspace: ring slots and their
 * bytes, attention splits per kv head, grid-barrier counters, shared memory
 * per CTA, grid barriers per layer (7, one less with the SwiGLU act-quant
 * fused into the up/gate phase, one less with the split merge fused into the
 * attention phase).  Inspection only (L3G_PERSIST_STAGES, L3G_PERSIST_SPLITS,
 * L3G_PERSIST_BAR_SPREAD, L3G_PERSIST_FUSE_QUANT and L3G_PERSIST_FUSE_MERGE,
 * read at workspace creation, cap or set them). */
int l3g_persist_layout(const l3g_workspace *ws, int32_t *stages, int32_t *slot_bytes,
                       int32_t *splits, int32_t *counters, int32_t *smem_bytes,
                       int32_t *barriers_per_layer);
/* After l3g_trace_step on a workspace that runs the persistent kernel: the
 * %globaltimer (ns) at which each CTA arrived at and left each grid barrier
 * of the traced step, out[(b * grid + cta) * 2 + {0, 1}] for barrier b (per
 * layer: after QKV, attention, merge, Wo, up/gate, [quantize,] down; the
 * last layer's down has none, so its slots stay 0).  *n_barriers = barriers
 * per layer x layers.  cap is out's length in 64-bit words.  No reference
 * counterpart (tracing). */
int l3g_persist_stamps(const l3g_workspace *ws, uint64_t *out, int64_t cap,
                       int32_t *n_barriers, int32_t *grid);

/* ---- Q8_0 matvec drop-in: matvec_q8_c (simd.h:8) / matVecQ8_0 ------------ */
/* Uploads a GGUF Q8_0 matrix (rows x cols, 34-byte blocks, host bytes). */
int l3g_matrix_upload(const void *q8_0_rows, int32_t rows, int32_t cols,
                      int32_t device, l3g_matrix **out);
/* out[r] = sum_b (fp16(w.d[r,b]) * x_scales[b]) * (sum_i w.q[r,b,i] *
 * x_qs[b*32+i]) for r in [start_row, end_row).  x_scales, x_qs, out are
 * DEVICE pointers; stream is a cudaStream_t (NULL = default stream). */
int l3g_matvec_q8(const l3g_matrix *w, const float *x_scales,
                  const int8_t *x_qs, float *out, int32_t start_row,
                  int32_t end_row, void *stream);
void l3g_matrix_free(l3g_matrix *w);
int l3g_matrix_device_bytes(const l3g_matrix *w, uint64_t *bytes);

/* ---- matvec + argmax without allocation ---------------------------------- */
/* No counterpart in the reference: the reference has no greedy or argmax
 * step at all (its Sampler forces a temperature of 0.8 when given 0,
 * sampling.go:20-22, and always samples).  This entry runs the same Q8_0
 * matvec as l3g_matvec_q8 over all rows and the argmax over the rows (ties
 * to the lowest row) in one launch.  It allocates nothing, at any call: the
 * cross-CTA reduction uses a fixed static device array of
 * L3G_ARGMAX_STATIC_MAX_CTAS per-CTA slots plus one arrival counter, so a
 * caller holding no workspace (the matrix handle is all it has, as with
 * matvec_q8_c) and unable to allocate (device memory fully committed to
 * weights and KV cache, or a stream that must not be stalled by
 * cudaMalloc/cudaFree, which synchronize the device) can still get a greedy
 * token without a host round trip over the logits.
 *  - x_scales, x_qs, out, result are DEVICE pointers; out may be NULL (the
 *    logits are then not stored).  *result is set on the stream to
 *    {-1, 0, 0, 0} and then receives {index, value, status, detail} from the
 *    launch: status 0 unless a bounded wait of the kernel gave up (then an
 *    internal code, detail = wait site).  An index still -1 after the stream
 *    completes means the launch's cross-CTA merge never ran (see overlap
 *    below).
 *  - max_ctas caps the CTAs of the launch (0: one per SM); values above
 *    L3G_ARGMAX_STATIC_MAX_CTAS, or an SM count above it, are rejected with
 *    L3G_E_INVALID.
 *  - The first call on a device does the set-up (looks up the static array's
 *    device address with that device current); make that first call before
 *    any stream capture on the device.  A failed set-up is not latched: it
 *    reports its CUDA error and the next call retries.  The caller's current
 *    device is the same after the call as before it.
 *  - The arrival counter must be zero when a launch starts: every call
 *    clears it on its stream before its launch; the slots need no initial
 *    value.  The array is shared by every call on the device, so calls that
 *    overlap in time (other streams, other threads) race and give wrong
 *    results, possibly index -1: issue them on one stream, or serialize
 *    them.  The next call after an overlap starts from a cleared counter. */
#define L3G_ARGMAX_STATIC_MAX_CTAS 1024
typedef struct l3g_argmax_result {
  int32_t index;  /* row of the largest value                        */
  float value;    /* out[index]                                      */
  int32_t status; /* 0, or the device error of a bounded wait        */
  int32_t detail; /* wait site when status != 0                      */
} l3g_argmax_result;
int l3g_matvec_q8_argmax_static(const l3g_matrix *w, const float *x_scales,
                                const int8_t *x_qs, float *out,
                                l3g_argmax_result *result, int32_t max_ctas,
                                void *stream);

/* QuantizeQ8_0Into, q8_0.go:22-79, on the device (DEVICE pointers): d has
 * ceil(n/32) floats, qs ceil(n/32)*32 bytes. */
int l3g_quantize_q8_0(const float *x, int32_t n, float *d, int8_t *qs,
                      void *stream);

/* ---- batched decode: many sessions, one step ----------------------------- */
/* One decode step for n independent sessions of one model, each an
 * l3g_state with its own KV cache, context length and position (no two
 * entries the same state).  Per session the step is ForwardTopKIntoWorkspace
 * (infer.go:269-511, with the exact exp of the full path, :130-175) followed
 * by Sampler.SampleTopK (sampling.go:103-143): state i ingests tokens[i] at
 * its position and advances by one, and next_tokens[i] receives a sample
 * from its top_k largest logits (top_k <= 0: 40, at most 64; ties to the
 * lower id) at temperature (<= 0: 0.8), drawn from Philox4x32-10 keyed by
 * seeds[i] with the state's position before the step as the draw index
 * (Go's math/rand stream is not reproduced).  logits_out (nullable, host
 * [n][vocab]) receives the logits.  The projections run as batched Q8_0
 * products over the n tokens on the tensor cores (l3g_gemm_q8); attention
 * is per session over its own cache.  The reference serves one session
 * (cmd/go-llama-chat/main.go:139-176); this has no counterpart there.
 * Tensor parallel: every rank calls with its own states of the same
 * sessions and the same tokens and seeds, and gets the same samples. */
#define L3G_BATCH_MAX 256
int l3g_batch_new(l3g_model *m, int32_t max_seqs, l3g_batch **out);
void l3g_batch_free(l3g_batch *b);
int l3g_batch_step(l3g_batch *b, l3g_state *const *states, int32_t n,
                   const int32_t *tokens, int32_t top_k, float temperature,
                   const uint64_t *seeds, int32_t *next_tokens,
                   float *logits_out);

/* ---- batched Q8_0 product on the tensor cores (tcgen05 kind::i8) --------- */
/* n_tok independent Q8_0 matvecs over one weight matrix, as one GEMM:
 * out[n][r] = sum_b (fp16(w.d[r,b]) * x.d[n,b]) * (sum_i w.q[r,b,i] *
 * x.q[n,b*32+i]), i.e. matvec_q8_c (simd.h:8, simd.c:33-110; matVecQ8_0,
 * matvec_cgo.go:14-30) of every token's activation quantized by
 * QuantizeQ8_0Into (q8_0.go:22-79).  One int8 MMA per Q8_0 block (K = 32)
 * and the fp32 rescale by w.d * x.d per block, so each block's integer sum
 * is exact as in the reference.  The reference has no batched call: it runs
 * prompt tokens one ForwardIntoWorkspace at a time
 * (cmd/go-llama-chat/main.go:276-286); this is the building block of batched
 * prefill and batched decode.
 *  - l3g_gemm_matrix_upload repacks GGUF Q8_0 rows (host bytes, values
 *    unchanged) into 128-row x 128-column chunks on the device;
 *    l3g_gemm_repack is the same repack into a host buffer of
 *    l3g_gemm_matrix_bytes bytes (no device needed).
 *  - l3g_gemm_quantize quantizes x [n_tok][cols] (DEVICE f32) into the
 *    product's activation buffer act (DEVICE, l3g_gemm_act_bytes bytes,
 *    16-byte aligned), bit-identical to QuantizeQ8_0Into per row.
 *  - l3g_gemm_q8 writes out [n_tok][rows] (DEVICE f32); asynchronous on
 *    stream.  A matrix with fewer 128-row tiles than SMs splits its K range
 *    over CTAs into scratch the matrix owns (sized for 128 tokens), so
 *    products over one matrix must not overlap in time (one stream).  l3g_gemm_status synchronizes the device and returns (and
 *    clears) the error word of the kernel's bounded waits: err 0, or 1 with
 *    `where` naming the wait that gave up. */
int l3g_gemm_matrix_bytes(int32_t rows, int32_t cols, uint64_t *bytes);
int l3g_gemm_repack(const void *q8_0_rows, int32_t rows, int32_t cols, void *dst,
                    uint64_t dst_bytes);
int l3g_gemm_matrix_upload(const void *q8_0_rows, int32_t rows, int32_t cols,
                           int32_t device, l3g_gemm_matrix **out);
void l3g_gemm_matrix_free(l3g_gemm_matrix *w);
int l3g_gemm_act_bytes(int32_t n_tok, int32_t cols, uint64_t *bytes);
int l3g_gemm_quantize(const float *x, int32_t n_tok, int32_t cols, void *act,
                      void *stream);
int l3g_gemm_q8(const l3g_gemm_matrix *w, const void *act, int32_t n_tok,
                float *out, void *stream);
int l3g_gemm_status(const l3g_gemm_matrix *w, int32_t *err, int32_t *where);

/* ---- inspection (tests, debugging) --------------------------------------- */
/* KV entries of one layer for positions [pos0, pos0+npos) in the reference
 * layout [pos][kv_head][head_dim] (f32, host), this rank's kv heads only. */
int l3g_state_read_kv(const l3g_state *s, int32_t layer, int32_t pos0,
                      int32_t npos, float *k_out, float *v_out);
/* Workspace buffers after the last forward (f32, host). */
#define L3G_BUF_HIDDEN 0  /* residual stream x after the last layer [n_emb]  */
#define L3G_BUF_Q 1       /* last layer's roped query [local heads * hd]     */
#define L3G_BUF_ATTN 2    /* last layer's attention output [local heads*hd]  */
#define L3G_BUF_FFN_ACT 3 /* last layer's SwiGLU output [local n_ff]         */
#define L3G_BUF_LOGITS 4  /* logits of the last forward that made them [V]   */
int l3g_workspace_read(const l3g_workspace *ws, int32_t which, float *out,
                       int32_t n);

/* Runs a kernel that waits, with the library's bounded-wait helper, on a
 * barrier nothing completes; *status receives the device error code the
 * kernel reports (L3G_E_DEVICE expected).  Exercises failure detection
 * without hanging the GPU. */
int l3g_selftest_bounded_wait(int32_t device, int32_t timeout_us,
                              int32_t *status);

#ifdef __cplusplus
}
#endif
#endif /* L3G_H */
