/*
 * ORACLE -- test infrastructure only, never part of the product path.
 *
 * A plain-C restatement of llama3.go's per-token decode loop
 * (the Go sources under internal/llama), used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py to check and to time the CUDA
 * library.  Each function cites the reference file:line it restates.
 *
 * Matvec / dot backends, chosen per call:
 *   - "cgo":  the reference's own internal/llama/simd.c (matvec_q8_c,
 *             dot_product), compiled from the reference tree into
 *             oracle/_ref/libref_simd.so and bound with orc_load_ref_simd().
 *             This is what the reference's CGO_ENABLED=1 build runs
 *             (matvec_cgo.go:14-30, dot_cgo.go:16-22).
 *   - "pure": the Go fallbacks restated here (matvec_q8.go:6-34 ->
 *             q8_0.go:87-105, dot_pure.go:5-10).
 *
 * Parity status: the Q8_0 matvec and f32 dot are pinned to the reference
 * itself (its simd.c).  The Go orchestration restated below (norms, act-quant,
 * RoPE, attention, SwiGLU, top-K) is unpinned by reference outputs: no Go
 * toolchain exists here and the reference ships no golden vectors.  It is
 * cross-checked in tests against an independent float64 numpy forward.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off: no FMA contraction, so
 * f32 expressions round exactly as written, like Go's default GOAMD64=v1).
 */
#include <dlfcn.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* Reference simd.c binding (simd.h:7-9)                                     */
/* ------------------------------------------------------------------------ */
typedef void (*matvec_q8_fn)(const void *, const float *, const int8_t *,
                             float *, int, int, int);
typedef float (*dot_fn)(const float *, const float *, int);

static matvec_q8_fn g_ref_matvec_q8 = NULL;
static dot_fn g_ref_dot = NULL;

/* Loads the reference's compiled simd.c; returns 0 on success. */
int orc_load_ref_simd(const char *path) {
  void *h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) return -1;
  matvec_q8_fn mv = (matvec_q8_fn)dlsym(h, "matvec_q8_c");
  dot_fn dp = (dot_fn)dlsym(h, "dot_product");
  if (!mv || !dp) return -2;
  g_ref_matvec_q8 = mv;
  g_ref_dot = dp;
  return 0;
}
int orc_have_ref_simd(void) { return g_ref_matvec_q8 != NULL; }

/* Direct calls into the reference kernels (for per-op parity tests). */
int orc_ref_matvec_q8(const void *w, const float *xd, const int8_t *xqs,
                      float *out, int start, int end, int cols) {
  if (!g_ref_matvec_q8) return -1;
  g_ref_matvec_q8(w, xd, xqs, out, start, end, cols);
  return 0;
}
float orc_ref_dot(const float *a, const float *b, int n) {
  return g_ref_dot ? g_ref_dot(a, b, n) : NAN;
}

/* ------------------------------------------------------------------------ */
/* WorkerPool.ParallelFor (workers.go:88-116): contiguous chunks of          */
/* ceil(n/w), serial when n < w*64.                                          */
/* ------------------------------------------------------------------------ */
typedef void (*range_fn)(void *arg, int start, int end);

typedef struct {
  int workers;
  pthread_t *th;
  pthread_mutex_t mu;
  pthread_cond_t cv_go, cv_done;
  unsigned long gen;
  int pending;
  int stop;
  range_fn fn;
  void *arg;
  int n, chunk;
} orc_pool;

typedef struct {
  orc_pool *p;
  int idx;
} pool_worker_arg;

static void *pool_main(void *a_) {
  pool_worker_arg *a = (pool_worker_arg *)a_;
  orc_pool *p = a->p;
  int idx = a->idx;
  free(a);
  unsigned long seen = 0;
  for (;;) {
    pthread_mutex_lock(&p->mu);
    while (p->gen == seen && !p->stop) pthread_cond_wait(&p->cv_go, &p->mu);
    if (p->stop) {
      pthread_mutex_unlock(&p->mu);
      return NULL;
    }
    seen = p->gen;
    range_fn fn = p->fn;
    void *arg = p->arg;
    int n = p->n, chunk = p->chunk;
    pthread_mutex_unlock(&p->mu);
    int start = idx * chunk;
    if (start < n) {
      int end = start + chunk;
      if (end > n) end = n;
      fn(arg, start, end);
    }
    pthread_mutex_lock(&p->mu);
    if (--p->pending == 0) pthread_cond_signal(&p->cv_done);
    pthread_mutex_unlock(&p->mu);
  }
}

static orc_pool *pool_new(int workers) {
  orc_pool *p = (orc_pool *)calloc(1, sizeof(orc_pool));
  if (workers <= 0) workers = 1;
  p->workers = workers;
  pthread_mutex_init(&p->mu, NULL);
  pthread_cond_init(&p->cv_go, NULL);
  pthread_cond_init(&p->cv_done, NULL);
  p->th = (pthread_t *)calloc((size_t)workers, sizeof(pthread_t));
  for (int i = 0; i < workers; i++) {
    pool_worker_arg *a = (pool_worker_arg *)malloc(sizeof(pool_worker_arg));
    a->p = p;
    a->idx = i;
    pthread_create(&p->th[i], NULL, pool_main, a);
  }
  return p;
}

static void pool_free(orc_pool *p) {
  if (!p) return;
  pthread_mutex_lock(&p->mu);
  p->stop = 1;
  pthread_cond_broadcast(&p->cv_go);
  pthread_mutex_unlock(&p->mu);
  for (int i = 0; i < p->workers; i++) pthread_join(p->th[i], NULL);
  free(p->th);
  free(p);
}

/* workers.go:88-116 */
static void parallel_for(orc_pool *p, int n, range_fn fn, void *arg) {
  if (n <= 0) return;
  int w = p ? p->workers : 1;
  if (w <= 1 || n < w * 64) {
    fn(arg, 0, n);
    return;
  }
  int chunk = (n + w - 1) / w;
  pthread_mutex_lock(&p->mu);
  p->fn = fn;
  p->arg = arg;
  p->n = n;
  p->chunk = chunk;
  p->pending = w;
  p->gen++;
  pthread_cond_broadcast(&p->cv_go);
  while (p->pending > 0) pthread_cond_wait(&p->cv_done, &p->mu);
  pthread_mutex_unlock(&p->mu);
}

/* ------------------------------------------------------------------------ */
/* Scalar helpers                                                            */
/* ------------------------------------------------------------------------ */

/* f16ToF32, float16.go:7-38 (normals, subnormals, inf/nan). */
float orc_f16_to_f32(uint16_t u) {
  uint32_t sign = (uint32_t)(u >> 15) & 1u;
  uint32_t ex = (uint32_t)(u >> 10) & 0x1fu;
  uint32_t frac = (uint32_t)u & 0x3ffu;
  uint32_t out;
  if (ex == 0) {
    if (frac == 0) {
      out = sign << 31;
    } else {
      float m = (float)frac / 1024.0f;
      float v = (float)ldexp((double)m, -14);
      return sign ? -v : v;
    }
  } else if (ex == 0x1f) {
    out = (sign << 31) | 0x7f800000u | (frac << 13);
  } else {
    out = (sign << 31) | (((ex - 15u + 127u) & 0xffu) << 23) | (frac << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

static inline uint16_t rd_u16(const uint8_t *p) {
  return (uint16_t)(p[0] | ((uint16_t)p[1] << 8));
}

/* QuantizeQ8_0Into, q8_0.go:22-79: per 32-block f32 scale = maxabs/127
 * (1e-8 when zero), q = trunc(v/scale +- 0.5) clamped to [-128, 127]. */
void orc_quantize_q8_0(const float *x, int n, float *D, int8_t *qs) {
  int blocks = (n + 31) / 32;
  for (int b = 0; b < blocks; b++) {
    int start = b * 32;
    int end = start + 32;
    if (end > n) end = n;
    float maxAbs = 0.0f;
    for (int i = start; i < end; i++) {
      float v = x[i];
      if (v < 0) v = -v;
      if (v > maxAbs) maxAbs = v;
    }
    float scale = maxAbs / 127.0f;
    if (scale == 0.0f) scale = 1e-8f;
    D[b] = scale;
    float inv = 1.0f / scale;
    for (int i = 0; i < 32; i++) {
      int idx = start + i;
      float v = idx < n ? x[idx] : 0.0f;
      float f = v * inv;
      int q;
      if (f >= 0)
        q = (int)(f + 0.5f);
      else
        q = (int)(f - 0.5f);
      if (q > 127)
        q = 127;
      else if (q < -128)
        q = -128;
      qs[b * 32 + i] = (int8_t)q;
    }
  }
}

/* dotQ8_0Row, q8_0.go:87-105 (34-byte GGUF blocks: fp16 d + 32 int8). */
float orc_dot_q8_0_row(const uint8_t *row, const float *xD, const int8_t *xQs,
                       int blocks) {
  float sum = 0.0f;
  for (int b = 0; b < blocks; b++) {
    const uint8_t *blk = row + (size_t)b * 34;
    float dw = orc_f16_to_f32(rd_u16(blk));
    float s = dw * xD[b];
    int32_t acc = 0;
    for (int i = 0; i < 32; i++)
      acc += (int32_t)(int8_t)blk[2 + i] * (int32_t)xQs[b * 32 + i];
    sum += s * (float)acc;
  }
  return sum;
}

/* dot_pure.go:5-10 */
static float dot_pure(const float *a, const float *b, int n) {
  float sum = 0.0f;
  for (int i = 0; i < n; i++) sum += a[i] * b[i];
  return sum;
}

/* rmsNorm, math.go:5-14: f32 sum of squares, f64 sqrt. */
void orc_rmsnorm(float *out, const float *x, const float *w, int n,
                 float eps) {
  float ss = 0.0f;
  for (int i = 0; i < n; i++) ss += x[i] * x[i];
  float scale = (float)(1.0 / sqrt((double)(ss / (float)n + eps)));
  for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

/* silu, math.go:16-19 */
float orc_silu(float x) { return x / (1.0f + (float)exp((double)(-x))); }

/* fastExp, infer.go:520-525.  Go converts float32 -> uint32 on amd64 through
 * int64 (truncation toward zero) and keeps the low 32 bits. */
float orc_fast_exp(float x) {
  const uint32_t magic = 12102203u;
  const uint32_t bias = 1064866816u;
  float prod = x * (float)magic;
  uint32_t res = (uint32_t)(int64_t)prod + bias;
  float f;
  memcpy(&f, &res, 4);
  return f;
}

/* ------------------------------------------------------------------------ */
/* Model                                                                     */
/* ------------------------------------------------------------------------ */
typedef struct {
  int vocab_size, n_layers, n_emb, n_heads, n_heads_kv, n_ff, rope_dim,
      ctx_len;
  float rms_eps, rope_base;
  /* llama3 RoPE frequency scaling: an extension, absent from the reference
   * (rope.go:15-37).  factor <= 0 disables it. */
  float rope_factor, rope_low_freq, rope_high_freq;
  int rope_orig_ctx;
} orc_hparams;

typedef struct {
  const uint8_t *wq, *wk, *wv, *wo, *wup, *wgate, *wdown; /* Q8_0 GGUF bytes */
  const float *attn_norm, *ffn_norm;                      /* f32 [n_emb]    */
} orc_layer;

typedef struct {
  orc_hparams hp;
  const uint8_t *tok_emb;  /* Q8_0 [vocab][n_emb] */
  const uint8_t *out_proj; /* Q8_0 [vocab][n_emb] (== tok_emb when tied) */
  const float *out_norm;
  orc_layer *layers;
  orc_pool *pool;
} orc_model;

orc_model *orc_model_new(const orc_hparams *hp, const uint8_t *tok_emb,
                         const uint8_t *out_proj, const float *out_norm,
                         const orc_layer *layers, int threads) {
  orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
  m->hp = *hp;
  if (m->hp.rope_dim == 0) m->hp.rope_dim = hp->n_emb / hp->n_heads;
  if (m->hp.n_heads_kv == 0) m->hp.n_heads_kv = hp->n_heads;
  m->tok_emb = tok_emb;
  m->out_proj = out_proj ? out_proj : tok_emb; /* model.go:91-94 */
  m->out_norm = out_norm;
  m->layers = (orc_layer *)calloc((size_t)hp->n_layers, sizeof(orc_layer));
  memcpy(m->layers, layers, sizeof(orc_layer) * (size_t)hp->n_layers);
  m->pool = pool_new(threads);
  return m;
}

void orc_model_free(orc_model *m) {
  if (!m) return;
  pool_free(m->pool);
  free(m->layers);
  free(m);
}

int orc_model_threads(orc_model *m) { return m->pool->workers; }

/* ------------------------------------------------------------------------ */
/* RoPE cache (rope.go:15-52) and state (state.go:3-64)                      */
/* ------------------------------------------------------------------------ */

/* Published Llama-3.1 frequency-scaling rule applied to the inverse
 * frequencies (extension; see orc_hparams). */
static double llama3_scale_freq(double freq, const orc_hparams *hp) {
  const double two_pi = 6.283185307179586;
  double low_wavelen = (double)hp->rope_orig_ctx / hp->rope_low_freq;
  double high_wavelen = (double)hp->rope_orig_ctx / hp->rope_high_freq;
  double wavelen = two_pi / freq;
  if (wavelen < high_wavelen) return freq;
  if (wavelen > low_wavelen) return freq / hp->rope_factor;
  double smooth = ((double)hp->rope_orig_ctx / wavelen - hp->rope_low_freq) /
                  (hp->rope_high_freq - hp->rope_low_freq);
  return (1.0 - smooth) * freq / hp->rope_factor + smooth * freq;
}

/* NewRopeCache, rope.go:15-37: tables [pos][half] in f64 -> f32. */
void orc_rope_tables(const orc_hparams *hp, int ctx, float *cosT,
                     float *sinT) {
  int rope_dim = hp->rope_dim;
  int half = rope_dim / 2;
  double *inv = (double *)malloc(sizeof(double) * (size_t)(half > 0 ? half : 1));
  double b = (double)hp->rope_base;
  for (int i = 0; i < half; i++) {
    double e = (double)(2 * i) / (double)rope_dim;
    inv[i] = 1.0 / pow(b, e);
    if (hp->rope_factor > 0) inv[i] = llama3_scale_freq(inv[i], hp);
  }
  for (int pos = 0; pos < ctx; pos++)
    for (int i = 0; i < half; i++) {
      double ang = (double)pos * inv[i];
      cosT[(size_t)pos * half + i] = (float)cos(ang);
      sinT[(size_t)pos * half + i] = (float)sin(ang);
    }
  free(inv);
}

/* ApplyInPlace, rope.go:39-52: rotate adjacent pairs (2i, 2i+1). */
static void rope_apply(float *vec, const float *cosT, const float *sinT,
                       int half, int pos) {
  size_t base = (size_t)pos * half;
  for (int i = 0; i < half; i++) {
    float c = cosT[base + i], s = sinT[base + i];
    float x0 = vec[2 * i], x1 = vec[2 * i + 1];
    vec[2 * i] = x0 * c - x1 * s;
    vec[2 * i + 1] = x0 * s + x1 * c;
  }
}

typedef struct {
  int pos, ctx, n_layers, n_heads_kv, head_dim, half;
  float *K, *V;       /* [layer][pos][kvh][d] f32, state.go:3-23 */
  float *cosT, *sinT; /* [ctx][half] */
  /* workspace (workspace.go:3-69) */
  float *x, *xn, *attn, *proj, *ffn_in, *ffn_up, *ffn_gate, *ffn_act,
      *ffn_down, *q, *k, *v, *scores;
  float *q8d;
  int8_t *q8qs;
} orc_state;

orc_state *orc_state_new(orc_model *m, int ctx) {
  const orc_hparams *hp = &m->hp;
  /* NewState, state.go:51-64 */
  if (ctx <= 0) ctx = hp->ctx_len;
  if (ctx > hp->ctx_len) ctx = hp->ctx_len;
  orc_state *s = (orc_state *)calloc(1, sizeof(orc_state));
  int hd = hp->n_emb / hp->n_heads;
  s->ctx = ctx;
  s->n_layers = hp->n_layers;
  s->n_heads_kv = hp->n_heads_kv;
  s->head_dim = hd;
  s->half = hp->rope_dim / 2;
  size_t sz = (size_t)hp->n_layers * ctx * hp->n_heads_kv * hd;
  s->K = (float *)calloc(sz, sizeof(float));
  s->V = (float *)calloc(sz, sizeof(float));
  s->cosT = (float *)calloc((size_t)ctx * (s->half ? s->half : 1), sizeof(float));
  s->sinT = (float *)calloc((size_t)ctx * (s->half ? s->half : 1), sizeof(float));
  orc_rope_tables(hp, ctx, s->cosT, s->sinT);
  int ne = hp->n_emb, nf = hp->n_ff;
  int nmax = ne > nf ? ne : nf;
  s->x = (float *)calloc((size_t)ne, 4);
  s->xn = (float *)calloc((size_t)ne, 4);
  s->attn = (float *)calloc((size_t)ne, 4);
  s->proj = (float *)calloc((size_t)ne, 4);
  s->ffn_in = (float *)calloc((size_t)ne, 4);
  s->ffn_up = (float *)calloc((size_t)nf, 4);
  s->ffn_gate = (float *)calloc((size_t)nf, 4);
  s->ffn_act = (float *)calloc((size_t)nf, 4);
  s->ffn_down = (float *)calloc((size_t)ne, 4);
  s->q = (float *)calloc((size_t)ne, 4);
  s->k = (float *)calloc((size_t)hp->n_heads_kv * hd, 4);
  s->v = (float *)calloc((size_t)hp->n_heads_kv * hd, 4);
  s->scores = (float *)calloc((size_t)hp->n_heads * ctx, 4);
  s->q8d = (float *)calloc((size_t)(nmax + 31) / 32, 4);
  s->q8qs = (int8_t *)calloc((size_t)((nmax + 31) / 32) * 32, 1);
  return s;
}

void orc_state_free(orc_state *s) {
  if (!s) return;
  free(s->K); free(s->V); free(s->cosT); free(s->sinT);
  free(s->x); free(s->xn); free(s->attn); free(s->proj); free(s->ffn_in);
  free(s->ffn_up); free(s->ffn_gate); free(s->ffn_act); free(s->ffn_down);
  free(s->q); free(s->k); free(s->v); free(s->scores); free(s->q8d);
  free(s->q8qs);
  free(s);
}

int orc_state_pos(orc_state *s) { return s->pos; }
void orc_state_set_pos(orc_state *s, int pos) { s->pos = pos; }
int orc_state_ctx(orc_state *s) { return s->ctx; }
float *orc_state_k(orc_state *s) { return s->K; }
float *orc_state_v(orc_state *s) { return s->V; }
float *orc_state_hidden(orc_state *s) { return s->x; }
float *orc_state_q(orc_state *s) { return s->q; }
float *orc_state_attn(orc_state *s) { return s->attn; }
float *orc_state_ffn_act(orc_state *s) { return s->ffn_act; }

/* KVCache.idx, state.go:21-23 */
static inline size_t kv_idx(const orc_state *s, int layer, int pos, int head) {
  return ((((size_t)layer * s->ctx + pos) * s->n_heads_kv) + head) *
         (size_t)s->head_dim;
}

/* ------------------------------------------------------------------------ */
/* Matvec dispatch: matVecQ8_0 (matvec_cgo.go:14-30 / matvec_q8.go:6-34)      */
/* ------------------------------------------------------------------------ */
typedef struct {
  const uint8_t *w;
  const float *xd;
  const int8_t *xqs;
  float *out;
  int cols;
  int use_ref;
} mv_args;

static void mv_range(void *a_, int start, int end) {
  mv_args *a = (mv_args *)a_;
  if (a->use_ref) {
    g_ref_matvec_q8(a->w, a->xd, a->xqs, a->out, start, end, a->cols);
  } else {
    size_t row_bytes = (size_t)(a->cols / 32) * 34;
    for (int r = start; r < end; r++)
      a->out[r] = orc_dot_q8_0_row(a->w + (size_t)r * row_bytes, a->xd,
                                   a->xqs, a->cols / 32);
  }
}

static void matvec_q8(orc_model *m, const uint8_t *w, const float *xd,
                      const int8_t *xqs, float *out, int rows, int cols,
                      int use_ref) {
  mv_args a = {w, xd, xqs, out, cols, use_ref && g_ref_matvec_q8 != NULL};
  parallel_for(m->pool, rows, mv_range, &a);
}

/* Exposed for per-op tests: whole-matrix Q8_0 matvec through the pool. */
void orc_matvec_q8(orc_model *m, const uint8_t *w, const float *xd,
                   const int8_t *xqs, float *out, int rows, int cols,
                   int use_ref) {
  matvec_q8(m, w, xd, xqs, out, rows, cols, use_ref);
}

/* Embedding row dequant: embedInto infer.go:513-518 ->
 * readRowVecAnyToF32Into Q8_0 branch, tensor_read.go:128-147. */
static int embed_into(orc_model *m, int32_t token, float *dst, char *err,
                      int errlen) {
  if (token < 0 || token >= m->hp.vocab_size) {
    snprintf(err, (size_t)errlen, "token out of range: %d", token);
    return -1;
  }
  int cols = m->hp.n_emb, blocks = cols / 32;
  const uint8_t *row = m->tok_emb + (size_t)token * blocks * 34;
  for (int b = 0; b < blocks; b++) {
    float dw = orc_f16_to_f32(rd_u16(row + (size_t)b * 34));
    for (int i = 0; i < 32; i++)
      dst[b * 32 + i] = dw * (float)(int8_t)row[(size_t)b * 34 + 2 + i];
  }
  return 0;
}

/* keepTopKInsert, topk.go:10-30 (replace-min, strict >). */
static int keep_topk_insert(int32_t *ids, float *lg, int len, int k,
                            int32_t cid, float cl) {
  if (k <= 0) return len;
  if (len < k) {
    ids[len] = cid;
    lg[len] = cl;
    return len + 1;
  }
  int min_idx = 0;
  float min_val = lg[0];
  for (int i = 1; i < len; i++)
    if (lg[i] < min_val) {
      min_val = lg[i];
      min_idx = i;
    }
  if (cl > min_val) {
    ids[min_idx] = cid;
    lg[min_idx] = cl;
  }
  return len;
}

/* ------------------------------------------------------------------------ */
/* Forward: ForwardIntoWorkspace (infer.go:21-267) when fast == 0,           */
/* the body of ForwardTopKIntoWorkspace (infer.go:269-496, fastExp softmax)  */
/* when fast == 1.  The final norm + logits are done by the callers.         */
/* ------------------------------------------------------------------------ */
typedef struct {
  orc_model *m;
  orc_state *s;
  int layer, group, head_dim, fast, use_ref;
} attn_args;

static void attn_range(void *a_, int h_start, int h_end) {
  attn_args *a = (attn_args *)a_;
  orc_state *s = a->s;
  int hd = a->head_dim;
  int nkv = a->m->hp.n_heads_kv;
  /* scale := float32(1.0 / math.Sqrt(float64(headDim))) */
  float scale = (float)(1.0 / sqrt((double)hd));
  for (int h = h_start; h < h_end; h++) {
    int kvh = h / a->group;
    if (kvh >= nkv) kvh = nkv - 1;
    const float *qh = s->q + (size_t)h * hd;
    float *scores = s->scores + (size_t)h * s->ctx;
    float max_score = -1e30f;
    for (int t = 0; t <= s->pos; t++) {
      const float *kt = s->K + kv_idx(s, a->layer, t, kvh);
      float d = a->use_ref ? g_ref_dot(qh, kt, hd) : dot_pure(qh, kt, hd);
      float sc = d * scale;
      scores[t] = sc;
      if (sc > max_score) max_score = sc;
    }
    float sum_exp = 0.0f;
    for (int t = 0; t <= s->pos; t++) {
      float e = a->fast ? orc_fast_exp(scores[t] - max_score)
                        : (float)exp((double)(scores[t] - max_score));
      scores[t] = e;
      sum_exp += e;
    }
    float inv_sum = 1.0f / sum_exp;
    float *out = s->attn + (size_t)h * hd;
    for (int i = 0; i < hd; i++) out[i] = 0.0f;
    for (int t = 0; t <= s->pos; t++) {
      float wgt = scores[t] * inv_sum;
      const float *vt = s->V + kv_idx(s, a->layer, t, kvh);
      for (int i = 0; i < hd; i++) out[i] += wgt * vt[i];
    }
  }
}

static int forward_layers(orc_model *m, orc_state *s, int32_t token, int fast,
                          int use_ref, char *err, int errlen) {
  const orc_hparams *hp = &m->hp;
  if (s->pos >= s->ctx) {
    snprintf(err, (size_t)errlen, "context length exceeded (%d)", s->ctx);
    return -1;
  }
  if (embed_into(m, token, s->x, err, errlen)) return -1;
  int ne = hp->n_emb, nh = hp->n_heads, nkv = hp->n_heads_kv;
  int hd = ne / nh;
  int rope_dim = hp->rope_dim;
  if (rope_dim > hd) rope_dim = hd;
  int half = rope_dim / 2;
  int group = nh / nkv;
  if (group <= 0) group = 1;
  int kvdim = nkv * hd;

  for (int l = 0; l < hp->n_layers; l++) {
    const orc_layer *L = &m->layers[l];
    orc_rmsnorm(s->xn, s->x, L->attn_norm, ne, hp->rms_eps);
    orc_quantize_q8_0(s->xn, ne, s->q8d, s->q8qs);
    matvec_q8(m, L->wq, s->q8d, s->q8qs, s->q, ne, ne, use_ref);
    matvec_q8(m, L->wk, s->q8d, s->q8qs, s->k, kvdim, ne, use_ref);
    matvec_q8(m, L->wv, s->q8d, s->q8qs, s->v, kvdim, ne, use_ref);
    /* RoPE, infer.go:112-119 (the table has rope.go's half; rotate only the
     * first ropeDim dims of each head) */
    for (int h = 0; h < nh; h++)
      rope_apply(s->q + (size_t)h * hd, s->cosT, s->sinT, half, s->pos);
    for (int h = 0; h < nkv; h++)
      rope_apply(s->k + (size_t)h * hd, s->cosT, s->sinT, half, s->pos);
    /* KV append, infer.go:122-127 */
    for (int h = 0; h < nkv; h++) {
      memcpy(s->K + kv_idx(s, l, s->pos, h), s->k + (size_t)h * hd,
             sizeof(float) * (size_t)hd);
      memcpy(s->V + kv_idx(s, l, s->pos, h), s->v + (size_t)h * hd,
             sizeof(float) * (size_t)hd);
    }
    /* attention, infer.go:130-175 (ParallelFor over heads) */
    attn_args aa = {m, s, l, group, hd, fast, use_ref && g_ref_dot != NULL};
    parallel_for(m->pool, nh, attn_range, &aa);
    /* Wo + residual, infer.go:178-191 */
    orc_quantize_q8_0(s->attn, ne, s->q8d, s->q8qs);
    matvec_q8(m, L->wo, s->q8d, s->q8qs, s->proj, ne, ne, use_ref);
    for (int i = 0; i < ne; i++) s->x[i] += s->proj[i];
    /* FFN, infer.go:194-246 */
    orc_rmsnorm(s->ffn_in, s->x, L->ffn_norm, ne, hp->rms_eps);
    orc_quantize_q8_0(s->ffn_in, ne, s->q8d, s->q8qs);
    matvec_q8(m, L->wup, s->q8d, s->q8qs, s->ffn_up, hp->n_ff, ne, use_ref);
    matvec_q8(m, L->wgate, s->q8d, s->q8qs, s->ffn_gate, hp->n_ff, ne,
              use_ref);
    for (int i = 0; i < hp->n_ff; i++)
      s->ffn_act[i] = orc_silu(s->ffn_gate[i]) * s->ffn_up[i];
    orc_quantize_q8_0(s->ffn_act, hp->n_ff, s->q8d, s->q8qs);
    matvec_q8(m, L->wdown, s->q8d, s->q8qs, s->ffn_down, ne, hp->n_ff,
              use_ref);
    for (int i = 0; i < ne; i++) s->x[i] += s->ffn_down[i];
  }
  return 0;
}

/* ForwardIntoWorkspace (infer.go:21-267).  logits may be NULL (prefill). */
int orc_forward(orc_model *m, orc_state *s, int32_t token, float *logits,
                int use_ref, char *err, int errlen) {
  if (forward_layers(m, s, token, 0, use_ref, err, errlen)) return -1;
  const orc_hparams *hp = &m->hp;
  if (logits) { /* infer.go:250-262 */
    orc_rmsnorm(s->xn, s->x, m->out_norm, hp->n_emb, hp->rms_eps);
    orc_quantize_q8_0(s->xn, hp->n_emb, s->q8d, s->q8qs);
    matvec_q8(m, m->out_proj, s->q8d, s->q8qs, logits, hp->vocab_size,
              hp->n_emb, use_ref);
  }
  s->pos++;
  return 0;
}

/* matVecTopKWS, matvec_topk.go:10-90: one chunk per worker, pure-Go
 * dotQ8_0Row, local replace-min top-K, then merge in chunk order. */
typedef struct {
  const uint8_t *w;
  const float *xd;
  const int8_t *xqs;
  int rows, cols, chunks, k;
  int32_t *loc_ids;
  float *loc_lg;
  int *loc_len;
} topk_args;

static void topk_chunk(void *a_, int c0, int c1) {
  topk_args *a = (topk_args *)a_;
  size_t row_bytes = (size_t)(a->cols / 32) * 34;
  for (int ci = c0; ci < c1; ci++) {
    int start = (int)((long long)ci * a->rows / a->chunks);
    int end = (int)((long long)(ci + 1) * a->rows / a->chunks);
    int32_t *ids = a->loc_ids + (size_t)ci * a->k;
    float *lg = a->loc_lg + (size_t)ci * a->k;
    int len = 0;
    for (int r = start; r < end; r++) {
      float logit = orc_dot_q8_0_row(a->w + (size_t)r * row_bytes, a->xd,
                                     a->xqs, a->cols / 32);
      len = keep_topk_insert(ids, lg, len, a->k, r, logit);
    }
    a->loc_len[ci] = len;
  }
}

/* The goroutines of matvec_topk.go:58-76 run one chunk each; here one pool
 * worker per chunk gives the same partition. */
static void run_chunks(orc_pool *p, int chunks, range_fn fn, void *arg) {
  if (!p || p->workers <= 1 || chunks <= 1) {
    fn(arg, 0, chunks);
    return;
  }
  pthread_mutex_lock(&p->mu);
  p->fn = fn;
  p->arg = arg;
  p->n = chunks;
  p->chunk = (chunks + p->workers - 1) / p->workers;
  p->pending = p->workers;
  p->gen++;
  pthread_cond_broadcast(&p->cv_go);
  while (p->pending > 0) pthread_cond_wait(&p->cv_done, &p->mu);
  pthread_mutex_unlock(&p->mu);
}

/* ForwardTopKIntoWorkspace (infer.go:269-511).  Returns the number of items
 * written (unsorted, in the reference's merge order). */
int orc_forward_topk(orc_model *m, orc_state *s, int32_t token, int topk,
                     int32_t *out_ids, float *out_logits, int use_ref,
                     char *err, int errlen) {
  if (topk <= 0) topk = 40;
  if (forward_layers(m, s, token, 1, use_ref, err, errlen)) return -1;
  const orc_hparams *hp = &m->hp;
  orc_rmsnorm(s->xn, s->x, m->out_norm, hp->n_emb, hp->rms_eps);
  orc_quantize_q8_0(s->xn, hp->n_emb, s->q8d, s->q8qs);
  int workers = m->pool->workers;
  if (workers <= 0) workers = 1;
  int rows = hp->vocab_size;
  int chunks = workers < rows ? workers : rows;
  topk_args a;
  a.w = m->out_proj;
  a.xd = s->q8d;
  a.xqs = s->q8qs;
  a.rows = rows;
  a.cols = hp->n_emb;
  a.chunks = chunks;
  a.k = topk;
  a.loc_ids = (int32_t *)malloc(sizeof(int32_t) * (size_t)chunks * topk);
  a.loc_lg = (float *)malloc(sizeof(float) * (size_t)chunks * topk);
  a.loc_len = (int *)calloc((size_t)chunks, sizeof(int));
  run_chunks(m->pool, chunks, topk_chunk, &a);
  int len = 0;
  for (int ci = 0; ci < chunks; ci++)
    for (int j = 0; j < a.loc_len[ci]; j++)
      len = keep_topk_insert(out_ids, out_logits, len, topk,
                             a.loc_ids[(size_t)ci * topk + j],
                             a.loc_lg[(size_t)ci * topk + j]);
  free(a.loc_ids);
  free(a.loc_lg);
  free(a.loc_len);
  s->pos++;
  return len;
}

/* ------------------------------------------------------------------------ */
/* Sampler (sampling.go:37-143) with the uniform draw supplied by the caller */
/* (Go's math/rand stream is not restated).                                  */
/* ------------------------------------------------------------------------ */

/* SampleTopK, sampling.go:103-143 */
int32_t orc_sample_topk(const int32_t *ids, const float *logits, int n,
                        float temperature, double r01) {
  if (n == 0) return 0;
  float max_logit = logits[0];
  for (int i = 1; i < n; i++)
    if (logits[i] > max_logit) max_logit = logits[i];
  double *exps = (double *)malloc(sizeof(double) * (size_t)n);
  double sum = 0;
  double invT = 1.0 / (double)temperature;
  for (int i = 0; i < n; i++) {
    double v = (double)(logits[i] - max_logit) * invT;
    exps[i] = exp(v);
    sum += exps[i];
  }
  double r = r01 * sum;
  double acc = 0;
  int32_t out = ids[n - 1];
  for (int i = 0; i < n; i++) {
    acc += exps[i];
    if (r <= acc) {
      out = ids[i];
      break;
    }
  }
  free(exps);
  return out;
}

/* Sample, sampling.go:37-99: top-k by insertion over the full logits, then
 * the same softmax draw. */
int32_t orc_sample(const float *logits, int n_vocab, int topk,
                   float temperature, double r01) {
  int k = topk < n_vocab ? topk : n_vocab;
  int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
  float *lg = (float *)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
  int len = 0;
  for (int i = 0; i < n_vocab; i++) {
    if (len < k) {
      ids[len] = i;
      lg[len] = logits[i];
      len++;
      continue;
    }
    int min_idx = 0;
    float min_val = lg[0];
    for (int j = 1; j < len; j++)
      if (lg[j] < min_val) {
        min_val = lg[j];
        min_idx = j;
      }
    if (logits[i] > min_val) {
      ids[min_idx] = i;
      lg[min_idx] = logits[i];
    }
  }
  int32_t out = orc_sample_topk(ids, lg, len, temperature, r01);
  free(ids);
  free(lg);
  return out;
}
