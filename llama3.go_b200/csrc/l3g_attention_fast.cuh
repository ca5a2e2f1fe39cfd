// Attention of the reference's top-K path (included by l3g_kernels.cuh):
// the loop of ForwardTopKIntoWorkspace, internal/llama/infer.go:376-423.
//
// That path weights each position by fastExp(score - max) (infer.go:404,
// 520-525), where max is the head's largest score over ALL positions
// (initialised to -1e30, infer.go:386).  fastExp is Schraudolph's bit trick,
// not an exponential: fastExp(a) * fastExp(b) != fastExp(a + b), so the
// online softmax of k_attention (running maximum, rescale by exp of the
// difference) cannot reproduce it.  Here the maximum is known before any
// weight is formed, as in the reference, in three short kernels:
//   k_attf_scores  grid (kv head, split): every score of the split's
//                  positions for the kv head's `group` query heads, stored
//                  [q head][ctx] (the reference's attentionScores layout),
//                  and the split's maximum per head;
//   k_attf_values  grid (kv head, split): the head's maximum over the
//                  splits, e = fastExp(score - max) per position, the
//                  split's sum of e and sum of e * V;
//   k_attf_merge   one warp per 32 outputs: the splits' sums in split order,
//                  out = sum(e * V) / sum(e), and its act-quant for Wo
//                  (QuantizeQ8_0Into, infer.go:426-427).
// K is read by the first pass and V by the second, so the cache bytes are
// those of k_attention.  Every kernel is a plain grid (no waits between
// CTAs, no bulk copies): it waits only for the previous kernel
// (griddepcontrol.wait) and is as deterministic as the reference's loop.
#pragma once

struct AttfArgs {
  const float* q;   // [local q heads][hd], roped
  KvMap kv;         // the state's KV cache (paged)
  int layer;        // this layer's rows are read
  int ctx, hd, group, splits;  // ctx: the scores buffer's row length
  int n_blocks;     // local q heads * hd / 32 (merge)
  float scale;      // float32(1/sqrt(hd)), infer.go:376
  const int* io;    // io[1] = position of this token
  float* scores;    // [local q heads][ctx]
  float* pmax;      // [kv heads][splits][group]
  float* psum;      // [kv heads][splits][group]
  float* po;        // [kv heads][splits][group][hd]
  float* out;       // [local q heads][hd]
  float* out_d;     // out quantized for the Wo matvec: block scales,
  int8_t* out_q;    //   int8 values
};

// fastExp, infer.go:520-525: bits = uint32(x * float32(12102203)) + 1064866816.
// Go converts float32 to uint32 on amd64 through a truncating int64
// conversion and keeps the low 32 bits; cvt.rzi.s64.f32 truncates the same
// way, so the (wrapping) bits below x ~ -88 match too.
__device__ __forceinline__ float fast_exp_ref(float x) {
  const float prod = __fmul_rn(x, 12102203.0f);
  const unsigned bits = (unsigned)(unsigned long long)(long long)prod + 1064866816u;
  return __uint_as_float(bits);
}

// Positions [t0, t1) of split s of n positions.
__device__ __forceinline__ void attf_range(int n, int splits, int s, int* t0, int* t1) {
  const int chunk = (n + splits - 1) / splits;
  *t0 = min(n, s * chunk);
  *t1 = min(n, *t0 + chunk);
}

constexpr int ATTF_THREADS = NW * 32;
constexpr int ATTF_MAX_HD = 128;

// Dynamic shared memory of the two passes.
struct AttfScoresSmem {
  float qs[MAXG * ATTF_MAX_HD];  // the kv head's query heads
  float wmax[NW][MAXG];          // per-warp maxima
};
struct AttfValuesSmem {
  float hmax[MAXG];                   // the heads' maxima over all splits
  float wsum[NW][MAXG];               // per-warp sums of e
  float wo[NW * MAXG * ATTF_MAX_HD];  // per-warp sums of e * V [warp][h][hd]
};

template <int DPL, typename KT>
__global__ void __launch_bounds__(ATTF_THREADS) k_attf_scores(const __grid_constant__ AttfArgs a) {
  L3G_DYNAMIC_SMEM(smem);
  AttfScoresSmem& sm = *reinterpret_cast<AttfScoresSmem*>(smem);
  float* qs = sm.qs;
  pdl_launch_dependents();
  pdl_wait();  // q, the appended K row and the position come from the QKV kernel
  const int g = blockIdx.x, s = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.hd, G = a.group;
  int t0, t1;
  attf_range(a.io[1] + 1, a.splits, s, &t0, &t1);
  for (int i = threadIdx.x; i < G * hd; i += ATTF_THREADS) qs[i] = __ldcg(a.q + (size_t)g * G * hd + i);
  __syncthreads();
  float mx[MAXG];
#pragma unroll
  for (int h = 0; h < MAXG; ++h) mx[h] = -1e30f;  // maxScore := float32(-1e30)
  for (int t = t0 + warp; t < t1; t += NW) {
    float k[DPL];
    load_row<DPL, KT>(reinterpret_cast<const KT*>(kv_row(a.kv, a.layer, g, t)) + lane * DPL, k);
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
      if (h < G) {  // uniform over the warp
        float d = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) d = fmaf(qs[h * hd + lane * DPL + j], k[j], d);
        d = warp_sum(d);  // identical on every lane
        const float sc = __fmul_rn(d, a.scale);
        if (lane == 0) a.scores[((size_t)g * G + h) * a.ctx + t] = sc;
        mx[h] = fmaxf(mx[h], sc);
      }
    }
  }
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < MAXG; ++h) sm.wmax[warp][h] = mx[h];
  __syncthreads();
  if (threadIdx.x < G) {
    float m = -1e30f;
#pragma unroll
    for (int w = 0; w < NW; ++w) m = fmaxf(m, sm.wmax[w][threadIdx.x]);
    a.pmax[((size_t)g * a.splits + s) * G + threadIdx.x] = m;
  }
}

template <int DPL, typename KT>
__global__ void __launch_bounds__(ATTF_THREADS) k_attf_values(const __grid_constant__ AttfArgs a) {
  L3G_DYNAMIC_SMEM(smem);
  AttfValuesSmem& sm = *reinterpret_cast<AttfValuesSmem*>(smem);
  float* hmax = sm.hmax;
  float* wo = sm.wo;
  pdl_launch_dependents();
  pdl_wait();  // the scores and split maxima of k_attf_scores
  const int g = blockIdx.x, s = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.hd, G = a.group, S = a.splits;
  int t0, t1;
  attf_range(a.io[1] + 1, S, s, &t0, &t1);
  if (threadIdx.x < G) {
    float m = -1e30f;
    for (int s2 = 0; s2 < S; ++s2) m = fmaxf(m, __ldcg(a.pmax + ((size_t)g * S + s2) * G + threadIdx.x));
    hmax[threadIdx.x] = m;
  }
  __syncthreads();
  float o[MAXG][DPL], l[MAXG], mh[MAXG];
#pragma unroll
  for (int h = 0; h < MAXG; ++h) {
    l[h] = 0.0f;
    mh[h] = h < G ? hmax[h] : 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[h][j] = 0.0f;
  }
  const float* sc = a.scores + (size_t)g * G * a.ctx;
  for (int t = t0 + warp; t < t1; t += NW) {
    float v[DPL];
    load_row<DPL, KT>(reinterpret_cast<const KT*>(kv_row(a.kv, a.layer, g, t)) + hd + lane * DPL, v);
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
      if (h < G) {
        const float e = fast_exp_ref(__fsub_rn(__ldcg(sc + (size_t)h * a.ctx + t), mh[h]));
        l[h] = __fadd_rn(l[h], e);
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[h][j] = fmaf(e, v[j], o[h][j]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < MAXG; ++h) {
    if (h < G) {
#pragma unroll
      for (int j = 0; j < DPL; ++j) wo[((size_t)warp * MAXG + h) * hd + lane * DPL + j] = o[h][j];
      if (lane == 0) sm.wsum[warp][h] = l[h];
    }
  }
  __syncthreads();
  const size_t pb = ((size_t)g * S + s) * G;
  for (int idx = threadIdx.x; idx < G * hd; idx += ATTF_THREADS) {
    const int h = idx / hd, d = idx % hd;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) acc = __fadd_rn(acc, wo[((size_t)w * MAXG + h) * hd + d]);
    a.po[(pb + h) * hd + d] = acc;
    if (d == 0) {
      float ls = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w) ls = __fadd_rn(ls, sm.wsum[w][h]);
      a.psum[pb + h] = ls;
    }
  }
}

static __global__ void __launch_bounds__(ATTF_THREADS) k_attf_merge(const __grid_constant__ AttfArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // the splits' sums of k_attf_values
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gb = blockIdx.x * NW + warp;
  if (gb >= a.n_blocks) return;  // whole warps
  const int S = a.splits, G = a.group, hd = a.hd, gh = G * hd;
  const int kvh = gb / (gh / 32), blk = gb % (gh / 32);
  const int h = blk * 32 / hd;  // a 32-output block lies inside one head (hd % 32 == 0)
  float L = 0.0f, O = 0.0f;
  for (int s = 0; s < S; ++s) {
    const size_t pb = ((size_t)kvh * S + s) * G;
    L = __fadd_rn(L, __ldcg(a.psum + pb + h));
    O = __fadd_rn(O, __ldcg(a.po + pb * hd + blk * 32 + lane));
  }
  // invSumExp := float32(1.0) / sumExp; out = sum(e * V) * invSumExp
  const float v = __fmul_rn(O, __frcp_rn(L));
  a.out[(size_t)kvh * gh + blk * 32 + lane] = v;
  quant_block(v, gb, lane, a.out_d, a.out_q);
}
