// Batched decode kernels (included by l3g_kernels.cuh after l3g_prefill.cuh).
//
// One step advances n independent sequences (each an l3g_state: its own KV
// cache, context length and position) by one token: per sequence exactly
// ForwardTopKIntoWorkspace (internal/llama/infer.go:269-511, here with the
// exact exp of the full path, :130-175) followed by Sampler.SampleTopK
// (sampling.go:103-143).  The projections run as batched Q8_0 products over
// the n tokens (k_gemm_q8) and the row-wise kernels of batched prefill; the
// kernels here are the per-sequence parts: KV append at each sequence's
// position, decode attention over each sequence's own cache, and top-K plus
// sampling per sequence.
#pragma once

// Per-sequence inputs of a step (host-filled, copied once per step).
struct SeqInfo {
  uint8_t* kv_pool;        // the sequence's KV cache: its pool (page 0) ...
  const int* kv_pages;     // ... and its page table
  const float* rope_cos;   // its RoPE tables [ctx][rope_half]
  const float* rope_sin;
  int kv_pps;              // its pages per (layer, kv head)
  int ctx;                 // its context length
  int pos;                 // position this step writes
  int token;               // token this step ingests
  uint64_t seed;           // sampler seed
  float temperature;       // sampler temperature (> 0)
  int pad;
};
static_assert(sizeof(SeqInfo) == 64, "SeqInfo layout");
// The KV map of a sequence (hkv local kv heads, rows of row_bytes).
__device__ __forceinline__ KvMap seq_kv(const SeqInfo& sq, int hkv, int row_bytes) {
  KvMap m;
  m.pool = sq.kv_pool;
  m.pages = sq.kv_pages;
  m.pps = sq.kv_pps;
  m.hkv = hkv;
  m.row_bytes = row_bytes;
  m.pad = 0;
  return m;
}

// x[b] = embedding row of seqs[b].token (infer.go:513-518).  grid (ceil(cols/256), n).
static __global__ void k_bd_embed(const uint8_t* emb, int vocab, int cols, const SeqInfo* seqs,
                           float* X, Result* res) {
  const int b = blockIdx.y;
  const int token = seqs[b].token;
  if (token < 0 || token >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(res, ERR_TOKEN, token);
    return;
  }
  const uint8_t* row = emb + (size_t)token * (cols / 32) * 34;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= cols) return;
  const uint8_t* blk = row + (size_t)(i >> 5) * 34;
  const unsigned short bits = (unsigned short)(blk[0] | (blk[1] << 8));
  const float d = __half2float(__ushort_as_half(bits));
  X[(size_t)b * cols + i] = __fmul_rn(d, (float)(int8_t)blk[2 + (i & 31)]);
}

// RoPE + KV append of row b at seqs[b].pos into layer `layer` of seqs[b]'s
// cache (as k_pf_qkv_rope, with a cache and position per row).
static __global__ void k_bd_qkv_rope(const float* QKV, int n, const SeqInfo* seqs, int layer, int nq,
                              int nkv, int hd, int rope_half, float* Q, int kv_f16) {
  const int rows = nq + 2 * nkv;
  const int half_rows = rows >> 1;
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (long long)n * half_rows) return;
  const int b = (int)(e / half_rows);
  const int row = (int)(e % half_rows) * 2;
  const SeqInfo& sq = seqs[b];
  const int pos = sq.pos;
  const float2 xv = *reinterpret_cast<const float2*>(QKV + (size_t)b * rows + row);
  float x0 = xv.x, x1 = xv.y;
  const bool is_q = row < nq;
  const bool is_k = !is_q && row < nq + nkv;
  if (is_q || is_k) {
    const int d = (is_q ? row : row - nq) % hd;
    const int i = d >> 1;
    if (i < rope_half) {
      const float c = sq.rope_cos[(size_t)pos * rope_half + i];
      const float s = sq.rope_sin[(size_t)pos * rope_half + i];
      const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
      x0 = y0;
      x1 = y1;
    }
  }
  if (is_q) {
    *reinterpret_cast<float2*>(Q + (size_t)b * nq + row) = make_float2(x0, x1);
  } else {
    const int r2 = is_k ? row - nq : row - nq - nkv;
    const int kvh = r2 / hd, d = r2 % hd;
    uint8_t* kvl = kv_row(seq_kv(sq, nkv / hd, 2 * hd * (kv_f16 ? 2 : 4)), layer, kvh, pos);
    const size_t off = (is_k ? 0 : hd) + d;
    if (kv_f16)
      *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(kvl) + off) = __floats2half2_rn(x0, x1);
    else
      *reinterpret_cast<float2*>(reinterpret_cast<float*>(kvl) + off) = make_float2(x0, x1);
  }
}

// Split-K decode attention (infer.go:130-175) of every sequence: CTA (split,
// kv head, sequence) covers positions [split * split_len, ...) up to the
// sequence's own position (split_len a multiple of BD_SPLIT, chosen per step
// by the host so that the grid holds a few waves of CTAs).  A producer warp
// streams the split's cache rows (K | V of 32 positions, contiguous in the
// cache) into a ring of BD_STAGES shared-memory stages with 1-D bulk copies.
// Compute warp w takes positions 4w..4w+3 of every 32-position tile: the
// partial dot products of its (position, query row) pairs (lane = dims
// lane * DPL..; 8 row slots per position) are reduced together by one
// transposed reduction (31 shuffles for 32 slots), then each lane holds
// one pair's score and the online softmax per query row (max, sum,
// weighted V) runs on those.  The 8 warps merge
// in shared memory and the CTA writes one partial (max, sum, o[HD]) per
// query head, merged across splits by k_bd_merge.  Every wait is bounded; after an abort the CTA drains its
// copies and writes nothing.
constexpr int BD_SPLIT = 256;  // split lengths are multiples of this
constexpr int BD_TILE = 32;    // positions per ring stage
constexpr int BD_STAGES = 3;
constexpr int BD_THREADS = 288;  // 8 compute warps + 1 producer warp
struct BdSmem {
  uint64_t full[BD_STAGES];
  uint64_t empty[BD_STAGES];
  int abort_flag, issued, producer_done;
  float m[8][MAXG], l[8][MAXG];
};
__host__ __device__ constexpr int bd_stage_bytes(int hd, int es) { return BD_TILE * 2 * hd * es; }
// the merge buffer (8 warps x GP rows x hd floats) reuses the ring; after
// it, each compute warp's sub-batch weights [32] and head statistics
// [MAXG][4]
constexpr int BD_WBUF = (8 * 32 + 8 * MAXG * 4) * 4;
__host__ __device__ constexpr int bd_smem_bytes(int hd, int es, int gp) {
  return 1024 + (BD_STAGES * bd_stage_bytes(hd, es) > 8 * gp * hd * 4
                     ? BD_STAGES * bd_stage_bytes(hd, es)
                     : 8 * gp * hd * 4) + BD_WBUF;
}
// GP: the group size rounded up to 1, 2, 4 or 8 (register arrays per row)
template <int HD, int GP, typename KT>
__global__ void __launch_bounds__(BD_THREADS) k_bd_attention(
    const float* Q, const SeqInfo* seqs, int layer, int group, int nq_heads, float scale,
    float* part_o, float* part_ml, int max_splits, int split_len, Result* res,
    unsigned long long wait_ns) {
  constexpr int DPL = HD / 32;
  constexpr int SB = bd_stage_bytes(HD, (int)sizeof(KT));
  static_assert(sizeof(BdSmem) <= 1024, "smem head");
  L3G_DYNAMIC_SMEM(bd_smem);
  BdSmem* sh = reinterpret_cast<BdSmem*>(bd_smem);
  uint8_t* ring = bd_smem + 1024;
  float(*sm_o)[GP][HD] = reinterpret_cast<float(*)[GP][HD]>(ring);  // after the ring drains
  // sub-batches: every warp takes SBP = 4 positions of every tile, and their
  // (position, query row) scores, 4 x 8 slots (rows beyond the group empty),
  // are reduced together; all 8 warps share each tile, so a stage is
  // consumed by one set of warps at a time and no wait can run two phases
  // ahead of its barrier
  constexpr int RS = 8;                 // row slots of the reduction
  constexpr int SBP = 32 / RS;
  static_assert(GP <= RS && SBP * 8 == BD_TILE, "sub-batch layout");
  float* wbuf = reinterpret_cast<float*>(
      ring + (BD_STAGES * SB > 8 * GP * HD * 4 ? BD_STAGES * SB : 8 * GP * HD * 4));
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const SeqInfo& sq = seqs[b];
  const int p0 = split * split_len;
  const int p1 = min(sq.pos + 1, p0 + split_len);
  const int ntiles = p1 > p0 ? (p1 - p0 + BD_TILE - 1) / BD_TILE : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < BD_STAGES; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 8);
    }
    sh->abort_flag = 0;
    sh->issued = 0;
    sh->producer_done = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const KvMap kvm = seq_kv(sq, (int)gridDim.y, 2 * HD * (int)sizeof(KT));
  float q[GP][DPL], o[GP][DPL], m[GP], l[GP];  // compute warps' online softmax
  if (warp == 8) {  // producer
    if (lane == 0) {
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % BD_STAGES;
        if (t >= BD_STAGES &&
            !mbar_wait(&sh->empty[s], ((t / BD_STAGES) - 1) & 1, &sh->abort_flag, res, 30, wait_ns))
          break;
        const int q0 = p0 + t * BD_TILE;
        const int np = min(BD_TILE, p1 - q0);
        const uint32_t bytes = (uint32_t)(np * 2 * HD * sizeof(KT));
        mbar_arrive_expect_tx(&sh->full[s], bytes);
        // q0 is a multiple of BD_TILE, which divides KV_PAGE: one page
        bulk_g2s(ring + (size_t)s * SB, kv_row(kvm, layer, kvh, q0), bytes, &sh->full[s]);
        *(volatile int*)&sh->issued = t + 1;
      }
      *(volatile int*)&sh->producer_done = 1;
    }
  } else {
    // lane = dims lane * DPL .. + DPL - 1 (K, V and q rows alike)
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.0f;
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        o[g][j] = 0.0f;
        q[g][j] = g < group ? Q[(size_t)b * nq_heads * HD + (size_t)(kvh * group + g) * HD +
                                lane * DPL + j]
                            : 0.0f;
      }
    }
    float* pbuf = wbuf + warp * 32;
    float* hbuf = wbuf + 8 * 32 + warp * MAXG * 4;
    const int my_h = lane % RS, my_p = lane / RS;  // after the transposed reduction
    for (int t = 0; t < ntiles; ++t) {
      const int s = t % BD_STAGES;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&sh->full[s], (t / BD_STAGES) & 1,
                                                        &sh->abort_flag, res, 31, wait_ns));
      if (!ok) break;
      const KT* tile = reinterpret_cast<const KT*>(ring + (size_t)s * SB);
      const int cnt = min(BD_TILE, p1 - (p0 + t * BD_TILE));  // positions in this tile
      const int pb = warp * SBP;                               // the warp's first position
      // partial dots of (position, row), then one transposed reduction
      float v[32];
#pragma unroll
      for (int p = 0; p < SBP; ++p) {
        float kf[DPL];
        if (pb + p < cnt) {
          load_row<DPL, KT>(tile + (size_t)(pb + p) * 2 * HD + lane * DPL, kf);
        } else {
#pragma unroll
          for (int j = 0; j < DPL; ++j) kf[j] = 0.0f;
        }
#pragma unroll
        for (int g = 0; g < RS; ++g) {
          float d = 0.0f;
          if (g < GP) {
#pragma unroll
            for (int j = 0; j < DPL; ++j) d = fmaf(q[g][j], kf[j], d);
          }
          v[p * RS + g] = d;
        }
      }
      const float dot = transpose_reduce32(v, lane);
      const bool valid = pb + my_p < cnt && my_h < group;
      const float sc = valid ? __fmul_rn(dot, scale) : -INFINITY;
      // per-row maximum and sum over the sub-batch's positions
      float mb = sc;
#pragma unroll
      for (int off = RS; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      float mo = -INFINITY;
#pragma unroll
      for (int g = 0; g < GP; ++g)
        if (g == my_h) mo = m[g];
      const float mn = fmaxf(mo, mb);
      const float pe = valid ? expf(sc - mn) : 0.0f;
      const float corr = mn == -INFINITY ? 1.0f : expf(mo - mn);
      float lb = pe;
#pragma unroll
      for (int off = RS; off < 32; off <<= 1) lb += __shfl_xor_sync(0xffffffffu, lb, off);
      pbuf[lane] = pe;
      if (lane < GP) {
        hbuf[lane * 4 + 0] = mn;
        hbuf[lane * 4 + 1] = corr;
        hbuf[lane * 4 + 2] = lb;
      }
      __syncwarp();
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        const float c = hbuf[g * 4 + 1];
        m[g] = hbuf[g * 4 + 0];
        l[g] = fmaf(l[g], c, hbuf[g * 4 + 2]);
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[g][j] *= c;
      }
      for (int p = 0; p < SBP && pb + p < cnt; ++p) {
        float vf[DPL];
        load_row<DPL, KT>(tile + (size_t)(pb + p) * 2 * HD + HD + lane * DPL, vf);
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          const float w = pbuf[p * RS + g];
#pragma unroll
          for (int j = 0; j < DPL; ++j) o[g][j] = fmaf(w, vf[j], o[g][j]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[s]);
    }
  }
  // after an abort: the producer has stopped, then the last copy issued to
  // each stage has landed (earlier ones were consumed before the refill)
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const uint64_t t_start = gtime();
    while (!*(volatile int*)&sh->producer_done && gtime() - t_start < 100000000ull) {
    }
    const int issued = *(volatile int*)&sh->issued;
    for (int s2 = 0; s2 < BD_STAGES && s2 < issued; ++s2) {
      const int t = s2 + ((issued - 1 - s2) / BD_STAGES) * BD_STAGES;
      int dummy = 0;
      mbar_wait(&sh->full[s2], (t / BD_STAGES) & 1, &dummy, res, 32, 100000000ull);
    }
  }
  __syncthreads();  // every copy consumed (or drained): the ring is free
  if (*(volatile int*)&sh->abort_flag) return;
  if (warp < 8) {
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      if (g >= group) break;
      if (lane == 0) {
        sh->m[warp][g] = m[g];
        sh->l[warp][g] = l[g];
      }
#pragma unroll
      for (int j = 0; j < DPL; ++j) sm_o[warp][g][lane * DPL + j] = o[g][j];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < group * HD; e += BD_THREADS) {
    const int g = e / HD, d = e % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, sh->m[w][g]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float f = sh->m[w][g] == -INFINITY ? 0.0f : expf(sh->m[w][g] - M);
        L = fmaf(sh->l[w][g], f, L);
        O = fmaf(sm_o[w][g][d], f, O);
      }
    }
    const size_t slot = ((size_t)b * nq_heads + kvh * group + g) * max_splits + split;
    part_o[slot * HD + d] = O;
    if (d == 0) {
      part_ml[slot * 2] = M;
      part_ml[slot * 2 + 1] = L;
    }
  }
}

// out[b][head] = sum over splits of o_s * exp(m_s - M) / sum of l_s * exp(m_s - M).
// grid (query heads, n), HD threads.
static __global__ void k_bd_merge(const float* part_o, const float* part_ml, const SeqInfo* seqs,
                           int nq_heads, int hd, int max_splits, int split_len, float* out) {
  const int head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  if (d >= hd) return;
  const int ns = (seqs[b].pos + 1 + split_len - 1) / split_len;
  const size_t slot0 = ((size_t)b * nq_heads + head) * max_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, part_ml[(slot0 + s) * 2]);
  float L = 0.0f, O = 0.0f;
  for (int s = 0; s < ns; ++s) {
    const float ms = part_ml[(slot0 + s) * 2];
    const float f = ms == -INFINITY ? 0.0f : expf(ms - M);
    L = fmaf(part_ml[(slot0 + s) * 2 + 1], f, L);
    O = fmaf(part_o[(slot0 + s) * hd + d], f, O);
  }
  out[(size_t)b * nq_heads * hd + (size_t)head * hd + d] = O / L;
}

// Top-K of each sequence's logits (keys as k_topk_partial: ordered float
// bits, lower id first on ties).  The logits of rank r's vocabulary shard
// for sequence b sit at L[(r * n + b) * v_l + v] (the allgather layout; one
// rank: r = 0), global id r * v_l + v; ids at or past vocab are padding.
// Phase 1: grid (chunks of TOPK_CHUNK ids, n).
static __global__ void k_bd_topk_partial(const float* L, int n, int v_l, int vocab, int k,
                                  uint64_t* part) {
  __shared__ uint64_t keys[TOPK_CHUNK];
  const int b = blockIdx.y, nchunks = gridDim.x;
  const int base = blockIdx.x * TOPK_CHUNK;
  for (int i = threadIdx.x; i < TOPK_CHUNK; i += blockDim.x) {
    const int id = base + i;
    uint64_t key = 0ull;
    if (id < vocab) {
      const int r = id / v_l, v = id % v_l;
      key = topk_key(L[((size_t)r * n + b) * v_l + v], id);
    }
    keys[i] = key;
  }
  __syncthreads();
  bitonic_desc(keys, TOPK_CHUNK);
  for (int i = threadIdx.x; i < k; i += blockDim.x)
    part[((size_t)b * nchunks + blockIdx.x) * k + i] = keys[i];
}
// Phase 2: grid n; cap (a power of two >= count) keys of dynamic shared memory.
static __global__ void k_bd_topk_final(const uint64_t* part, int count, int cap, int k, int* ids,
                                float* logits) {
  L3G_DYNAMIC_SMEM(keys3_raw);
  uint64_t* keys3 = reinterpret_cast<uint64_t*>(keys3_raw);
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < cap; i += blockDim.x)
    keys3[i] = i < count ? part[(size_t)b * count + i] : 0ull;
  __syncthreads();
  bitonic_desc(keys3, cap);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    ids[(size_t)b * k + i] = key_index(keys3[i]);
    logits[(size_t)b * k + i] = key_value(keys3[i]);
  }
}

// SampleTopK (sampling.go:103-143) per sequence, as k_sample: float64
// softmax with 1/T over the items in order, r = uniform * sum from
// Philox4x32-10 keyed by the sequence's seed, counted by its position, then
// the cumulative pick.  grid n, one warp.
static __global__ void k_bd_sample(const int* ids, const float* logits, int k, const SeqInfo* seqs,
                            Result* out) {
  __shared__ double e[MAX_TOPK];
  const int b = blockIdx.x, lane = threadIdx.x;
  const int* id = ids + (size_t)b * k;
  const float* lg = logits + (size_t)b * k;
  float mx = lg[0];
  for (int i = 1; i < k; ++i) mx = fmaxf(mx, lg[i]);
  const double invT = 1.0 / (double)seqs[b].temperature;
  for (int i = lane; i < k; i += 32) e[i] = exp((double)(lg[i] - mx) * invT);
  __syncwarp();
  if (lane != 0) return;
  double sum = 0.0;
  for (int i = 0; i < k; ++i) sum += e[i];
  const uint64_t ctr = (uint64_t)seqs[b].pos;
  uint32_t c[4] = {(uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u};
  philox4x32_10(c, (uint32_t)seqs[b].seed, (uint32_t)(seqs[b].seed >> 32));
  const uint64_t x = ((uint64_t)c[0] << 32) | c[1];
  const double r = (double)(x >> 11) * 0x1.0p-53 * sum;
  double acc = 0.0;
  int pick = k - 1;
  for (int i = 0; i < k; ++i) {
    acc += e[i];
    if (r <= acc) {
      pick = i;
      break;
    }
  }
  out[b].token = id[pick];
  out[b].logit = lg[pick];
  out[b].err = 0;
  out[b].where = 0;
}
