// Split-K GQA attention of libl3g (included by l3g_kernels.cuh), the
// attention loop of ForwardIntoWorkspace (internal/llama/infer.go:130-175).
//
// The KV cache interleaves K and V per position: [kv head][pos][K hd | V hd].
// Grid (local kv heads, splits).  CTA (g, s) takes a contiguous range of
// positions of kv head g for the `group` query heads sharing it, streams the
// K|V rows of P positions per stage through a shared-memory ring (one ~32 KB
// bulk copy per stage), and keeps an online softmax per warp:
//   - lanes split the head dimension (DPL = hd / 32 values each);
//   - a warp takes nbw positions of a stage in sub-batches of 32 / GP
//     positions (GP = group rounded up to a power of two), computes the
//     partial dots of every (position, head) pair and transpose-reduces them
//     so lane i ends with complete score i (31 shuffles per sub-batch); when
//     a stage holds fewer than 8 sub-batches the warps form two groups that
//     take alternate stages, so every sub-batch is full;
//   - probabilities are broadcast through a warp-private buffer for the V
//     accumulation.
// The per-warp states merge in the CTA.  The CTAs (splits) of one kv head
// then merge in split order (deterministic) either
//   - CL: as one thread-block cluster, each CTA leaving its (m, l, o) in its
//     own shared memory; after a cluster barrier CTA r merges output slice r
//     (one or more Q8_0 blocks) reading the others' partials over
//     distributed shared memory, then a second barrier keeps every CTA's
//     shared memory alive until all reads are done;
//   - otherwise through global partials: every CTA publishes its own, waits
//     until all splits of its kv head have (they are all resident), and
//     merges one slice of the outputs.
#pragma once

struct AttnArgs {
  const float* q;     // [local q heads][hd], roped
  KvMap kv;           // the state's KV cache (paged)
  int layer;          // this layer's rows are read
  int hd, group, n_splits, P, nstages, stage_bytes;
  float scale;        // float32(1/sqrt(hd)), infer.go:130
  const int* io;      // io[1] = position of this token
  float* part_o;      // [kv heads][splits][group][hd]
  float* part_ml;     // [kv heads][splits][group][2]
  unsigned* counters; // [2][kv heads]: arrivals, departures; zero between launches
  float* out;         // [local q heads][hd]
  float* out_d;       // out quantized (QuantizeQ8_0Into) for the Wo matvec:
  int8_t* out_q;      //   [local q heads * hd / 32] scales, int8 values
  Result* res;
  unsigned long long* trace;  // device timeline (nullptr: off)
  int trace_seq;
  unsigned long long wait_ns;  // bound of every wait (WAIT_TIMEOUT_NS or _PEER_NS)
};

struct AttnSmem {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  int abort_flag;
  int issued;
  int producer_done;
  int last;
};
constexpr int AT_HEAD = 512;
static_assert(sizeof(AttnSmem) <= AT_HEAD, "attn smem head");

// Shared memory after the head: per-warp probability buffer [NW][32] and
// head statistics [NW][MAXG][4], then the ring (reused as merge scratch).
constexpr int AT_BUF = (NW * 32 + NW * MAXG * 4) * 4;
__host__ __device__ __forceinline__ int at_ring_offset() { return AT_HEAD + align_up(AT_BUF, 128); }

template <int DPL, typename KT>
__device__ __forceinline__ void load_row(const KT* p, float* v) {
  if constexpr (sizeof(KT) == 4) {
    if constexpr (DPL == 4) {
      const float4 t = *reinterpret_cast<const float4*>(p);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else if constexpr (DPL == 2) {
      const float2 t = *reinterpret_cast<const float2*>(p);
      v[0] = t.x; v[1] = t.y;
    } else {
      v[0] = *reinterpret_cast<const float*>(p);
    }
  } else {
    const __half* h = reinterpret_cast<const __half*>(p);
    if constexpr (DPL == 4) {
      const uint2 raw = *reinterpret_cast<const uint2*>(h);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(h));
      v[0] = a.x; v[1] = a.y;
    }
  }
}

// v[i] on every lane -> lane l returns sum over lanes of v[l].
__device__ __forceinline__ float transpose_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) {
    const bool upper = lane & k;
#pragma unroll
    for (int j = 0; j < k; ++j) {
      const float send = upper ? v[j] : v[j + k];
      const float keep = upper ? v[j + k] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, k);
    }
  }
  return v[0];
}

// Shared-memory merge scratch in the ring after the loop (floats):
// [NW][MAXG][2] per-warp (m, l), [NW][G][hd] per-warp o, then (CL) the CTA's
// combined [MAXG][2] (m, l) and [G][hd] o read by the cluster's other CTAs,
// then the per-head warp weights [NW][MAXG] and (M, L) [MAXG][2].
__host__ __device__ __forceinline__ int at_scratch_floats(int G, int hd) {
  return NW * MAXG * 2 + NW * G * hd + MAXG * 2 + G * hd + NW * MAXG + MAXG * 2;
}

// Merge of one 32-output block of a kv head across its S splits (one warp;
// lane = output).  Split s published its query head h's running max and sum
// at ml[(s * G + h) * 2 + {0, 1}] and its unnormalised outputs at po[s * gh
// + col].  out = (sum_s o_s e_s) / (sum_s l_s e_s), e_s = exp(m_s - max_s
// m_s); the sums run in split order (deterministic).  The loads are issued
// together -- every split's (m, l) pair and, for up to 32 splits at a time,
// this lane's outputs -- so a merge costs one round trip to L2 per 32
// splits instead of one per step of the arithmetic.  wbuf: 32 floats of
// shared memory per 32 splits for the weights e_s.
__device__ __forceinline__ float merge_split_block(const float* ml, const float* po, int S,
                                                   int G, int gh, int h, int col, int lane,
                                                   float* wbuf) {
  constexpr int MB = 32;  // splits loaded per batch
  float ov[MB];
#pragma unroll
  for (int u = 0; u < MB; ++u) ov[u] = u < S ? __ldcg(po + (size_t)u * gh + col) : 0.0f;
  float M = -INFINITY;
  for (int s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, __ldcg(ml + ((size_t)s2 * G + h) * 2));
  M = warp_max(M);
  float L = 0.0f;
  for (int s0 = 0; s0 < S; s0 += 32) {
    const int s2 = s0 + lane;
    float le = 0.0f;
    if (s2 < S) {
      const float2 p = __ldcg(reinterpret_cast<const float2*>(ml + ((size_t)s2 * G + h) * 2));
      const float e = p.x == -INFINITY ? 0.0f : expf(p.x - M);
      wbuf[s2] = e;
      le = p.y * e;
    }
    L += warp_sum(le);
  }
  __syncwarp();
  float O = 0.0f;
#pragma unroll
  for (int u = 0; u < MB; ++u)
    if (u < S) O = fmaf(ov[u], wbuf[u], O);
  for (int s0 = MB; s0 < S; s0 += MB) {
#pragma unroll
    for (int u = 0; u < MB; ++u)
      ov[u] = s0 + u < S ? __ldcg(po + (size_t)(s0 + u) * gh + col) : 0.0f;
#pragma unroll
    for (int u = 0; u < MB; ++u)
      if (s0 + u < S) O = fmaf(ov[u], wbuf[s0 + u], O);
  }
  __syncwarp();
  return __fmul_rn(O, __frcp_rn(L));
}

// One CTA per SM (the registers of one attention CTA leave no room for a
// matvec CTA beside it).  Capping the registers so that an attention CTA
// and a matvec CTA share an SM was measured slower: the early K|V stream
// then competes with the QKV matvec's prologue and weight stream and every
// kernel of the layer slows down.  A merge by the last CTA of each kv head
// to publish (no waiting) was measured slower too: the one CTA's merge of
// all the head's outputs takes longer than the wait plus one slice each.
template <int DPL, typename KT, int GP, bool CL>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attention(const __grid_constant__ AttnArgs a) {
  constexpr int SB = 32 / GP;  // positions per sub-batch
  L3G_DYNAMIC_SMEM(smem);
  AttnSmem* sh = reinterpret_cast<AttnSmem*>(smem);
  float* pbuf_all = reinterpret_cast<float*>(smem + AT_HEAD);
  float* hbuf_all = pbuf_all + NW * 32;
  uint8_t* ring = smem + at_ring_offset();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, split = blockIdx.y, S = a.n_splits;
  const int hd = a.hd, G = a.group, ns = a.nstages, P = a.P;
  const int pos = a.io[1];  // written by the step's host copy, not a kernel
  const int n = pos + 1;
  const int chunk = align_up((n + S - 1) / S, P);
  const int t0 = min(n, split * chunk), t1 = min(n, t0 + chunk);
  const int nst = (t1 - t0 + P - 1) / P;
  const int row = 2 * hd;  // elements per position: K then V
  // Stage groups: when a stage holds fewer than NW sub-batches, the warps
  // split into two groups of NW/2 that take alternate stages, so a warp's
  // share of a stage (nbw positions) still fills whole sub-batches.  Two
  // groups never outrun a ring of >= 2 stages, which keeps every mbarrier
  // wait within one phase of the barrier's state.
  const int wsz = (P / SB >= NW) ? NW : NW / 2;  // warps per stage
  const int ngrp = NW / wsz;
  const int nbw = P / wsz;                        // positions per warp and stage

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], wsz);
    }
    sh->abort_flag = 0;
    sh->issued = 0;
    sh->producer_done = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  trace_mark(a.trace, a.trace_seq, TR_ENTRY);

  if (warp == NW) {
    if (lane == 0) {
      bool waited = false;
      for (int st = 0; st < nst; ++st) {
        const int s = st % ns;
        if (st >= ns &&
            !mbar_wait(&sh->empty[s], ((st / ns) - 1) & 1, &sh->abort_flag, a.res, 4, a.wait_ns))
          break;
        const int ta = t0 + st * P, tb = min(t1, ta + P);
        // past positions are immutable: only the stage holding this step's
        // own K/V (written by the QKV kernel) waits for the previous grid
        if (!waited && tb > pos) {
          pdl_wait();
          waited = true;
        }
        // a stage starts at a multiple of P, which divides KV_PAGE: its
        // rows are contiguous inside one page
        const uint32_t bytes = (uint32_t)((tb - ta) * row * sizeof(KT));
        mbar_arrive_expect_tx(&sh->full[s], bytes);
        bulk_g2s(ring + (size_t)s * a.stage_bytes, kv_row(a.kv, a.layer, kvh, ta), bytes,
                 &sh->full[s]);
        *(volatile int*)&sh->issued = st + 1;
      }
      *(volatile int*)&sh->producer_done = 1;
    }
    if constexpr (CL) {  // the cluster barriers count every thread
      __syncwarp();
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // warm the translations of q and of the merge buffers before the wait
  if (lane == 0) {
    if (warp == 0) touch_page(a.q + (size_t)kvh * G * hd);
    if (warp == 1) touch_page(a.part_o + ((size_t)kvh * S + split) * G * hd);
    if (warp == 2) touch_page(a.part_ml + ((size_t)kvh * S + split) * G * 2);
    if (warp == 3) touch_page(a.counters + kvh);
    if (warp == 4) touch_page(a.out + (size_t)kvh * G * hd);
  }
  pdl_wait();  // q comes from the previous kernel
  trace_mark(a.trace, a.trace_seq, TR_WAITED);
  float q[GP][DPL];
#pragma unroll
  for (int h = 0; h < GP; ++h)
#pragma unroll
    for (int j = 0; j < DPL; ++j)
      q[h][j] = h < G ? a.q[((size_t)kvh * G + h) * hd + lane * DPL + j] : 0.0f;
  float m[GP], l[GP], o[GP][DPL];
#pragma unroll
  for (int h = 0; h < GP; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[h][j] = 0.0f;
  }
  float* pbuf = pbuf_all + warp * 32;
  float* hbuf = hbuf_all + warp * MAXG * 4;
  const int my_h = lane % GP;      // after the transpose-reduce: lane -> (pos, head)
  const int my_p = lane / GP;
  const int grp = warp / wsz, wj = warp % wsz;

  for (int st = grp; st < nst; st += ngrp) {
    const int s = st % ns;
    // warp-uniform: a stage is either consumed by the whole warp or, after
    // an abort, not at all (and then not released: no copy can be issued
    // into a slot whose previous copy may still be in flight)
    const bool ok = __all_sync(0xffffffffu,
                               mbar_wait(&sh->full[s], (st / ns) & 1, &sh->abort_flag, a.res, 5, a.wait_ns));
    if (!ok) break;
    {
      const int cnt = min(t1, t0 + st * P + P) - (t0 + st * P);
      const KT* Ks = reinterpret_cast<const KT*>(ring + (size_t)s * a.stage_bytes);
      const KT* Vs = Ks + hd;
      for (int sb = 0; sb < nbw; sb += SB) {
        const int p0 = wj * nbw + sb;        // first position of the sub-batch
        const int np = min(SB, nbw - sb);    // positions of this warp in it
        // partial dots of (position, head), then the transpose-reduce
        float v[32];
#pragma unroll
        for (int p = 0; p < SB; ++p) {
          float kv[DPL];
          if (p < np && p0 + p < cnt) {
            load_row<DPL, KT>(Ks + (size_t)(p0 + p) * row + lane * DPL, kv);
          } else {
#pragma unroll
            for (int j = 0; j < DPL; ++j) kv[j] = 0.0f;
          }
#pragma unroll
          for (int h = 0; h < GP; ++h) {
            float d = 0.0f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) d = fmaf(q[h][j], kv[j], d);
            v[p * GP + h] = d;
          }
        }
        const float dot = transpose_reduce32(v, lane);
        const bool valid = my_p < np && p0 + my_p < cnt && my_h < G;
        const float sc = valid ? dot * a.scale : -INFINITY;
        // per-head maximum and sum over the sub-batch's positions
        float mb = sc;
#pragma unroll
        for (int off = GP; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        float mo = -INFINITY;
#pragma unroll
        for (int h = 0; h < GP; ++h)
          if (h == my_h) mo = m[h];
        const float mn = fmaxf(mo, mb);
        const float pe = valid ? expf(sc - mn) : 0.0f;
        const float corr = mn == -INFINITY ? 1.0f : expf(mo - mn);
        float lb = pe;
#pragma unroll
        for (int off = GP; off < 32; off <<= 1) lb += __shfl_xor_sync(0xffffffffu, lb, off);
        pbuf[lane] = pe;
        if (lane < GP) {
          hbuf[lane * 4 + 0] = mn;
          hbuf[lane * 4 + 1] = corr;
          hbuf[lane * 4 + 2] = lb;
        }
        __syncwarp();
#pragma unroll
        for (int h = 0; h < GP; ++h) {
          const float c = hbuf[h * 4 + 1];
          m[h] = hbuf[h * 4 + 0];
          l[h] = fmaf(l[h], c, hbuf[h * 4 + 2]);
#pragma unroll
          for (int j = 0; j < DPL; ++j) o[h][j] *= c;
        }
        for (int p = 0; p < np && p0 + p < cnt; ++p) {
          float vv[DPL];
          load_row<DPL, KT>(Vs + (size_t)(p0 + p) * row + lane * DPL, vv);
          float w[GP];
          if constexpr (GP % 4 == 0) {
#pragma unroll
            for (int k = 0; k < GP / 4; ++k) {
              const float4 t = reinterpret_cast<const float4*>(pbuf + p * GP)[k];
              w[4 * k] = t.x; w[4 * k + 1] = t.y; w[4 * k + 2] = t.z; w[4 * k + 3] = t.w;
            }
          } else {
#pragma unroll
            for (int h = 0; h < GP; ++h) w[h] = pbuf[p * GP + h];
          }
#pragma unroll
          for (int h = 0; h < GP; ++h) {
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[h][j] = fmaf(w[h], vv[j], o[h][j]);
          }
        }
        __syncwarp();
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[s]);
  }

  trace_mark(a.trace, a.trace_seq, TR_LOOP);
  // After an abort: wait (bounded) until the producer has stopped issuing,
  // then for the last copy issued to each ring slot (earlier copies to a
  // slot were consumed before it was refilled).  Then the ring is free to
  // reuse as merge scratch.
  consumer_sync();
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const uint64_t t_start = gtime();
    while (!*(volatile int*)&sh->producer_done && gtime() - t_start < 100000000ull) {
    }
    const int issued = *(volatile int*)&sh->issued;
    for (int s2 = 0; s2 < ns && s2 < issued; ++s2) {
      const int t = s2 + ((issued - 1 - s2) / ns) * ns;
      int dummy = 0;
      mbar_wait(&sh->full[s2], (t / ns) & 1, &dummy, a.res, 6, 100000000ull);
    }
  }
  consumer_sync();
  float* sm_ml = reinterpret_cast<float*>(ring);  // [NW][G][2], then [S][G][2]
  float* sm_o = sm_ml + NW * MAXG * 2;            // [NW][G][hd]
#pragma unroll
  for (int h = 0; h < GP; ++h) {
    if (h < G) {
      if (lane == 0) {
        sm_ml[(warp * MAXG + h) * 2] = m[h];
        sm_ml[(warp * MAXG + h) * 2 + 1] = l[h];
      }
#pragma unroll
      for (int j = 0; j < DPL; ++j)
        sm_o[((size_t)warp * G + h) * hd + lane * DPL + j] = o[h][j];
    }
  }
  consumer_sync();
  float* cta_ml = sm_o + NW * G * hd;  // CL: this CTA's combined state
  float* cta_o = cta_ml + MAXG * 2;
  float* sm_e = cta_o + G * hd;        // [NW][MAXG] the warps' weights per query head
  float* sm_hl = sm_e + NW * MAXG;     // [MAXG][2] per query head: M, L
  // per query head (one thread each): M = max_w m_w, e_w = exp(m_w - M),
  // L = sum_w l_w e_w in warp order; every output of the head then only
  // weighs the warps' partial outputs by e_w
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_ml[(w * MAXG + h) * 2]);
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = sm_ml[(w * MAXG + h) * 2];
      const float e = M == -INFINITY || mw == -INFINITY ? 0.0f : expf(mw - M);
      L = fmaf(sm_ml[(w * MAXG + h) * 2 + 1], e, L);
      sm_e[w * MAXG + h] = e;
    }
    sm_hl[h * 2] = M;
    sm_hl[h * 2 + 1] = L;
  }
  consumer_sync();
  const size_t pbase = ((size_t)kvh * S + split) * G;
  for (int idx = threadIdx.x; idx < G * hd; idx += NW * 32) {
    const int h = idx / hd, d = idx % hd;
    // all NW warps' values loaded up front (independent), then combined
    float ow[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) ow[w] = sm_o[((size_t)w * G + h) * hd + d];
    const float M = sm_hl[h * 2], L = sm_hl[h * 2 + 1];
    float O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) O = fmaf(ow[w], sm_e[w * MAXG + h], O);
    }
    if constexpr (CL) {
      cta_o[idx] = O;
      if (d == 0) {
        cta_ml[h * 2] = M;
        cta_ml[h * 2 + 1] = L;
      }
    } else {
      a.part_o[(pbase + h) * hd + d] = O;
      if (d == 0) {
        a.part_ml[(pbase + h) * 2] = M;
        a.part_ml[(pbase + h) * 2 + 1] = L;
      }
    }
  }
  if constexpr (CL) {
    cluster_sync_all();
    trace_mark(a.trace, a.trace_seq, 5);  // partials visible to the cluster
    // merge slice `rank` of the G*hd outputs: whole warps, whole blocks
    const int gh = G * hd;
    const uint32_t rank = cluster_ctarank();
    const int chunk = align_up((gh + S - 1) / S, 32);
    for (int j = threadIdx.x; j < chunk; j += NW * 32) {
      const int idx = (int)rank * chunk + j;
      if (idx >= gh) break;  // uniform per warp
      const int h = idx / hd;
      float ms[16], ls[16], os[16];
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) {
        if (s2 < S) {
          ms[s2] = ld_cluster_f32(cta_ml + h * 2, s2);
          ls[s2] = ld_cluster_f32(cta_ml + h * 2 + 1, s2);
          os[s2] = ld_cluster_f32(cta_o + idx, s2);
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2)
        if (s2 < S) M = fmaxf(M, ms[s2]);
      float L = 0.0f, O = 0.0f;
#pragma unroll
      for (int s2 = 0; s2 < 16; ++s2) {
        if (s2 < S) {
          const float e = ms[s2] == -INFINITY ? 0.0f : expf(ms[s2] - M);
          L = fmaf(ls[s2], e, L);
          O = fmaf(os[s2], e, O);
        }
      }
      const float v = __fmul_rn(O, __frcp_rn(L));
      a.out[(size_t)kvh * gh + idx] = v;
      quant_block(v, (kvh * gh + idx) >> 5, lane, a.out_d, a.out_q);
    }
    trace_mark(a.trace, a.trace_seq, 7);  // merged
    cluster_sync_all();  // the others' reads of this CTA's shared memory are done
    trace_mark(a.trace, a.trace_seq, TR_EXIT);
    return;
  }
  // Publish this split's partial, then wait (bounded) until every split of
  // this kv head has published: the grid has at most one CTA per SM, so all
  // of them are resident.  Then each CTA merges its own slice of the G*hd
  // outputs (whole Q8_0 blocks), reading every split's (m, l) and that
  // slice of their partial outputs: one small gather per CTA instead of one
  // CTA gathering everything.  counters[kvh] counts arrivals,
  // counters[gridDim.x + kvh] departures; the last to depart resets both.
  consumer_sync();
  unsigned* arrived = a.counters + kvh;
  unsigned* departed = a.counters + gridDim.x + kvh;
  if (threadIdx.x == 0) {
    atom_add_acq_rel_gpu(arrived, 1u);
    const uint64_t t0 = gtime();
    while (ld_acquire_gpu_u32(arrived) < (unsigned)S) {
      if (gtime() - t0 > a.wait_ns) {
        report(a.res, ERR_TIMEOUT, 9);
        break;
      }
    }
  }
  consumer_sync();
  trace_mark(a.trace, a.trace_seq, 5);  // every split published
  const int gh = G * hd;
  const int slice = align_up((gh + S - 1) / S, 32);  // outputs merged per CTA
  const int b0 = min(gh, split * slice) / 32, b1 = min(gh, (split + 1) * slice) / 32;
  float* wbuf = reinterpret_cast<float*>(ring) + warp * align_up(S, 32);  // e_s per warp
  const float* ml = a.part_ml + (size_t)kvh * S * G * 2;
  const float* po = a.part_o + (size_t)kvh * S * gh;
  for (int blk = b0 + warp; blk < b1; blk += NW) {  // one warp per block of 32 outputs
    const int h = blk * 32 / hd;
    const float v = merge_split_block(ml, po, S, G, gh, h, blk * 32 + lane, lane, wbuf);
    a.out[(size_t)kvh * gh + blk * 32 + lane] = v;
    quant_block(v, kvh * gh / 32 + blk, lane, a.out_d, a.out_q);
  }
  trace_mark(a.trace, a.trace_seq, 7);  // slice merged
  consumer_sync();
  if (threadIdx.x == 0 && atom_add_acq_rel_gpu(departed, 1u) == (unsigned)S - 1) {
    *arrived = 0u;
    *departed = 0u;
  }
  trace_mark(a.trace, a.trace_seq, TR_EXIT);
}
