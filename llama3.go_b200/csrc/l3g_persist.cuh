// Persistent decode-step kernel of libl3g (included by l3g_kernels.cuh):
// every layer of one token (ForwardIntoWorkspace, internal/llama/infer.go:
// 56-246) in one launch of one CTA per SM, the phases of a layer separated
// by grid barriers (schedule and phase list: l3g_persist_plan.h).
//
// Why: the per-kernel step (one launch per matvec / attention / quantize)
// pays, per launch, the wake-up of a dependent launch, a pipeline ramp and a
// tail, ~8-9 us of a ~74 us layer on one GPU and most of a layer under
// tensor parallelism.  Here one producer warp per CTA streams every tile the
// CTA consumes through one ring, across phase boundaries, so the weight
// stream does not stop while the consumers wait at a barrier, and a barrier
// costs one round trip through L2 instead of a launch.
//
// Arithmetic is that of the per-kernel step with four rows per warp: the
// same Q8_0 block products and fp32 sums in the same order (matvec_q8_c,
// simd.c:33-110), the same rmsNorm and act-quant (math.go:5-14,
// q8_0.go:22-79), RoPE and KV append (rope.go:39-52, infer.go:122-127), the
// same split-K attention and split merge (infer.go:130-175) and SwiGLU
// (infer.go:228-230): for the same splits its results are bit-identical.
//
// Data written by one CTA and read by another inside the launch is read
// with ld.global.cg (L2) after a grid barrier (release fence + atomic
// arrival, acquire spin); the KV rows appended in the QKV phase are read by
// other CTAs' bulk copies (the async proxy), so their writers and the
// copying producer both issue fence.proxy.async.global around the barrier.
// Every wait is bounded; a failed wait sets the step's abort word, which
// every other wait checks, and the CTA drains its copies before returning.
#pragma once

// l3g_persist_plan.h (the schedule) is included by l3g_kernels.cuh.

struct PersistLayer {
  const uint8_t* w[persist::N_MAT];  // tiled QKV, Wo, up/gate, down (four rows per warp)
  const float* attn_norm;
  const float* ffn_norm;
};

struct PersistArgs {
  persist::Plan plan;
  const PersistLayer* layers;  // [n_layers] on the device
  int nstages, slot_bytes;     // ring
  int union_bytes, xq_off;     // phase scratch; int8 activation offset in it
  float eps, scale;            // rmsNorm eps; float32(1/sqrt(hd)), infer.go:130
  int n_emb, n_ff, hq, head_dim, group, rope_half;
  float* xa;      // residual stream: layer input (k_embed writes the embedding)
  float* xb;      // residual after the attention block
  float* y;       // Wo / down output
  float* q;       // [hq][hd] roped queries
  float* attn;    // [hq][hd] attention output, and Q8_0 for Wo:
  float* attn_d;
  int8_t* attn_q;
  float* act;     // SwiGLU output, and Q8_0 for down:
  float* act_d;
  int8_t* act_q;
  float* part_o;  // [hkv][splits][group][hd]
  float* part_ml; // [hkv][splits][group][2]
  const float* rope_cos;  // [ctx][rope_half]
  const float* rope_sin;
  const int* io;          // io[1] = position of this token
  KvMap kv;               // the state's KV cache (paged)
  unsigned* bar;          // barrier counters, abort word, handshakes (persist::BAR_*), zeroed by k_embed
  int nsub;               // barrier counters in use (1 .. BAR_MAX_SUB)
  int fuse_quant;         // the SwiGLU act-quant runs in the up/gate phase (no QUANT phase)
  int fuse_merge;         // the split merge runs in the attention phase (k_layers<..., true>)
  int bpl;                // grid barriers per layer (7, less one per fusion)
  Result* res;
  unsigned long long wait_ns;
  TpExchange tp;          // tp.world > 1: Wo / down rows pushed to every rank
  unsigned long long* stamps;  // nullable: [barrier][cta] {arrival, release} %globaltimer
};

struct PSmem {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  float ssred[NW];
  int abort_flag;
  int issued;
  int producer_done;
  int stop;  // the CTA's decision at a grid barrier (written by thread 0)
  int merge_last;  // fused merge: this CTA published its kv head's last partial
  // fused act-quant: warps done with the CTA's k-th up/gate group, slot
  // k % GSLOTS (warps drift apart by at most the ring's depth in tiles, so at
  // most MAX_STAGES groups: slots never alias)
  int gcnt[MAX_STAGES + 2];
};
constexpr int GSLOTS = MAX_STAGES + 2;
constexpr int PS_HEAD = 512;
static_assert(sizeof(PSmem) <= PS_HEAD, "persistent kernel smem head");

// Phase scratch, a union: the matvec phases' activation (fp32 block scales,
// then int8 values), or the attention phase's per-warp buffers and partial
// states, or the merge phase's per-warp split weights.
__host__ __device__ inline int ps_xq_off(int max_cols) { return align_up(max_cols / 32 * 4, 128); }
__host__ __device__ inline int ps_union_bytes(int max_cols, int group, int hd, int splits) {
  const int mv = ps_xq_off(max_cols) + align_up(max_cols, 128);
  const int att = AT_BUF + (NW * MAXG * 2 + NW * group * hd) * 4;
  const int mrg = NW * align_up(splits, 32) * 4;
  int u = mv > att ? mv : att;
  u = u > mrg ? u : mrg;
  return align_up(u, 1024);
}

__device__ __forceinline__ unsigned* ps_abort_word(const PersistArgs& a) {
  return a.bar + persist::BAR_ABORT;
}

// Bounded wait until barrier `idx` is complete (producer side, one thread:
// every counter, in order).
__device__ __forceinline__ bool ps_wait_barrier(const PersistArgs& a, int idx, PSmem* sh,
                                                int where) {
  const uint64_t t0 = gtime();
  for (int i = 0; i < a.nsub; ++i) {
    const unsigned target = (unsigned)(idx + 1) * persist::sub_count(gridDim.x, a.nsub, i);
    while (ld_acquire_gpu_u32(a.bar + i * persist::BAR_STRIDE) < target) {
      if (*(volatile int*)&sh->abort_flag || *(volatile unsigned*)ps_abort_word(a)) {
        sh->abort_flag = 1;
        return false;
      }
      if (gtime() - t0 > a.wait_ns) {
        sh->abort_flag = 1;
        report(a.res, ERR_TIMEOUT, where);
        atomicExch(ps_abort_word(a), 1u);
        return false;
      }
    }
  }
  return true;
}

// Grid barrier `idx` of the step, consumer warps only.  It is also where a
// CTA decides, for all its warps at once, to stop after an abort: a failed
// wait inside a phase only skips work (every warp still runs the phase's
// CTA barriers), so the warps always reach the same barriers.  Returns false
// when the step is aborting (this CTA's flag or the step's abort word).
// Warp 0 polls: lane i < nsub watches counter i (acquire), and the CTA
// barrier after it passes what those lanes acquired to every thread.
__device__ __forceinline__ bool ps_barrier(const PersistArgs& a, int idx, PSmem* sh) {
  consumer_sync();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const uint64_t t_arr = gtime();
    int stop = 0;
    if (lane == 0) {
      stop = *(volatile int*)&sh->abort_flag;
      if (stop) {
        atomicExch(ps_abort_word(a), 1u);  // the other CTAs stop waiting for this one
      } else {
        // release: this CTA's writes of the phase, ordered before it by the
        // CTA barrier above
        red_release_gpu_add(a.bar + (blockIdx.x % a.nsub) * persist::BAR_STRIDE, 1u);
      }
    }
    stop = __shfl_sync(0xffffffffu, stop, 0);
    if (!stop) {
      const bool mine = lane < a.nsub;
      const unsigned* ctr = a.bar + (mine ? lane : 0) * persist::BAR_STRIDE;
      const unsigned target =
          mine ? (unsigned)(idx + 1) * persist::sub_count(gridDim.x, a.nsub, lane) : 0u;
      for (;;) {
        const bool ready = !mine || ld_acquire_gpu_u32(ctr) >= target;
        if (__all_sync(0xffffffffu, ready)) break;
        int s = 0;
        if (lane == 0) {
          if (*(volatile int*)&sh->abort_flag || *(volatile unsigned*)ps_abort_word(a)) {
            s = 1;
          } else if (gtime() - t_arr > a.wait_ns) {
            report(a.res, ERR_TIMEOUT, 50);
            atomicExch(ps_abort_word(a), 1u);
            s = 1;
          }
        }
        if (__shfl_sync(0xffffffffu, s, 0)) {
          stop = 1;
          break;
        }
      }
      // the acquire loads above, then the CTA barrier below, order every
      // thread's reads of the next phase after the other CTAs' writes
    }
    if (lane == 0) {
      if (stop) sh->abort_flag = 1;  // the producer stops too
      sh->stop = stop;
      if (a.stamps) {
        unsigned long long* st = a.stamps + ((size_t)idx * gridDim.x + blockIdx.x) * 2;
        st[0] = t_arr;
        st[1] = gtime();
      }
    }
  }
  consumer_sync();
  return !sh->stop;
}

// ---------------------------------------------------------------------------
// producer: every tile of this CTA, in consumption order
// ---------------------------------------------------------------------------
static __device__ void ps_produce(const PersistArgs& a, PSmem* sh, uint8_t* ring) {
  using namespace persist;
  const Plan& p = a.plan;
  const int b = blockIdx.x, ns = a.nstages;
  uint32_t t = 0;
  int pos = -1;
  bool ok = true;
  auto issue = [&](const uint8_t* src, uint32_t bytes) -> bool {
    const int s = (int)(t % (uint32_t)ns);
    if (t >= (uint32_t)ns &&
        !mbar_wait(&sh->empty[s], ((t / ns) - 1) & 1, &sh->abort_flag, a.res, 40, a.wait_ns))
      return false;
    mbar_arrive_expect_tx(&sh->full[s], bytes);
    bulk_g2s(ring + (size_t)s * a.slot_bytes, src, bytes, &sh->full[s]);
    ++t;
    *(volatile int*)&sh->issued = (int)t;
    return true;
  };
  for (int l = 0; l < p.n_layers && ok; ++l) {
    const PersistLayer& L = a.layers[l];  // written at load time, not by this step
    for (int m = 0; m < N_MAT && ok; ++m) {
      if (m == M_WO) {  // the attention item's K|V stages come between QKV and Wo
        if (pos < 0) {
          pdl_wait();  // the position is set by the step's first copy / k_advance
          pos = a.io[1];
        }
        int kvh, split;
        if (my_item(p, l, b, &kvh, &split)) {
          int t0, t1;
          item_range(p, split, pos + 1, &t0, &t1);
          const int nst = item_stages(p, t0, t1);
          bool waited = false;
          for (int st = 0; st < nst && ok; ++st) {
            const int ta = t0 + st * p.P;
            const int tb = min(t1, ta + p.P);
            if (!waited && tb > pos) {
              // this step's own K/V row is appended in the QKV phase
              ok = ps_wait_barrier(a, barrier_index(l, 0, a.bpl), sh, 42);
              fence_proxy_async_global();
              waited = true;
              if (!ok) break;
            }
            // ta is a multiple of P, which divides KV_PAGE: one page
            ok = issue(kv_row(a.kv, l, kvh, ta), (uint32_t)((tb - ta) * p.row_bytes));
          }
        }
      }
      const int ngr = my_groups(p, l, m, b);
      for (int k = 0; k < ngr && ok; ++k) {
        const int g = my_group(p, l, m, b, k);
        for (int s = 0; s < p.nsl[m] && ok; ++s)
          ok = issue(L.w[m] + tile_offset(p, m, g, s), (uint32_t)p.tile_bytes[m]);
      }
    }
  }
  *(volatile int*)&sh->producer_done = 1;
}

// ---------------------------------------------------------------------------
// consumer phases
// ---------------------------------------------------------------------------
// Residual add (infer.go:189-191 / :244-246), rmsNorm (math.go:5-14), block
// act-quant into shared memory; CTA 0 stores the new residual.  The same
// arithmetic as k_matvec's PRO_RMS prologue.
static __device__ void ps_rms(const PersistArgs& a, const float* x_in, const float* y_in,
                       const float* norm_w, float* x_out, float* xd, int8_t* xqs, PSmem* sh) {
  constexpr int VKM = 8;  // float4 per thread: n_emb <= 8192
  const int C = a.n_emb, nv = C >> 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float4* x4 = reinterpret_cast<const float4*>(x_in);
  const float4* y4 = reinterpret_cast<const float4*>(y_in);
  float4 v[VKM];
#pragma unroll
  for (int k = 0; k < VKM; ++k) {
    const int i = tid + k * NW * 32;
    v[k] = i < nv ? __ldcg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (y_in && i < nv) {
      const float4 yy = __ldcg(y4 + i);
      v[k].x = __fadd_rn(v[k].x, yy.x);
      v[k].y = __fadd_rn(v[k].y, yy.y);
      v[k].z = __fadd_rn(v[k].z, yy.z);
      v[k].w = __fadd_rn(v[k].w, yy.w);
    }
  }
  const bool wx = x_out != nullptr && blockIdx.x == 0;
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < VKM; ++k) {
    const int i = tid + k * NW * 32;
    if (wx && i < nv) reinterpret_cast<float4*>(x_out)[i] = v[k];
    ss = fmaf(v[k].x, v[k].x, ss);
    ss = fmaf(v[k].y, v[k].y, ss);
    ss = fmaf(v[k].z, v[k].z, ss);
    ss = fmaf(v[k].w, v[k].w, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) sh->ssred[warp] = ss;
  consumer_sync();
  float tot = 0.0f;
#pragma unroll
  for (int q = 0; q < NW; ++q) tot += sh->ssred[q];
  const float scale = (float)(1.0 / sqrt((double)__fadd_rn(__fdiv_rn(tot, (float)C), a.eps)));
  const float4* w4 = reinterpret_cast<const float4*>(norm_w);
#pragma unroll
  for (int k = 0; k < VKM; ++k) {
    const int i = tid + k * NW * 32;
    if (k * NW * 32 >= nv) break;  // uniform: nv is a multiple of 8
    const float4 w = i < nv ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 u = v[k];
    u.x = __fmul_rn(__fmul_rn(u.x, scale), w.x);
    u.y = __fmul_rn(__fmul_rn(u.y, scale), w.y);
    u.z = __fmul_rn(__fmul_rn(u.z, scale), w.z);
    u.w = __fmul_rn(__fmul_rn(u.w, scale), w.w);
    quant_quad(u, i < nv, i >> 3, lane & 7, xd, xqs);
  }
  consumer_sync();
}

// Copy of an activation another phase quantized (the attention merge, the
// SwiGLU quantize phase) into shared memory.
static __device__ void ps_preq(const float* d_in, const int8_t* q_in, int C, float* xd, int8_t* xqs) {
  const int tid = threadIdx.x;
  for (int i = tid * 16; i < C; i += NW * 32 * 16)
    *reinterpret_cast<int4*>(xqs + i) = __ldcg(reinterpret_cast<const int4*>(q_in + i));
  for (int i = tid; i < C / 32; i += NW * 32) xd[i] = __ldcg(d_in + i);
  consumer_sync();
}

enum PsEpi { PE_STORE = 0, PE_QKV = 1, PE_SWIGLU = 2, PE_PUSH = 3 };

// Epilogue of the four rows row0..row0+3 of one warp; lane r < 4 holds row
// row0 + r.  Pairs (RoPE, up/gate) sit in lanes (0,1) and (2,3).
template <int EPI>
__device__ __forceinline__ void ps_epilogue(const PersistArgs& a, int m, int l, int row0, float v,
                                            int lane, float* out, int pos, size_t push_off,
                                            unsigned push_e) {
  const int row = row0 + lane;
  const bool live = lane < 4 && row < a.plan.rows[m];
  if constexpr (EPI == PE_STORE) {
    if (live) out[row] = v;
  } else if constexpr (EPI == PE_PUSH) {
    if (live) {
      const unsigned long long word = ((unsigned long long)push_e << 32) | __float_as_uint(v);
#pragma unroll
      for (int r = 0; r < MAX_WORLD; ++r)
        if (r < a.tp.world) st_relaxed_sys_u64(a.tp.recv[r] + push_off + row, word);
    }
  } else if constexpr (EPI == PE_SWIGLU) {
    // rows interleave (up_i, gate_i); act_i = silu(gate_i) * up_i
    const float gate = __shfl_down_sync(0xffffffffu, v, 1);
    if (live && !(lane & 1)) out[row >> 1] = __fmul_rn(silu_ref(gate), v);
  } else {  // PE_QKV
    const float v1 = __shfl_down_sync(0xffffffffu, v, 1);
    if (live && !(lane & 1)) {
      float x0 = v, x1 = v1;
      const int hd = a.head_dim;
      const int nq = a.hq * hd, nkv = a.plan.hkv * hd;
      const bool is_q = row < nq;
      const bool is_k = !is_q && row < nq + nkv;
      if (is_q || is_k) {  // RoPE on the adjacent pair, rope.go:39-52
        const int d = (is_q ? row : row - nq) % hd;
        const int i = d >> 1;
        if (i < a.rope_half) {
          const float c = a.rope_cos[(size_t)pos * a.rope_half + i];
          const float s = a.rope_sin[(size_t)pos * a.rope_half + i];
          const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
          const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
          x0 = y0;
          x1 = y1;
        }
      }
      if (is_q) {
        *reinterpret_cast<float2*>(out + row) = make_float2(x0, x1);
      } else {  // KV append at this position, infer.go:122-127
        const int r2 = is_k ? row - nq : row - nq - nkv;
        const int kvh = r2 / hd, d = r2 % hd;
        const size_t off = (is_k ? 0 : hd) + d;
        uint8_t* base = kv_row(a.kv, l, kvh, pos);
        if (a.plan.row_bytes == 4 * hd)  // f16 cache: 2 * hd elements of 2 bytes
          *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + off) =
              __floats2half2_rn(x0, x1);
        else
          *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + off) = make_float2(x0, x1);
        fence_proxy_async_global();  // read next by other CTAs' bulk copies
      }
    }
  }
}

// Fused act-quant of the SwiGLU output (QuantizeQ8_0Into, infer.go:233-234),
// run by a warp right after its epilogue of up/gate row group g (the CTA's
// k-th): group g holds act values [16g, 16g + 16), half of Q8_0 block g / 2.
// The last of the CTA's warps to finish the group (a shared-memory count)
// adds one to the block's counter in global memory; whoever brings it to 2,
// in this CTA or another, reads the block's 32 values back and quantizes
// them (quant_block, as ps_quant would), then zeroes the counter for the
// next layer.  Ordering: each warp's lanes' act stores (via __syncwarp) come
// before its CTA-scope acquire-release count; the warp that completes the
// group thus follows every warp's stores, and its device-scope
// acquire-release add on the block's counter publishes them all (and, for
// the second arriver, acquires the other half's).
__device__ __forceinline__ void ps_swiglu_quant(const PersistArgs& a, PSmem* sh, int k, int g,
                                                int lane) {
  __syncwarp();
  int last = 0;
  if (lane == 0)
    last = atom_add_acq_rel_cta_shared(reinterpret_cast<unsigned*>(&sh->gcnt[k % GSLOTS]), 1u) ==
           (unsigned)(NW - 1);
  if (!__shfl_sync(0xffffffffu, last, 0)) return;
  const int blk = g >> 1;
  unsigned* cnt = a.bar + persist::BAR_QCNT + blk;
  int second = 0;
  if (lane == 0) {
    sh->gcnt[k % GSLOTS] = 0;  // its next use is GSLOTS groups later
    second = atom_add_acq_rel_gpu(cnt, 1u) == 1u;
  }
  if (!__shfl_sync(0xffffffffu, second, 0)) return;
  const int i = blk * 32 + lane;
  quant_block(i < a.n_ff ? __ldcg(a.act + i) : 0.0f, blk, lane, a.act_d, a.act_q);
  if (lane == 0) *cnt = 0u;
}

// This CTA's row groups of matrix m: four rows per warp, dp4a against the
// int8 activation in shared memory, fp16(d_w) * d_x per 32-block.  After a
// failed wait the warp neither uses nor releases its tiles (no copy can then
// be issued into a slot whose previous copy may be in flight) and skips its
// epilogues; the following waits return at once.
template <int EPI>
__device__ void ps_matvec(const PersistArgs& a, int m, int l, uint32_t& t, const float* xd,
                          const int8_t* xqs, PSmem* sh, const uint8_t* ring, float* out,
                          int pos, size_t push_off, unsigned push_e) {
  using namespace persist;
  const Plan& p = a.plan;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.nstages;
  const int ck = p.ck[m], nsl = p.nsl[m], wr = p.wr[m];
  const int nchunks = ck >> 4, nbk = ck >> 5;
  const int ngr = my_groups(p, l, m, blockIdx.x);
  bool alive = true;
  for (int k = 0; k < ngr; ++k) {
    const int g = my_group(p, l, m, blockIdx.x, k);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int sl = 0; sl < nsl; ++sl, ++t) {
      const int s = (int)(t % (uint32_t)ns);
      alive = alive && __all_sync(0xffffffffu, mbar_wait(&sh->full[s], (t / ns) & 1,
                                                         &sh->abort_flag, a.res, 41, a.wait_ns));
      if (!alive) continue;
      const uint8_t* tile = ring + (size_t)s * a.slot_bytes;
      const uint8_t* wq = tile + (size_t)warp * 4 * ck;
      const __half* wd = reinterpret_cast<const __half*>(tile + (size_t)wr * ck) + warp * 4 * nbk;
      const int8_t* xq = xqs + sl * ck;
      const float* xs = xd + sl * nbk;
#pragma unroll 2
      for (int c = lane; c < nchunks; c += 32) {
        const int4 x4 = *reinterpret_cast<const int4*>(xq + c * 16);
        const float sx = xs[c >> 1];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int4 w4 = *reinterpret_cast<const int4*>(wq + (size_t)r * ck + c * 16);
          int isum = __dp4a(w4.x, x4.x, 0);
          isum = __dp4a(w4.y, x4.y, isum);
          isum = __dp4a(w4.z, x4.z, isum);
          isum = __dp4a(w4.w, x4.w, isum);
          acc[r] = fmaf((float)isum, __half2float(wd[r * nbk + (c >> 1)]) * sx, acc[r]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[s]);
    }
    if (!alive) continue;
    float v = 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float sr = warp_sum(acc[r]);
      if (lane == r) v = sr;
    }
    ps_epilogue<EPI>(a, m, l, g * wr + warp * 4, v, lane, out, pos, push_off, push_e);
    if constexpr (EPI == PE_SWIGLU)
      if (a.fuse_quant) ps_swiglu_quant(a, sh, k, g, lane);
  }
}

// This CTA's attention item: the loop of k_attention (same sub-batches,
// stage groups and online softmax), then the merge of the warps' states into
// the item's (m, l, o) partial.  Every warp waits for and releases every
// stage; a stage group computes only its own stages.  After a failed wait
// the warp skips the remaining stages' work (as in ps_matvec) but still
// joins the CTA merge, so every warp reaches the same CTA barriers.
template <int DPL, typename KT, int GP>
__device__ void ps_attention(const PersistArgs& a, int l, int n, uint32_t& t, uint8_t* uni,
                             const uint8_t* ring, PSmem* sh) {
  using namespace persist;
  constexpr int SB = 32 / GP;
  const Plan& p = a.plan;
  int kvh, split;
  if (!my_item(p, l, blockIdx.x, &kvh, &split)) return;  // uniform over the CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = a.head_dim, G = a.group, P = p.P, S = p.splits, ns = a.nstages;
  int t0, t1;
  item_range(p, split, n, &t0, &t1);
  const int nst = item_stages(p, t0, t1);
  const int row = 2 * hd;
  const int wsz = (P / SB >= NW) ? NW : NW / 2;
  const int ngrp = NW / wsz;
  const int nbw = P / wsz;
  float* pbuf_all = reinterpret_cast<float*>(uni);
  float* hbuf_all = pbuf_all + NW * 32;
  float* sm_ml = reinterpret_cast<float*>(uni + AT_BUF);  // [NW][MAXG][2]
  float* sm_o = sm_ml + NW * MAXG * 2;                     // [NW][G][hd]

  float q[GP][DPL];
#pragma unroll
  for (int h = 0; h < GP; ++h)
#pragma unroll
    for (int j = 0; j < DPL; ++j)
      q[h][j] = h < G ? __ldcg(a.q + ((size_t)kvh * G + h) * hd + lane * DPL + j) : 0.0f;
  float mx[GP], ls[GP], o[GP][DPL];
#pragma unroll
  for (int h = 0; h < GP; ++h) {
    mx[h] = -INFINITY;
    ls[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[h][j] = 0.0f;
  }
  float* pbuf = pbuf_all + warp * 32;
  float* hbuf = hbuf_all + warp * MAXG * 4;
  const int my_h = lane % GP;
  const int my_p = lane / GP;
  const int grp = warp / wsz, wj = warp % wsz;

  bool alive = true;
  for (int st = 0; st < nst; ++st, ++t) {
    const int s = (int)(t % (uint32_t)ns);
    alive = alive && __all_sync(0xffffffffu, mbar_wait(&sh->full[s], (t / ns) & 1,
                                                       &sh->abort_flag, a.res, 43, a.wait_ns));
    if (!alive) continue;
    if (st % ngrp == grp) {
      const int cnt = min(t1, t0 + st * P + P) - (t0 + st * P);
      const KT* Ks = reinterpret_cast<const KT*>(ring + (size_t)s * a.slot_bytes);
      const KT* Vs = Ks + hd;
      for (int sb = 0; sb < nbw; sb += SB) {
        const int p0 = wj * nbw + sb;
        const int np = min(SB, nbw - sb);
        float v[32];
#pragma unroll
        for (int pp = 0; pp < SB; ++pp) {
          float kv[DPL];
          if (pp < np && p0 + pp < cnt) {
            load_row<DPL, KT>(Ks + (size_t)(p0 + pp) * row + lane * DPL, kv);
          } else {
#pragma unroll
            for (int j = 0; j < DPL; ++j) kv[j] = 0.0f;
          }
#pragma unroll
          for (int h = 0; h < GP; ++h) {
            float d = 0.0f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) d = fmaf(q[h][j], kv[j], d);
            v[pp * GP + h] = d;
          }
        }
        const float dot = transpose_reduce32(v, lane);
        const bool valid = my_p < np && p0 + my_p < cnt && my_h < G;
        const float sc = valid ? dot * a.scale : -INFINITY;
        float mb = sc;
#pragma unroll
        for (int off = GP; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        float mo = -INFINITY;
#pragma unroll
        for (int h = 0; h < GP; ++h)
          if (h == my_h) mo = mx[h];
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
          mx[h] = hbuf[h * 4 + 0];
          ls[h] = fmaf(ls[h], c, hbuf[h * 4 + 2]);
#pragma unroll
          for (int j = 0; j < DPL; ++j) o[h][j] *= c;
        }
        for (int pp = 0; pp < np && p0 + pp < cnt; ++pp) {
          float vv[DPL];
          load_row<DPL, KT>(Vs + (size_t)(p0 + pp) * row + lane * DPL, vv);
          float w[GP];
          if constexpr (GP % 4 == 0) {
#pragma unroll
            for (int k = 0; k < GP / 4; ++k) {
              const float4 t4 = reinterpret_cast<const float4*>(pbuf + pp * GP)[k];
              w[4 * k] = t4.x;
              w[4 * k + 1] = t4.y;
              w[4 * k + 2] = t4.z;
              w[4 * k + 3] = t4.w;
            }
          } else {
#pragma unroll
            for (int h = 0; h < GP; ++h) w[h] = pbuf[pp * GP + h];
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

  // the warps' states -> this item's partial, k_attention's CTA merge
#pragma unroll
  for (int h = 0; h < GP; ++h) {
    if (h < G) {
      if (lane == 0) {
        sm_ml[(warp * MAXG + h) * 2] = mx[h];
        sm_ml[(warp * MAXG + h) * 2 + 1] = ls[h];
      }
#pragma unroll
      for (int j = 0; j < DPL; ++j) sm_o[((size_t)warp * G + h) * hd + lane * DPL + j] = o[h][j];
    }
  }
  consumer_sync();
  const size_t pbase = ((size_t)kvh * S + split) * G;
  for (int idx = threadIdx.x; idx < G * hd; idx += NW * 32) {
    const int h = idx / hd, d = idx % hd;
    float mw[NW], lw[NW], ow[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      mw[w] = sm_ml[(w * MAXG + h) * 2];
      lw[w] = sm_ml[(w * MAXG + h) * 2 + 1];
      ow[w] = sm_o[((size_t)w * G + h) * hd + d];
    }
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, mw[w]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float e = mw[w] == -INFINITY ? 0.0f : expf(mw[w] - M);
        L = fmaf(lw[w], e, L);
        O = fmaf(ow[w], e, O);
      }
    }
    a.part_o[(pbase + h) * hd + d] = O;
    if (d == 0) {
      a.part_ml[(pbase + h) * 2] = M;
      a.part_ml[(pbase + h) * 2 + 1] = L;
    }
  }
}

// Merge of the splits of kv head kvh for output block blk (32 outputs of one
// query head) in split order, k_attention's global merge, and its act-quant
// for Wo.  One warp; wbuf holds align_up(splits, 32) floats of its own.
static __device__ void ps_merge_block(const PersistArgs& a, float* wbuf, int kvh, int blk, int lane) {
  const int S = a.plan.splits, G = a.group, hd = a.head_dim, gh = G * hd;
  const int h = blk * 32 / hd;
  const float* ml = a.part_ml + (size_t)kvh * S * G * 2;
  const float* po = a.part_o + (size_t)kvh * S * gh;
  const float v = merge_split_block(ml, po, S, G, gh, h, blk * 32 + lane, lane, wbuf);
  a.attn[(size_t)kvh * gh + blk * 32 + lane] = v;
  quant_block(v, kvh * gh / 32 + blk, lane, a.attn_d, a.attn_q);
}

// Merge of output blocks gb0, gb0 + step, ... < gb1 (block gb: kv head
// gb / (group * hd / 32), its block gb % (group * hd / 32)), one warp each.
// Unfused, after the attention barrier, the grid's warps share every block;
// with the fused merge, the warps of the CTA that claimed a kv head take its
// blocks.  One call site, so the merge is inlined once into k_layers.
static __device__ void ps_merge(const PersistArgs& a, uint8_t* uni, int gb0, int gb1, int step) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = a.group * a.head_dim / 32;
  float* wbuf = reinterpret_cast<float*>(uni) + warp * align_up(a.plan.splits, 32);
  for (int gb = gb0; gb < gb1; gb += step) ps_merge_block(a, wbuf, gb / per, gb % per, lane);
}

// The merge folded into the attention phase (fuse_merge): after publishing
// its item's partial, a CTA adds one to its kv head's arrival counter (after
// the quantization handshake words of the barrier area); the CTA that brings
// it to the split count claims that kv head -- its warps merge the head's
// blocks (ps_merge, the same arithmetic, so results are unchanged) -- and
// returns the counter to 0 for the next layer.  Returns the claimed kv head
// or -1.  Ordering as at a grid barrier: every thread's partial stores, the
// CTA barrier, then thread 0's acquire-release add (release for this CTA's
// partials, acquire for the claimer), then the CTA barrier before the
// claimer's warps read the partials.
static __device__ int ps_merge_claim(const PersistArgs& a, int l, PSmem* sh) {
  int kvh, split;
  if (!persist::my_item(a.plan, l, blockIdx.x, &kvh, &split)) return -1;  // uniform over the CTA
  consumer_sync();
  if (threadIdx.x == 0) {
    unsigned* cnt = a.bar + persist::BAR_QCNT + a.n_ff / 32 + kvh;
    const bool last = atom_add_acq_rel_gpu(cnt, 1u) == (unsigned)(a.plan.splits - 1);
    if (last) *cnt = 0u;  // read again only after the next grid barrier
    sh->merge_last = last ? 1 : 0;
  }
  consumer_sync();
  return sh->merge_last ? kvh : -1;
}

// Act-quant of the SwiGLU output (infer.go:233-234), one warp per block.
static __device__ void ps_quant(const PersistArgs& a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = a.n_ff, nb = (n + 31) / 32;
  for (int blk = blockIdx.x * NW + warp; blk < nb; blk += gridDim.x * NW) {
    const int i = blk * 32 + lane;
    quant_block(i < n ? __ldcg(a.act + i) : 0.0f, blk, lane, a.act_d, a.act_q);
  }
}

// Tensor-parallel sum of the phase's pushed rows in rank order (k_tp_reduce
// spread over the grid's threads).
static __device__ void ps_reduce(const PersistArgs& a, unsigned e) {
  const TpExchange& t = a.tp;
  const int i = blockIdx.x * (NW * 32) + threadIdx.x;
  if (4 * i >= t.n) return;
  const unsigned long long* rb = t.my_recv + (size_t)(e & 1u) * t.world * t.n + 4 * i;
  const uint64_t t_start = gtime();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  bool late = false;
#pragma unroll
  for (int r = 0; r < MAX_WORLD; ++r) {
    if (r >= t.world) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      unsigned long long w = ld_relaxed_sys_u64(rb + (size_t)r * t.n + j);
      while (!late && (unsigned)(w >> 32) != e) {
        if (*(volatile unsigned*)ps_abort_word(a) || gtime() - t_start > a.wait_ns) {
          if (!*(volatile unsigned*)ps_abort_word(a)) report(a.res, ERR_TIMEOUT, 51);
          atomicExch(ps_abort_word(a), 1u);
          late = true;
          break;
        }
        w = ld_relaxed_sys_u64(rb + (size_t)r * t.n + j);
      }
      const float v = __uint_as_float((unsigned)w);
      acc[j] = r == 0 ? v : __fadd_rn(acc[j], v);
    }
  }
  reinterpret_cast<float4*>(a.y)[i] = make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// FM: the split merge folded into the attention phase (a.fuse_merge), a
// separate instantiation so that the unfused kernel's registers are its own.
template <int DPL, typename KT, int GP, bool FM>
__global__ void __launch_bounds__(NTHREADS, 1) k_layers(const __grid_constant__ PersistArgs a) {
  using namespace persist;
  L3G_DYNAMIC_SMEM(smem);
  PSmem* sh = reinterpret_cast<PSmem*>(smem);
  uint8_t* uni = smem + PS_HEAD;
  uint8_t* ring = uni + a.union_bytes;
  const Plan& p = a.plan;
  const int warp = threadIdx.x >> 5;
  const int ns = a.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], NW);
    }
    sh->abort_flag = 0;
    sh->issued = 0;
    sh->producer_done = 0;
    for (int i = 0; i < GSLOTS; ++i) sh->gcnt[i] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NW) {  // producer
    if ((threadIdx.x & 31) == 0) ps_produce(a, sh, ring);
    return;
  }

  float* xd = reinterpret_cast<float*>(uni);
  int8_t* xqs = reinterpret_cast<int8_t*>(uni + a.xq_off);
  pdl_wait();  // the embedding row, the position and the step counter
  const int pos = a.io[1];
  const unsigned e0 = a.tp.world > 1 ? *a.tp.step * (unsigned)a.tp.nphase : 0u;
  const bool tp = a.tp.world > 1;
  uint32_t t = 0;
  int bi = 0;  // grid barriers passed (barrier_index order)
  for (int l = 0; l < p.n_layers; ++l) {
    const PersistLayer& L = a.layers[l];
    const bool last = l + 1 == p.n_layers;
    // QKV: RMSNorm -> act-quant -> QKV -> RoPE -> KV append, infer.go:67-127
    ps_rms(a, a.xa, l ? a.y : nullptr, L.attn_norm, a.xb, xd, xqs, sh);
    ps_matvec<PE_QKV>(a, M_QKV, l, t, xd, xqs, sh, ring, a.q, pos, 0, 0);
    if (!ps_barrier(a, bi++, sh)) break;
    // attention, infer.go:130-175
    ps_attention<DPL, KT, GP>(a, l, pos + 1, t, uni, ring, sh);
    if constexpr (FM) {  // the merge by the CTA that claims a kv head
      const int kvh = ps_merge_claim(a, l, sh), per = a.group * a.head_dim / 32;
      if (kvh >= 0) ps_merge(a, uni, kvh * per + warp, (kvh + 1) * per, NW);
    } else {  // the merge spread over the grid after a barrier
      if (!ps_barrier(a, bi++, sh)) break;
      ps_merge(a, uni, blockIdx.x * NW + warp, a.hq * a.head_dim / 32, gridDim.x * NW);
    }
    if (!ps_barrier(a, bi++, sh)) break;
    // Wo, infer.go:178-187 (the residual add is fused into the next norm)
    ps_preq(a.attn_d, a.attn_q, p.cols[M_WO], xd, xqs);
    if (tp) {
      const unsigned e = e0 + 2u * l;
      const size_t off = (size_t)((e & 1u) * a.tp.world + a.tp.rank) * a.tp.n;
      ps_matvec<PE_PUSH>(a, M_WO, l, t, xd, xqs, sh, ring, nullptr, pos, off, e);
      ps_reduce(a, e);
    } else {
      ps_matvec<PE_STORE>(a, M_WO, l, t, xd, xqs, sh, ring, a.y, pos, 0, 0);
    }
    if (!ps_barrier(a, bi++, sh)) break;
    // residual -> RMSNorm -> act-quant -> up/gate -> SwiGLU, infer.go:189-230
    // (and its act-quant, infer.go:233-234, when fused)
    ps_rms(a, a.xb, a.y, L.ffn_norm, a.xa, xd, xqs, sh);
    ps_matvec<PE_SWIGLU>(a, M_UPGATE, l, t, xd, xqs, sh, ring, a.act, pos, 0, 0);
    if (!ps_barrier(a, bi++, sh)) break;
    if (!a.fuse_quant) {
      ps_quant(a);
      if (!ps_barrier(a, bi++, sh)) break;
    }
    // down, infer.go:233-242
    if (last) pdl_launch_dependents();  // the logits kernel may take SMs as CTAs finish
    ps_preq(a.act_d, a.act_q, p.cols[M_DOWN], xd, xqs);
    if (tp) {
      const unsigned e = e0 + 2u * l + 1u;
      const size_t off = (size_t)((e & 1u) * a.tp.world + a.tp.rank) * a.tp.n;
      ps_matvec<PE_PUSH>(a, M_DOWN, l, t, xd, xqs, sh, ring, nullptr, pos, off, e);
      ps_reduce(a, e);
    } else {
      ps_matvec<PE_STORE>(a, M_DOWN, l, t, xd, xqs, sh, ring, a.y, pos, 0, 0);
    }
    if (!last && !ps_barrier(a, bi++, sh)) break;
  }

  // After an abort: wait (bounded) until the producer has stopped issuing,
  // then for the last copy issued to each ring slot.
  consumer_sync();
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const uint64_t t_start = gtime();
    while (!*(volatile int*)&sh->producer_done && gtime() - t_start < 100000000ull) {
    }
    const int issued = *(volatile int*)&sh->issued;
    for (int s2 = 0; s2 < ns && s2 < issued; ++s2) {
      const int tt = s2 + ((issued - 1 - s2) / ns) * ns;
      int dummy = 0;
      mbar_wait(&sh->full[s2], (tt / ns) & 1, &dummy, a.res, 44, 100000000ull);
    }
  }
}
