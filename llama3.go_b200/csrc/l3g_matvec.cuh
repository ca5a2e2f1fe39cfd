// Q8_0 matvec kernels of libl3g (included by l3g_kernels.cuh).
#pragma once

// ---------------------------------------------------------------------------
// Repacked Q8_0 matrix.  Rows are grouped by `wr` (= NW * rows per warp) and
// columns sliced by `ck`;
// tile (g, s) holds rows [g*wr, g*wr+wr) x cols [s*ck, s*ck+ck):
//   int8 q[wr][ck] followed by fp16 d[wr][ck/32], padded to 16 bytes.
// Tiles are stored g-major: each tile is one contiguous bulk copy, and the
// grid as a whole walks the matrix front to back.
// ---------------------------------------------------------------------------
struct Q8Tiles {
  const uint8_t* data;
  int rows, cols, wr, ck, nslices, tile_bytes, n_groups;
};

enum Pro { PRO_PREQ = 0, PRO_RMS = 2 };
enum Epi { EPI_STORE = 0, EPI_QKV = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3, EPI_PUSH = 4 };

// Tensor-parallel reduction over peer memory (one process per GPU, receive
// buffers mapped with CUDA IPC).  The producer (EPI_PUSH: the Wo and down
// matvecs, whose rows are partial sums over this rank's columns) stores each
// row into slot `rank` of every rank's receive buffer as one 64-bit word
// {float bits, epoch}; a naturally aligned 64-bit access is single-copy
// atomic, so the consumer (k_tp_reduce, launched right after the producer)
// knows an element has arrived when its epoch matches, with no fence or
// flag.  It sums the ranks' values in rank order into this rank's y, so
// every rank gets bit-identical sums.  Receive
// buffers alternate between two parities by epoch: a rank cannot get two
// phases ahead of a reader, since its next-but-one push depends on the
// reader's push of the phase in between.
constexpr int MAX_WORLD = 8;
struct TpExchange {
  int world, rank, n;                    // ranks, this rank, vector length
  int nphase, phase;                     // epoch = *step * nphase + phase
  const unsigned* step;                  // device step counter (k_embed)
  unsigned long long* recv[MAX_WORLD];   // producer: rank r's buffer [2][world][n]
  const unsigned long long* my_recv;     // consumer: this rank's buffer
};
__device__ __forceinline__ unsigned tp_epoch(const TpExchange& t) {
  return *t.step * (unsigned)t.nphase + (unsigned)t.phase;
}

struct MatvecArgs {
  Q8Tiles w;
  int nstages;
  int row_lo, row_hi;  // rows this launch covers / writes
  // prologue
  const float* x_in;    // PRO_RMS: residual
  const float* y_in;    // PRO_RMS: delta added to x_in first (or null)
  const float* norm_w;  // PRO_RMS
  float* x_out;         // PRO_RMS: x_in + y_in written by CTA 0 (or null)
  float eps;
  const float* xd_in;   // PRO_PREQ: pre-quantized activation (device)
  const int8_t* xqs_in;
  // epilogue
  float* out;
  // EPI_QKV: rows are [q | k | v] of this rank's heads
  int nq, nkv, head_dim, rope_half, layer, kv_f16;
  const float* rope_cos;  // [ctx][rope_half]
  const float* rope_sin;
  const int* io;          // io[0] token, io[1] position
  KvMap kv;               // the state's KV cache; this layer's rows are written
  // EPI_LOGITS: fused argmax
  int row_offset;         // vocab id of local row 0
  float* am_val;          // [gridDim.x] per-CTA best
  int* am_idx;
  unsigned* am_counter;   // zero between launches
  Result* res;            // error word, argmax result
  unsigned long long* trace;  // device timeline (nullptr: off)
  int trace_seq;
  TpExchange tp_out;      // EPI_PUSH
  unsigned long long wait_ns;  // bound of every wait (WAIT_TIMEOUT_NS or _PEER_NS)
};

// Row-group partial sums: a ring of slots, one per group in flight.  Warps
// drift apart by at most MAX_STAGES tiles (the producer refills a stage only
// after every consumer warp released it), so MAX_STAGES + 2 slots never alias.
constexpr int RED_SLOTS = MAX_STAGES + 2;

struct MatvecSmem {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  float red[RED_SLOTS][NW];
  int cnt[RED_SLOTS];
  float ssred[NW];
  float best_v[NW];
  int best_i[NW];
  int abort_flag;
  int issued;
  int producer_done;
  int last;
};
constexpr int MV_HEAD = 1024;
static_assert(sizeof(MatvecSmem) <= MV_HEAD, "matvec smem head");

__host__ __device__ __forceinline__ int mv_smem_bytes(int cols, int nstages,
                                                      int tile_bytes) {
  return MV_HEAD + align_up(cols / 32 * 4, 128) + align_up(cols, 128) +
         nstages * tile_bytes;
}

// VK: float4 of the input row per thread for PRO_RMS (C <= 1024 * VK).
template <int PRO, int VK>
__device__ __forceinline__ void mv_prologue(const MatvecArgs& a, float* xd,
                                            int8_t* xqs, MatvecSmem* sh,
                                            const float4* w) {
  const int C = a.w.cols;
  const int nb = C >> 5;
  const int tid = threadIdx.x;  // < NW*32
  const int warp = tid >> 5, lane = tid & 31;
  if constexpr (PRO == PRO_PREQ) {
    // copy the quantized activation, 16 KB of int8 and 512 scales per
    // round: each thread's loads of a round are issued before its stores
    for (int base = 0; base < C; base += 4 * NW * 32 * 16) {
      int4 q[4];
      float dv[2];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = base + (tid + k * NW * 32) * 16;
        q[k] = i < C ? *reinterpret_cast<const int4*>(a.xqs_in + i) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = base / 32 + tid + k * NW * 32;
        dv[k] = i < nb ? a.xd_in[i] : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = base + (tid + k * NW * 32) * 16;
        if (i < C) *reinterpret_cast<int4*>(xqs + i) = q[k];
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = base / 32 + tid + k * NW * 32;
        if (i < nb) xd[i] = dv[k];
      }
    }
    trace_mark(a.trace, a.trace_seq, 7);  // copied
  } else {
    // residual add (infer.go:189-191 / :244-246), rmsNorm (math.go:5-14),
    // then the block quantization; w (the norm weights, loaded before the
    // dependency wait) and v hold this thread's VK float4 of the row.
    const int nv = C >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(a.x_in);
    const float4* y4 = reinterpret_cast<const float4*>(a.y_in);
    const bool has_y = a.y_in != nullptr;
    // v = x + delta, one float4 of each at a time
    float4 v[VK];
#pragma unroll
    for (int k = 0; k < VK; ++k) {
      const int i = tid + k * NW * 32;
      v[k] = i < nv ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (has_y && i < nv) {
        const float4 y = y4[i];
        v[k].x = __fadd_rn(v[k].x, y.x);
        v[k].y = __fadd_rn(v[k].y, y.y);
        v[k].z = __fadd_rn(v[k].z, y.z);
        v[k].w = __fadd_rn(v[k].w, y.w);
      }
    }
    const bool wx = a.x_out != nullptr && blockIdx.x == 0;
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VK; ++k) {
      const int i = tid + k * NW * 32;
      if (wx && i < nv) reinterpret_cast<float4*>(a.x_out)[i] = v[k];
      ss = fmaf(v[k].x, v[k].x, ss);
      ss = fmaf(v[k].y, v[k].y, ss);
      ss = fmaf(v[k].z, v[k].z, ss);
      ss = fmaf(v[k].w, v[k].w, ss);
    }
    trace_mark(a.trace, a.trace_seq, 5);  // inputs loaded
    ss = warp_sum(ss);
    if (lane == 0) sh->ssred[warp] = ss;
    consumer_sync();
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < NW; ++q) tot += sh->ssred[q];
    const float scale = (float)(1.0 / sqrt((double)__fadd_rn(__fdiv_rn(tot, (float)C), a.eps)));
    trace_mark(a.trace, a.trace_seq, 6);  // scale known
#pragma unroll
    for (int k = 0; k < VK; ++k) {
      const int i = tid + k * NW * 32;
      if (k * NW * 32 >= nv) break;  // uniform: nv is a multiple of 8
      float4 u = v[k];
      u.x = __fmul_rn(__fmul_rn(u.x, scale), w[k].x);
      u.y = __fmul_rn(__fmul_rn(u.y, scale), w[k].y);
      u.z = __fmul_rn(__fmul_rn(u.z, scale), w[k].z);
      u.w = __fmul_rn(__fmul_rn(u.w, scale), w[k].w);
      quant_quad(u, i < nv, i >> 3, lane & 7, xd, xqs);
    }
    trace_mark(a.trace, a.trace_seq, 7);  // quantized
  }
}

// Epilogue of `nrows` consecutive rows starting at row0, run by one whole
// warp; lane i < nrows holds the value of row row0 + i (nrows even, so the
// adjacent pairs of RoPE and of the up/gate interleave stay in one warp).
template <int EPI>
__device__ __forceinline__ void mv_epilogue(const MatvecArgs& a, int row0, int nrows,
                                            float v, int lane, float& best_v,
                                            int& best_i, size_t push_off,
                                            unsigned push_e) {
  const int row = row0 + lane;
  const bool live = lane < nrows && row < a.w.rows;
  if constexpr (EPI == EPI_PUSH) {
    // push_off: this rank's slot of this phase's parity in every receive
    // buffer, push_e: the phase's epoch (both computed once per thread)
    if (live && row >= a.row_lo && row < a.row_hi) {
      const TpExchange& t = a.tp_out;
      const unsigned long long word = ((unsigned long long)push_e << 32) | __float_as_uint(v);
      const size_t off = push_off + row;
#pragma unroll
      for (int r = 0; r < MAX_WORLD; ++r)
        if (r < t.world) st_relaxed_sys_u64(t.recv[r] + off, word);
    }
  } else if constexpr (EPI == EPI_STORE) {
    if (live && row >= a.row_lo && row < a.row_hi) a.out[row] = v;
  } else if constexpr (EPI == EPI_QKV) {
    const float v1 = __shfl_down_sync(0xffffffffu, v, 1);
    if (live && !(lane & 1)) {
      float x0 = v, x1 = v1;
      const int hd = a.head_dim;
      const int pos = a.io[1];
      const bool is_q = row < a.nq;
      const bool is_k = !is_q && row < a.nq + a.nkv;
      if (is_q || is_k) {
        // RoPE on the adjacent pair, rope.go:39-52
        const int d = (is_q ? row : row - a.nq) % hd;
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
        *reinterpret_cast<float2*>(a.out + row) = make_float2(x0, x1);
      } else {
        // KV append at this position, infer.go:122-127
        const int r2 = is_k ? row - a.nq : row - a.nq - a.nkv;
        const int kvh = r2 / hd, d = r2 % hd;
        const size_t off = (is_k ? 0 : hd) + d;
        uint8_t* base = kv_row(a.kv, a.layer, kvh, pos);
        if (a.kv_f16)
          *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + off) =
              __floats2half2_rn(x0, x1);
        else
          *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + off) =
              make_float2(x0, x1);
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // rows interleave (up_i, gate_i); act_i = silu(gate_i) * up_i,
    // infer.go:228-230
    const float gate = __shfl_down_sync(0xffffffffu, v, 1);
    if (live && !(lane & 1)) a.out[row >> 1] = __fmul_rn(silu_ref(gate), v);
  } else {  // EPI_LOGITS
    if (live && a.out) a.out[row] = v;
    float bv = live ? v : -INFINITY;
    int bi = live ? row : 0x7fffffff;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bv > best_v || (bv == best_v && bi < best_i)) {
      best_v = bv;
      best_i = bi;
    }
  }
}

// Batch-1 Q8_0 matvec, out[r] = sum_b d_w[r,b]*d_x[b] * sum_i q_w[r,b,i]*q_x[b,i]
// (matvec_q8_c, simd.c:33-110), with a fused prologue producing the int8
// activation and a fused epilogue consuming the row results.
//
// Schedule: CTA b takes row groups b, b + grid, b + 2*grid, ...; a tile is
// ~32 KB (one bulk copy: the per-copy cost of the TMA path makes small copies
// slow) and the ring holds ~3 of them.  Warp w owns rows [w*RPW, w*RPW+RPW)
// of every tile, loads each activation chunk once for all of them, and
// finishes those rows itself; with RPW == 1 the pairs of the RoPE and SwiGLU
// epilogues span two warps, so the last warp to post its row of a group runs
// the epilogue of the whole group (fixed order, no CTA barrier).
template <int PRO, int EPI, int RPW, int VK>
__global__ void __launch_bounds__(NTHREADS, 2)  // two CTAs per SM (PDL overlap)
    k_matvec(const __grid_constant__ MatvecArgs a) {
  L3G_DYNAMIC_SMEM(smem);
  MatvecSmem* sh = reinterpret_cast<MatvecSmem*>(smem);
  const int C = a.w.cols;
  float* xd = reinterpret_cast<float*>(smem + MV_HEAD);
  int8_t* xqs = reinterpret_cast<int8_t*>(smem + MV_HEAD + align_up(C / 32 * 4, 128));
  uint8_t* ring = smem + MV_HEAD + align_up(C / 32 * 4, 128) + align_up(C, 128);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.nstages;
  const int wr = a.w.wr, ck = a.w.ck, nsl = a.w.nslices, tb = a.w.tile_bytes;

  // row groups covering [row_lo, row_hi), dealt round-robin over the grid
  const int gl = a.row_lo / wr;
  const int ng = (a.row_hi + wr - 1) / wr - gl;
  const int G = (int)gridDim.x, b = (int)blockIdx.x;
  const int my_groups = b < ng ? (ng - b + G - 1) / G : 0;
  const int ntiles = my_groups * nsl;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], NW);
    }
    for (int s = 0; s < RED_SLOTS; ++s) sh->cnt[s] = 0;
    sh->abort_flag = 0;
    sh->issued = 0;
    sh->producer_done = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  trace_mark(a.trace, a.trace_seq, TR_ENTRY);

  if (warp == NW) {  // producer: weights never depend on the previous kernel
    if (lane == 0) {
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % ns;
        if (t >= ns &&
            !mbar_wait(&sh->empty[s], ((t / ns) - 1) & 1, &sh->abort_flag, a.res, 1, a.wait_ns))
          break;
        const int g = gl + b + (t / nsl) * G;
        const uint8_t* src = a.w.data + ((size_t)g * nsl + (t % nsl)) * tb;
        mbar_arrive_expect_tx(&sh->full[s], tb);
        bulk_g2s(ring + (size_t)s * tb, src, tb, &sh->full[s]);
        *(volatile int*)&sh->issued = t + 1;
      }
      *(volatile int*)&sh->producer_done = 1;
    }
    return;
  }

  // the norm weights are constants: fetch them before the dependency wait
  float4 nw[PRO == PRO_RMS ? VK : 1];
#pragma unroll
  for (int k = 0; k < (PRO == PRO_RMS ? VK : 1); ++k) {
    const int i = threadIdx.x + k * NW * 32;
    nw[k] = (PRO == PRO_RMS && i < C / 4) ? reinterpret_cast<const float4*>(a.norm_w)[i]
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // warm the translations of the activation inputs (one line per warp
  // spread over each vector) while the previous kernel still runs
  if (lane == 0) {
    if constexpr (PRO == PRO_PREQ) {
      touch_page(a.xqs_in + (size_t)warp * (C / NW));
      touch_page(a.xd_in + (size_t)warp * (C / 32 / NW));
    } else {
      touch_page(a.x_in + (size_t)warp * (C / NW));
      if (PRO == PRO_RMS && a.y_in) touch_page(a.y_in + (size_t)warp * (C / NW));
    }
  }
  pdl_wait();  // activations come from the previous kernel
  trace_mark(a.trace, a.trace_seq, TR_WAITED);
  // EPI_PUSH: the phase's epoch and this rank's slot of its parity
  size_t push_off = 0;
  unsigned push_e = 0;
  if constexpr (EPI == EPI_PUSH) {
    push_e = tp_epoch(a.tp_out);
    push_off = (size_t)((push_e & 1u) * a.tp_out.world + a.tp_out.rank) * a.tp_out.n;
  }
  mv_prologue<PRO, VK>(a, xd, xqs, sh, nw);
  consumer_sync();
  trace_mark(a.trace, a.trace_seq, TR_PROLOGUE);

  const int nchunks = ck >> 4;
  const int nbk = ck >> 5;
  float acc[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = 0.0f;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % ns;
    // warp-uniform; after an abort the tile is neither used nor released (no
    // copy can then be issued into a slot whose previous copy may be in flight)
    const bool ok = __all_sync(0xffffffffu,
                               mbar_wait(&sh->full[s], (t / ns) & 1, &sh->abort_flag, a.res, 2, a.wait_ns));
    if (!ok) break;
    const int slice = t % nsl;
    {
      const uint8_t* tile = ring + (size_t)s * tb;
      const uint8_t* wq = tile + (size_t)warp * RPW * ck;
      const __half* wd = reinterpret_cast<const __half*>(tile + (size_t)wr * ck) + warp * RPW * nbk;
      const int8_t* xq = xqs + slice * ck;
      const float* xs = xd + slice * nbk;
#pragma unroll 2
      for (int c = lane; c < nchunks; c += 32) {
        const int4 x4 = *reinterpret_cast<const int4*>(xq + c * 16);
        const float sx = xs[c >> 1];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const int4 w4 = *reinterpret_cast<const int4*>(wq + (size_t)r * ck + c * 16);
          int isum = __dp4a(w4.x, x4.x, 0);
          isum = __dp4a(w4.y, x4.y, isum);
          isum = __dp4a(w4.z, x4.z, isum);
          isum = __dp4a(w4.w, x4.w, isum);
          acc[r] = fmaf((float)isum, __half2float(wd[r * nbk + (c >> 1)]) * sx, acc[r]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[s]);
    if (slice == nsl - 1) {
      const int k = t / nsl;
      const int g = gl + b + k * G;
      float v = 0.0f;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const float sr = warp_sum(acc[r]);
        if (lane == r) v = sr;
        acc[r] = 0.0f;
      }
      if constexpr (RPW >= 2) {
        mv_epilogue<EPI>(a, g * wr + warp * RPW, RPW, v, lane, best_v, best_i, push_off, push_e);
      } else {
        const int slot = k % RED_SLOTS;
        int old = 0;
        if (lane == 0) {
          sh->red[slot][warp] = v;
          __threadfence_block();
          old = atomicAdd(&sh->cnt[slot], 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == NW - 1) {  // every warp has posted its row: finish the group
          __threadfence_block();
          const float vv = lane < NW ? sh->red[slot][lane] : 0.0f;
          __syncwarp();
          if (lane == 0) sh->cnt[slot] = 0;
          mv_epilogue<EPI>(a, g * wr, NW, vv, lane, best_v, best_i, push_off, push_e);
        }
      }
    }
  }
  trace_mark(a.trace, a.trace_seq, TR_LOOP);

  if constexpr (EPI == EPI_LOGITS) {
    // per-warp best -> per-CTA best -> the last CTA merges in a fixed order
    if (lane == 0) {
      sh->best_v[warp] = best_v;
      sh->best_i[warp] = best_i;
    }
    consumer_sync();
    if (warp == 0) {
      float bv = lane < NW ? sh->best_v[lane] : -INFINITY;
      int bi = lane < NW ? sh->best_i[lane] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        a.am_val[blockIdx.x] = bv;
        a.am_idx[blockIdx.x] = bi;
        __threadfence();
        const unsigned prev = atomicAdd(a.am_counter, 1u);
        sh->last = prev == gridDim.x - 1;
      }
      __syncwarp();
      if (*(volatile int*)&sh->last) {
        __threadfence();
        bv = -INFINITY;
        bi = 0x7fffffff;
        for (int i = lane; i < (int)gridDim.x; i += 32) {
          const float v = __ldcg(a.am_val + i);
          const int id = __ldcg(a.am_idx + i);
          if (v > bv || (v == bv && id < bi)) {
            bv = v;
            bi = id;
          }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          a.res->token = bi + a.row_offset;
          a.res->logit = bv;
          *a.am_counter = 0u;
        }
      }
    }
  }

  // After an abort: wait (bounded) until the producer has stopped issuing,
  // then for the last copy issued to each ring slot (earlier copies to a
  // slot were consumed before it was refilled).
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const uint64_t t_start = gtime();
    while (!*(volatile int*)&sh->producer_done && gtime() - t_start < 100000000ull) {
    }
    const int issued = *(volatile int*)&sh->issued;
    for (int s2 = 0; s2 < ns && s2 < issued; ++s2) {
      const int t = s2 + ((issued - 1 - s2) / ns) * ns;
      int dummy = 0;
      mbar_wait(&sh->full[s2], (t / ns) & 1, &dummy, a.res, 3, 100000000ull);
    }
  }
  trace_mark(a.trace, a.trace_seq, TR_EXIT);
}

