// Device code of libl3g: the per-token decode kernels for sm_100a.
//
// Every weight-streaming kernel has the same shape: one CTA per SM, one
// producer warp that streams contiguous weight (or KV) tiles from HBM into a
// shared-memory ring with 1-D bulk copies (cp.async.bulk ... mbarrier
// complete_tx), and NW consumer warps that compute from shared memory.  The
// producer starts streaming before griddepcontrol.wait (programmatic
// dependent launch): weights and past KV entries never depend on the previous
// kernel, so the ring fills while the previous kernel drains.  Every wait on
// an mbarrier is bounded (globaltimer); on timeout the kernel records an
// error in the workspace's result word, drains its in-flight copies and
// returns.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace l3g {

constexpr int NW = 8;                   // consumer warps
constexpr int NTHREADS = 32 * (NW + 1); // + one producer warp
constexpr int MAX_STAGES = 8;
constexpr int RING_BYTES = 64 * 1024;   // bytes in flight per CTA
constexpr int TILE_TARGET = 16 * 1024;  // int8 bytes per weight tile
constexpr int MAXG = 8;                 // max query heads per kv head
constexpr unsigned long long WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s

// device error codes (Result::err); Result::where names the wait site
enum { ERR_NONE = 0, ERR_TIMEOUT = 1, ERR_TOKEN = 2 };

struct Result {        // copied to the host at the end of every step
  int32_t token;       // argmax id (greedy)
  float logit;         // its logit
  int32_t err;         // ERR_*
  int32_t where;       // wait site / detail
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)),
               "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b,
                                                      uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b))
               : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 1-D bulk copy global -> this CTA's shared memory; completion is signalled
// as transaction bytes on the mbarrier.  src, dst 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src,
                                         uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// barrier 1: the NW consumer warps only (the producer warp never joins)
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report(Result* res, int code, int where) {
  if (atomicCAS(&res->err, 0, code) == 0) atomicExch(&res->where, where);
}

// Bounded wait for the phase of parity `parity` of mbarrier b.  Returns false
// when the CTA's abort flag is set or when timeout_ns pass; the latter sets
// the abort flag and reports ERR_TIMEOUT at `where`.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity,
                                          volatile int* abort_flag,
                                          Result* res, int where,
                                          unsigned long long timeout_ns =
                                              WAIT_TIMEOUT_NS) {
  if (mbar_test(b, parity)) return true;
  const uint64_t t0 = gtime();
  for (;;) {
    if (mbar_test(b, parity)) return true;
    if (*abort_flag) return false;
    if (gtime() - t0 > timeout_ns) {
      *abort_flag = 1;
      report(res, ERR_TIMEOUT, where);
      return false;
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__host__ __device__ __forceinline__ int align_up(int x, int a) {
  return (x + a - 1) / a * a;
}

// silu, internal/llama/math.go:16-19 (f64 exp, f32 divide)
__device__ __forceinline__ float silu_ref(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, (float)exp(-(double)x)));
}

// One 32-element block of QuantizeQ8_0Into (q8_0.go:36-77), one value per
// lane: scale = maxabs/127 (1e-8 when 0), q = trunc(v/scale +- 0.5) clamped.
// Bit-identical to the reference for identical inputs.
__device__ __forceinline__ void quant_block(float v, int b, int lane,
                                            float* xd, int8_t* xqs) {
  const float m = warp_max(fabsf(v));
  float scale = __fdiv_rn(m, 127.0f);
  if (scale == 0.0f) scale = 1e-8f;
  const float inv = __fdiv_rn(1.0f, scale);
  const float f = __fmul_rn(v, inv);
  int q = f >= 0.0f ? (int)__fadd_rn(f, 0.5f) : (int)__fsub_rn(f, 0.5f);
  q = min(127, max(-128, q));
  xqs[b * 32 + lane] = (int8_t)q;
  if (lane == 0) xd[b] = scale;
}

// ---------------------------------------------------------------------------
// Repacked Q8_0 matrix.  Rows are grouped by `wr` and columns sliced by `ck`;
// tile (g, s) holds rows [g*wr, g*wr+wr) x cols [s*ck, s*ck+ck):
//   int8 q[wr][ck] followed by fp16 d[wr][ck/32], padded to 16 bytes.
// Tiles are stored g-major, so a CTA's row groups are one contiguous run of
// bytes that a single bulk-copy stream walks in order.
// ---------------------------------------------------------------------------
struct Q8Tiles {
  const uint8_t* data;
  int rows, cols, wr, ck, nslices, tile_bytes, n_groups;
};

enum Pro { PRO_PREQ = 0, PRO_QUANT = 1, PRO_RMS = 2 };
enum Epi { EPI_STORE = 0, EPI_QKV = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

struct MatvecArgs {
  Q8Tiles w;
  int nstages;
  int row_lo, row_hi;  // rows this launch covers / writes
  // prologue
  const float* x_in;    // PRO_QUANT: vector to quantize; PRO_RMS: residual
  const float* y_in;    // PRO_RMS: delta added to x_in first (or null)
  const float* norm_w;  // PRO_RMS
  float* x_out;         // PRO_RMS: x_in + y_in written by CTA 0 (or null)
  float eps;
  const float* xd_in;   // PRO_PREQ: pre-quantized activation (device)
  const int8_t* xqs_in;
  // epilogue
  float* out;
  // EPI_QKV: rows are [q | k | v] of this rank's heads
  int nq, nkv, head_dim, rope_half, ctx, kv_f16;
  const float* rope_cos;  // [ctx][rope_half]
  const float* rope_sin;
  const int* io;          // io[0] token, io[1] position
  void* kc;               // this layer's K cache [kv heads][ctx][hd]
  void* vc;
  // EPI_LOGITS: fused argmax
  int row_offset;         // vocab id of local row 0
  float* am_val;          // [gridDim.x] per-CTA best
  int* am_idx;
  unsigned* am_counter;   // zero between launches
  Result* res;            // error word, argmax result
};

struct MatvecSmem {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  float red[2][NW];
  float ssred[NW];
  int abort_flag;
  int issued;
  int last;
};
constexpr int MV_HEAD = 256;
static_assert(sizeof(MatvecSmem) <= MV_HEAD, "matvec smem head");

__host__ __device__ __forceinline__ int mv_smem_bytes(int cols, int nstages,
                                                      int tile_bytes) {
  return MV_HEAD + align_up(cols / 32 * 4, 128) + align_up(cols, 128) +
         nstages * tile_bytes;
}

template <int PRO>
__device__ __forceinline__ void mv_prologue(const MatvecArgs& a, float* xd,
                                            int8_t* xqs, MatvecSmem* sh) {
  const int C = a.w.cols;
  const int nb = C >> 5;
  const int tid = threadIdx.x;  // < NW*32
  const int warp = tid >> 5, lane = tid & 31;
  if constexpr (PRO == PRO_PREQ) {
    for (int i = tid; i < nb; i += NW * 32) xd[i] = a.xd_in[i];
    for (int i = tid * 16; i < C; i += NW * 32 * 16)
      *reinterpret_cast<int4*>(xqs + i) =
          *reinterpret_cast<const int4*>(a.xqs_in + i);
  } else if constexpr (PRO == PRO_QUANT) {
    for (int b = warp; b < nb; b += NW) quant_block(a.x_in[b * 32 + lane], b, lane, xd, xqs);
  } else {
    // residual add (infer.go:189-191 / :244-246) then rmsNorm (math.go:5-14)
    float ss = 0.0f;
    const bool wx = a.x_out != nullptr && blockIdx.x == 0;
    for (int i = tid; i < C; i += NW * 32) {
      float v = a.x_in[i];
      if (a.y_in) v = __fadd_rn(v, a.y_in[i]);
      if (wx) a.x_out[i] = v;
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) sh->ssred[warp] = ss;
    consumer_sync();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += sh->ssred[w];
    const float scale =
        (float)(1.0 / sqrt((double)__fadd_rn(__fdiv_rn(tot, (float)C), a.eps)));
    for (int b = warp; b < nb; b += NW) {
      const int i = b * 32 + lane;
      float v = a.x_in[i];
      if (a.y_in) v = __fadd_rn(v, a.y_in[i]);
      quant_block(__fmul_rn(__fmul_rn(v, scale), a.norm_w[i]), b, lane, xd, xqs);
    }
  }
}

// Epilogue of one row group, run by warp 0; lanes < wr hold one row each.
template <int EPI>
__device__ __forceinline__ void mv_epilogue(const MatvecArgs& a, int g,
                                            float v, int lane, float& best_v,
                                            int& best_i) {
  const int wr = a.w.wr;
  const int row = g * wr + lane;
  const bool live = lane < wr && row < a.w.rows;
  if constexpr (EPI == EPI_STORE) {
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
        const size_t off = ((size_t)kvh * a.ctx + pos) * hd + d;
        void* base = is_k ? a.kc : a.vc;
        if (a.kv_f16)
          *reinterpret_cast<__half2*>(static_cast<__half*>(base) + off) =
              __floats2half2_rn(x0, x1);
        else
          *reinterpret_cast<float2*>(static_cast<float*>(base) + off) =
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
template <int PRO, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_matvec(const __grid_constant__ MatvecArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  MatvecSmem* sh = reinterpret_cast<MatvecSmem*>(smem);
  const int C = a.w.cols;
  float* xd = reinterpret_cast<float*>(smem + MV_HEAD);
  int8_t* xqs = reinterpret_cast<int8_t*>(smem + MV_HEAD + align_up(C / 32 * 4, 128));
  uint8_t* ring = smem + MV_HEAD + align_up(C / 32 * 4, 128) + align_up(C, 128);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.nstages;
  const int wr = a.w.wr, ck = a.w.ck, nsl = a.w.nslices, tb = a.w.tile_bytes;

  // contiguous, balanced share of the row groups covering [row_lo, row_hi)
  const int gl = a.row_lo / wr;
  const int ng = (a.row_hi + wr - 1) / wr - gl;
  const int g0 = gl + (int)((long long)blockIdx.x * ng / gridDim.x);
  const int g1 = gl + (int)((long long)(blockIdx.x + 1) * ng / gridDim.x);
  const int ntiles = (g1 - g0) * nsl;
  const uint8_t* src = a.w.data + (size_t)g0 * nsl * tb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], NW);
    }
    sh->abort_flag = 0;
    sh->issued = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == NW) {  // producer: weights never depend on the previous kernel
    if (lane == 0) {
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % ns;
        if (t >= ns &&
            !mbar_wait(&sh->empty[s], ((t / ns) - 1) & 1, &sh->abort_flag, a.res, 1))
          break;
        mbar_arrive_expect_tx(&sh->full[s], tb);
        bulk_g2s(ring + (size_t)s * tb, src + (size_t)t * tb, tb, &sh->full[s]);
        *(volatile int*)&sh->issued = t + 1;
      }
    }
    return;
  }

  pdl_wait();  // activations come from the previous kernel
  mv_prologue<PRO>(a, xd, xqs, sh);
  consumer_sync();

  const int r_in = warp % wr, part = warp / wr, nparts = NW / wr;
  const int nchunks = ck >> 4;
  float acc = 0.0f;
  int gpar = 0;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  int consumed = 0;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % ns;
    const bool ok = mbar_wait(&sh->full[s], (t / ns) & 1, &sh->abort_flag, a.res, 2);
    const int slice = t % nsl;
    if (ok) {
      consumed = t + 1;
      const uint8_t* tile = ring + (size_t)s * tb;
      const uint8_t* wq = tile + r_in * ck;
      const __half* wd = reinterpret_cast<const __half*>(tile + wr * ck) + r_in * (ck >> 5);
      const int8_t* xq = xqs + slice * ck;
      const float* xs = xd + slice * (ck >> 5);
#pragma unroll 4
      for (int c = part * 32 + lane; c < nchunks; c += nparts * 32) {
        const int4 w4 = *reinterpret_cast<const int4*>(wq + c * 16);
        const int4 x4 = *reinterpret_cast<const int4*>(xq + c * 16);
        int isum = __dp4a(w4.x, x4.x, 0);
        isum = __dp4a(w4.y, x4.y, isum);
        isum = __dp4a(w4.z, x4.z, isum);
        isum = __dp4a(w4.w, x4.w, isum);
        acc = fmaf((float)isum, __half2float(wd[c >> 1]) * xs[c >> 1], acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[s]);
    if (slice == nsl - 1) {
      acc = warp_sum(acc);
      if (lane == 0) sh->red[gpar][warp] = acc;
      consumer_sync();
      if (warp == 0) {
        float v = 0.0f;
        if (lane < wr)
          for (int p = 0; p < nparts; ++p) v += sh->red[gpar][lane + p * wr];
        mv_epilogue<EPI>(a, g0 + t / nsl, v, lane, best_v, best_i);
      }
      gpar ^= 1;
      acc = 0.0f;
    }
  }

  if constexpr (EPI == EPI_LOGITS) {
    // per-CTA best, then the last CTA to finish merges in a fixed order
    if (warp == 0) {
      if (lane == 0) {
        a.am_val[blockIdx.x] = best_v;
        a.am_idx[blockIdx.x] = best_i;
        __threadfence();
        const unsigned prev = atomicAdd(a.am_counter, 1u);
        sh->last = prev == gridDim.x - 1;
      }
      __syncwarp();
      if (*(volatile int*)&sh->last) {
        __threadfence();
        float bv = -INFINITY;
        int bi = 0x7fffffff;
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

  // after an abort, wait (bounded) for copies still in flight to this ring
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const int issued = *(volatile int*)&sh->issued;
    for (int t = consumed; t < issued; ++t) {
      int dummy = 0;
      mbar_wait(&sh->full[t % ns], (t / ns) & 1, &dummy, a.res, 3, 100000000ull);
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K GQA attention over the HBM KV cache (infer.go:130-175).
// Grid (kv heads, splits).  CTA (g, s) takes a contiguous range of positions
// of kv head g for all `group` query heads sharing it, streams K and V rows
// through the shared-memory ring and keeps an online softmax per warp.  The
// last CTA of each kv head merges the splits in split order (deterministic).
// ---------------------------------------------------------------------------
struct AttnArgs {
  const float* q;     // [local q heads][hd], roped
  const void* kc;     // this layer [local kv heads][ctx][hd]
  const void* vc;
  int ctx, hd, group, n_splits, P, nstages, stage_bytes;
  float scale;        // float32(1/sqrt(hd)), infer.go:130
  const int* io;      // io[1] = position of this token
  float* part_o;      // [kv heads][splits][group][hd]
  float* part_ml;     // [kv heads][splits][group][2]
  unsigned* counters; // [kv heads], zero between launches
  float* out;         // [local q heads][hd]
  Result* res;
};

struct AttnSmem {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  int abort_flag;
  int issued;
  int last;
};
constexpr int AT_HEAD = 256;
static_assert(sizeof(AttnSmem) <= AT_HEAD, "attn smem head");

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
#pragma unroll
      for (int j = 0; j < DPL; ++j) v[j] = reinterpret_cast<const float*>(p)[j];
    }
  } else {
    const __half* h = reinterpret_cast<const __half*>(p);
#pragma unroll
    for (int j = 0; j < DPL; j += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(h + j));
      v[j] = f.x;
      if (j + 1 < DPL) v[j + 1] = f.y;
    }
  }
}

template <int DPL, typename KT>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attention(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  AttnSmem* sh = reinterpret_cast<AttnSmem*>(smem);
  uint8_t* ring = smem + AT_HEAD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, split = blockIdx.y, S = a.n_splits;
  const int hd = a.hd, G = a.group, ns = a.nstages, P = a.P;
  const int pos = a.io[1];  // written by the step's host copy, not a kernel
  const int n = pos + 1;
  const int chunk = align_up((n + S - 1) / S, P);
  const int t0 = min(n, split * chunk), t1 = min(n, t0 + chunk);
  const int nst = (t1 - t0 + P - 1) / P;
  const size_t head_off = (size_t)kvh * a.ctx * hd;
  const int half_stage = a.stage_bytes / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], NW);
    }
    sh->abort_flag = 0;
    sh->issued = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == NW) {
    if (lane == 0) {
      bool waited = false;
      for (int st = 0; st < nst; ++st) {
        const int s = st % ns;
        if (st >= ns &&
            !mbar_wait(&sh->empty[s], ((st / ns) - 1) & 1, &sh->abort_flag, a.res, 4))
          break;
        const int ta = t0 + st * P, tb = min(t1, ta + P);
        // past positions are immutable: only the stage holding this step's
        // own K/V (written by the QKV kernel) waits for the previous grid
        if (!waited && tb > pos) {
          pdl_wait();
          waited = true;
        }
        const uint32_t bytes = (uint32_t)((tb - ta) * hd * sizeof(KT));
        const size_t off = (head_off + (size_t)ta * hd) * sizeof(KT);
        mbar_arrive_expect_tx(&sh->full[s], 2 * bytes);
        bulk_g2s(ring + (size_t)s * a.stage_bytes,
                 static_cast<const uint8_t*>(a.kc) + off, bytes, &sh->full[s]);
        bulk_g2s(ring + (size_t)s * a.stage_bytes + half_stage,
                 static_cast<const uint8_t*>(a.vc) + off, bytes, &sh->full[s]);
        *(volatile int*)&sh->issued = st + 1;
      }
    }
    return;
  }

  pdl_wait();  // q comes from the previous kernel
  float q[MAXG][DPL];
#pragma unroll
  for (int h = 0; h < MAXG; ++h)
#pragma unroll
    for (int j = 0; j < DPL; ++j)
      q[h][j] = h < G ? a.q[((size_t)kvh * G + h) * hd + lane * DPL + j] : 0.0f;
  float m[MAXG], l[MAXG], o[MAXG][DPL];
#pragma unroll
  for (int h = 0; h < MAXG; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[h][j] = 0.0f;
  }

  int consumed = 0;
  for (int st = 0; st < nst; ++st) {
    const int s = st % ns;
    const bool ok = mbar_wait(&sh->full[s], (st / ns) & 1, &sh->abort_flag, a.res, 5);
    if (ok) {
      consumed = st + 1;
      const int ta = t0 + st * P, cnt = min(t1, ta + P) - ta;
      const KT* Ks = reinterpret_cast<const KT*>(ring + (size_t)s * a.stage_bytes);
      const KT* Vs = reinterpret_cast<const KT*>(ring + (size_t)s * a.stage_bytes + half_stage);
      for (int p = warp; p < cnt; p += NW) {
        float kv[DPL], vv[DPL];
        load_row<DPL, KT>(Ks + (size_t)p * hd + lane * DPL, kv);
        load_row<DPL, KT>(Vs + (size_t)p * hd + lane * DPL, vv);
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
          if (h < G) {
            float d = 0.0f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) d = fmaf(q[h][j], kv[j], d);
            const float sc = warp_sum(d) * a.scale;
            const float mn = fmaxf(m[h], sc);
            const float corr = expf(m[h] - mn);
            const float pr = expf(sc - mn);
            l[h] = fmaf(l[h], corr, pr);
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[h][j] = fmaf(o[h][j], corr, pr * vv[j]);
            m[h] = mn;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[s]);
  }

  // drain after an abort, then reuse the ring as scratch
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const int issued = *(volatile int*)&sh->issued;
    for (int t = consumed; t < issued; ++t) {
      int dummy = 0;
      mbar_wait(&sh->full[t % ns], (t / ns) & 1, &dummy, a.res, 6, 100000000ull);
    }
  }
  consumer_sync();
  float* sm_ml = reinterpret_cast<float*>(ring);        // [NW][G][2]
  float* sm_o = sm_ml + NW * MAXG * 2;                  // [NW][G][hd]
  // (the host sizes the ring to hold this scratch)
#pragma unroll
  for (int h = 0; h < MAXG; ++h) {
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
  const size_t pbase = ((size_t)kvh * S + split) * G;
  for (int idx = threadIdx.x; idx < G * hd; idx += NW * 32) {
    const int h = idx / hd, d = idx % hd;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_ml[(w * MAXG + h) * 2]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < NW; ++w) {
        const float mw = sm_ml[(w * MAXG + h) * 2];
        if (mw == -INFINITY) continue;
        const float e = expf(mw - M);
        L = fmaf(sm_ml[(w * MAXG + h) * 2 + 1], e, L);
        O = fmaf(sm_o[((size_t)w * G + h) * hd + d], e, O);
      }
    }
    a.part_o[(pbase + h) * hd + d] = O;
    if (d == 0) {
      a.part_ml[(pbase + h) * 2] = M;
      a.part_ml[(pbase + h) * 2 + 1] = L;
    }
  }
  __threadfence();
  consumer_sync();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counters + kvh, 1u);
    sh->last = prev == (unsigned)S - 1;
  }
  consumer_sync();
  if (!*(volatile int*)&sh->last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < G * hd; idx += NW * 32) {
    const int h = idx / hd, d = idx % hd;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s)
      M = fmaxf(M, __ldcg(a.part_ml + (((size_t)kvh * S + s) * G + h) * 2));
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < S; ++s) {
      const size_t pb = ((size_t)kvh * S + s) * G + h;
      const float ms = __ldcg(a.part_ml + pb * 2);
      if (ms == -INFINITY) continue;
      const float e = expf(ms - M);
      L = fmaf(__ldcg(a.part_ml + pb * 2 + 1), e, L);
      O = fmaf(__ldcg(a.part_o + pb * hd + d), e, O);
    }
    a.out[((size_t)kvh * G + h) * hd + d] = __fmul_rn(O, __fdiv_rn(1.0f, L));
  }
  if (threadIdx.x == 0) a.counters[kvh] = 0u;
}

// ---------------------------------------------------------------------------
// Embedding row dequant (infer.go:513-518, tensor_read.go:128-147) from the
// raw GGUF Q8_0 rows: x[i] = f16(d) * q[i].
// ---------------------------------------------------------------------------
__global__ void k_embed(const uint8_t* emb, int vocab, int cols, const int* io,
                        float* x, Result* res) {
  pdl_launch_dependents();
  pdl_wait();
  const int token = io[0];
  if (token < 0 || token >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(res, ERR_TOKEN, token);
    return;
  }
  const uint8_t* row = emb + (size_t)token * (cols / 32) * 34;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
    const uint8_t* blk = row + (size_t)(i >> 5) * 34;
    const unsigned short bits = (unsigned short)(blk[0] | (blk[1] << 8));
    const float d = __half2float(__ushort_as_half(bits));
    x[i] = __fmul_rn(d, (float)(int8_t)blk[2 + (i & 31)]);
  }
}

// End of a device-fed greedy step: record the argmax and make it the next
// step's token at the next position (io = {token, pos, step}).
__global__ void k_advance(int* io, const Result* res, int* tokens) {
  pdl_wait();
  if (threadIdx.x == 0) {
    const int t = res->token;
    tokens[io[2]] = t;
    io[0] = t;
    io[1] += 1;
    io[2] += 1;
  }
}

// Standalone activation quantization (QuantizeQ8_0Into), one warp per block.
__global__ void k_quantize(const float* x, int n, float* d, int8_t* qs) {
  const int lane = threadIdx.x & 31;
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (b >= (n + 31) / 32) return;
  const int i = b * 32 + lane;
  quant_block(i < n ? x[i] : 0.0f, b, lane, d, qs);
}

// ---------------------------------------------------------------------------
// Top-K selection over logits: 64-bit keys (ordered float bits, ~index) so a
// descending sort gives larger logits first and lower ids first on ties.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t topk_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)u << 32) | (uint32_t)(~(uint32_t)idx);
}
__device__ __forceinline__ float key_value(uint64_t k) {
  uint32_t u = (uint32_t)(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}
__device__ __forceinline__ int key_index(uint64_t k) {
  return (int)(~(uint32_t)k);
}

__device__ void bitonic_desc(uint64_t* keys, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = keys[i], y = keys[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
}

constexpr int TOPK_CHUNK = 2048;
// Phase 1: each CTA sorts one chunk of logits and keeps its best k keys.
__global__ void k_topk_partial(const float* logits, int n, int k, int id_offset,
                               uint64_t* part) {
  __shared__ uint64_t keys[TOPK_CHUNK];
  pdl_wait();
  const int base = blockIdx.x * TOPK_CHUNK;
  for (int i = threadIdx.x; i < TOPK_CHUNK; i += blockDim.x) {
    const int r = base + i;
    keys[i] = r < n ? topk_key(logits[r], r + id_offset) : 0ull;
  }
  __syncthreads();
  bitonic_desc(keys, TOPK_CHUNK);
  for (int i = threadIdx.x; i < k; i += blockDim.x)
    part[(size_t)blockIdx.x * k + i] = keys[i];
}
// Phase 2: one CTA merges all partial keys (count <= cap, cap a power of 2).
__global__ void k_topk_final(const uint64_t* part, int count, int cap, int k,
                             int* out_ids, float* out_logits) {
  extern __shared__ uint64_t keys2[];
  pdl_wait();
  for (int i = threadIdx.x; i < cap; i += blockDim.x)
    keys2[i] = i < count ? part[i] : 0ull;
  __syncthreads();
  bitonic_desc(keys2, cap);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    out_ids[i] = key_index(keys2[i]);
    out_logits[i] = key_value(keys2[i]);
  }
}

// ---------------------------------------------------------------------------
// Load-time repack: GGUF Q8_0 rows (34-byte blocks, already on the device)
// into the tiled layout.  Destination row r takes source row map(r):
// concatenation of up to three row ranges, or the interleave (a_i, b_i).
// Values are copied unchanged.
// ---------------------------------------------------------------------------
struct RepackArgs {
  const uint8_t* src[3];
  int src_row0[3];
  int seg_rows[3];
  int nseg;
  int interleave2;        // dst 2i <- seg0 row i, dst 2i+1 <- seg1 row i
  int src_blocks;         // blocks per source row
  int blk0;               // first source block of the column slice
  Q8Tiles dst;            // rows/cols of the destination
  uint8_t* out;
};

__global__ void k_repack(const __grid_constant__ RepackArgs a) {
  const int nbc = a.dst.cols / 32;
  const long long total = (long long)a.dst.n_groups * a.dst.wr * nbc;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / nbc), b = (int)(e % nbc);
    const int g = r / a.dst.wr, i = r % a.dst.wr;
    const int bpt = a.dst.ck / 32;
    const int s = b / bpt, bb = b % bpt;
    uint8_t* tile = a.out + ((size_t)g * a.dst.nslices + s) * a.dst.tile_bytes;
    uint8_t* qd = tile + (size_t)i * a.dst.ck + bb * 32;
    uint8_t* dd = tile + (size_t)a.dst.wr * a.dst.ck + ((size_t)i * bpt + bb) * 2;
    const uint8_t* blk = nullptr;
    if (r < a.dst.rows) {
      int seg = 0, sr = r;
      if (a.interleave2) {
        seg = r & 1;
        sr = r >> 1;
      } else {
        while (seg < a.nseg - 1 && sr >= a.seg_rows[seg]) sr -= a.seg_rows[seg++];
      }
      blk = a.src[seg] + ((size_t)(a.src_row0[seg] + sr) * a.src_blocks + a.blk0 + b) * 34;
    }
    if (blk) {
      dd[0] = blk[0];
      dd[1] = blk[1];
#pragma unroll 8
      for (int j = 0; j < 32; ++j) qd[j] = blk[2 + j];
    } else {
      dd[0] = 0;
      dd[1] = 0;
      for (int j = 0; j < 32; ++j) qd[j] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Failure-detection self test: a bounded wait on an mbarrier that nothing
// completes must give up and report ERR_TIMEOUT.
// ---------------------------------------------------------------------------
__global__ void k_selftest_wait(Result* res, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, res, 99, timeout_ns);
}

}  // namespace l3g
