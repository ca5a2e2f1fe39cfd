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

#include "l3g_gemm_layout.h"
#include "l3g_persist_plan.h"

namespace l3g {

constexpr int NW = 8;                   // consumer warps
constexpr int NTHREADS = 32 * (NW + 1); // + one producer warp
constexpr int MAX_STAGES = 16;
// Shared memory per CTA kept under half an SM's 228 KB, so the next kernel's
// CTA (programmatic dependent launch) can be resident and prefetching.
constexpr int CTA_SMEM_SHARE = 112 * 1024;
// Weight tile target: a 1-D bulk copy costs about 0.25 us per copy per CTA
// on top of its bytes, so copies of ~32 KB are needed to approach HBM speed.
constexpr int TILE_TARGET = 32 * 1024;
constexpr int MAXG = 8;                 // max query heads per kv head
constexpr unsigned long long WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s
constexpr int MAX_TOPK = 64;  // largest top-K a workspace serves
// Waits of a tensor-parallel step: a wait can depend, directly or through the
// kernels launched early behind it, on another GPU's progress, which host
// skew between the ranks' processes can delay by more than the local bound.
constexpr unsigned long long WAIT_TIMEOUT_PEER_NS = 30000000000ull;  // 30 s

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
// An L2-only load whose value is discarded, issued before the dependency wait
// on a buffer the previous kernel is still writing: it warms the address
// translation of that buffer's page so the real loads after the wait do not
// pay for it.  `.cg` keeps the (stale) line out of L1, so nothing read after
// the wait can come from it.
__device__ __forceinline__ void touch_page(const void* p) {
  unsigned v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  (void)v;
}
// Device-scope atomic add with acquire-release semantics; returns the old value.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Device-scope acquire load (counters shared by the CTAs of a grid).
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// System-scope acquire load / release store (flags shared across GPUs).
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// System-scope relaxed 64-bit accesses: single-copy atomic, so a {value,
// epoch} word written by another GPU is seen whole or not at all.
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Thread-block cluster helpers (distributed shared memory).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster: release this CTA's shared-memory
// writes, acquire the others'.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The float at the same shared-memory offset as p in CTA `rank` of the cluster.
__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
  return v;
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

// Device timeline (off when tr == nullptr): thread 0 of every CTA (up to
// TRACE_CTAS per launch) stamps %globaltimer at a few points; launch `seq` of
// the step owns tr[(seq * TRACE_CTAS + cta) * 8 + event].
enum { TR_ENTRY = 0, TR_WAITED = 1, TR_PROLOGUE = 2, TR_LOOP = 3, TR_EXIT = 4 };
constexpr int TRACE_CTAS = 256;
__device__ __forceinline__ void trace_mark(unsigned long long* tr, int seq, int ev) {
  if (tr == nullptr || threadIdx.x != 0) return;
  const unsigned lin = blockIdx.x + blockIdx.y * gridDim.x;
  if (lin >= (unsigned)TRACE_CTAS) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  tr[((size_t)seq * TRACE_CTAS + lin) * 8 + ev] = t;
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

// The same block quantization with four consecutive values per lane and the
// eight lanes (lane & 7) of an aligned lane group sharing one 32-value block
// `blk`.  Every lane of the warp must call it (shuffles); lanes with
// live == false only join the shuffles.
__device__ __forceinline__ int8_t quant_one(float v, float inv) {
  const float f = __fmul_rn(v, inv);
  const int q = f >= 0.0f ? (int)__fadd_rn(f, 0.5f) : (int)__fsub_rn(f, 0.5f);
  return (int8_t)min(127, max(-128, q));
}
__device__ __forceinline__ void quant_quad(float4 u, bool live, int blk, int sub, float* xd,
                                           int8_t* xqs) {
  float m = fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w)));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
  if (!live) return;
  float scale = __fdiv_rn(m, 127.0f);
  if (scale == 0.0f) scale = 1e-8f;
  const float inv = __fdiv_rn(1.0f, scale);
  char4 q;
  q.x = quant_one(u.x, inv);
  q.y = quant_one(u.y, inv);
  q.z = quant_one(u.z, inv);
  q.w = quant_one(u.w, inv);
  *reinterpret_cast<char4*>(xqs + blk * 32 + sub * 4) = q;
  if (sub == 0) xd[blk] = scale;
}

#include "l3g_matvec.cuh"

#include "l3g_attention.cuh"

#include "l3g_persist.cuh"

#include "l3g_gemm.cuh"

#include "l3g_prefill.cuh"

// ---------------------------------------------------------------------------
// Tensor-parallel reduction, the receiving half of the exchange (the pushing
// half is the EPI_PUSH epilogue of the Wo / down matvecs): thread i waits for
// elements 4i..4i+3 of every rank's slot of this phase (their epoch words,
// bounded wait) and writes their sum, in rank order, to y.  It replaces the
// reference's single-process residual input (infer.go:189-191, :244-246) in
// a sharded step: y is the full Wo / down output on every rank.
// ---------------------------------------------------------------------------
__global__ void k_tp_reduce(const TpExchange t, float* y, Result* res,
                            unsigned long long wait_ns) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (4 * i >= t.n) return;
  const unsigned e = tp_epoch(t);
  const unsigned long long* rb = t.my_recv + (size_t)(e & 1u) * t.world * t.n + 4 * i;
  const uint64_t t_start = gtime();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < MAX_WORLD; ++r) {
    if (r >= t.world) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      unsigned long long w = ld_relaxed_sys_u64(rb + (size_t)r * t.n + j);
      while ((unsigned)(w >> 32) != e) {
        if (gtime() - t_start > wait_ns) {
          report(res, ERR_TIMEOUT, 8);
          break;
        }
        w = ld_relaxed_sys_u64(rb + (size_t)r * t.n + j);
      }
      const float v = __uint_as_float((unsigned)w);
      acc[j] = r == 0 ? v : __fadd_rn(acc[j], v);
    }
  }
  reinterpret_cast<float4*>(y)[i] = make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// ---------------------------------------------------------------------------
// Embedding row dequant (infer.go:513-518, tensor_read.go:128-147) from the
// raw GGUF Q8_0 rows: x[i] = f16(d) * q[i].
// ---------------------------------------------------------------------------
// It also advances the workspace's step counter (the epoch base of the
// tensor-parallel exchange), once per step on every rank, and, when the step
// runs the persistent layer kernel, zeroes that kernel's nbar barrier,
// abort and handshake words (bar, nullable): every earlier kernel has
// completed by then, so an aborted step leaves no stale count behind.
__global__ void k_embed(const uint8_t* emb, int vocab, int cols, const int* io,
                        float* x, Result* res, unsigned* step, unsigned* bar, int nbar) {
  pdl_launch_dependents();
  pdl_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) *step += 1u;
  if (bar)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nbar; i += gridDim.x * blockDim.x)
      bar[i] = 0u;
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

// ---------------------------------------------------------------------------
// Sampler.SampleTopK (sampling.go:103-143) on the device, after the top-K
// kernels: maxLogit over the items, e_i = exp(float64(l_i - maxLogit) / T)
// in float64, r = U * sum e_i, the first item (in the list's order) whose
// running sum reaches r.  U is a uniform double in [0, 1) from Philox4x32-10
// (Salmon, Moraes, Dror, Shaw, SC 2011) keyed by the caller's seed and
// counted by the draw index (the reference draws from Go's math/rand, whose
// stream is not reproduced).
// ---------------------------------------------------------------------------
struct SampleParams {      // copied from the host before a step
  float temperature;       // > 0
  int32_t pad;
  uint64_t seed;
  uint64_t counter;        // draw index of this step (device-fed loop: + io[2])
  uint64_t pad2;
};

__host__ __device__ inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = (uint32_t)p1;
    c[2] = n2;
    c[3] = (uint32_t)p0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

__global__ void k_sample(const int* ids, const float* logits, int k, const SampleParams* sp,
                         const int* io, Result* res) {
  __shared__ double e[MAX_TOPK];
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x;
  float mx = logits[0];
  for (int i = 1; i < k; ++i) mx = fmaxf(mx, logits[i]);
  const double invT = 1.0 / (double)sp->temperature;
  for (int i = lane; i < k; i += 32) e[i] = exp((double)(logits[i] - mx) * invT);
  __syncwarp();
  if (lane != 0) return;
  double sum = 0.0;
  for (int i = 0; i < k; ++i) sum += e[i];
  const uint64_t ctr = sp->counter + (io ? (uint64_t)io[2] : 0ull);
  uint32_t c[4] = {(uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u};
  philox4x32_10(c, (uint32_t)sp->seed, (uint32_t)(sp->seed >> 32));
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
  res->token = ids[pick];
  res->logit = logits[pick];
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
// QuantizeQ8_0Into (q8_0.go:22-79): one warp per 32-value block.  In the
// decode step it quantizes the SwiGLU output once for every CTA of the down
// matvec (which then only copies the int8 vector), as a dependent launch.
__global__ void k_quantize(const float* x, int n, float* d, int8_t* qs) {
  pdl_launch_dependents();
  pdl_wait();
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

// batched decode (uses the top-K keys and the sampler's Philox above)
#include "l3g_batch.cuh"

}  // namespace l3g
