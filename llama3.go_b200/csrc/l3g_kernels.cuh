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

#include "l3g_base.cuh"

// The inline-PTX layer (the kernels above it are plain CUDA C++); a host
// build of the kernels for the CPU checks names its own in L3G_PTX_HEADER.
#ifndef L3G_PTX_HEADER
#include "l3g_ptx.cuh"

#include "l3g_tcgen05.cuh"
#else
#include L3G_PTX_HEADER
#endif

#include "l3g_helpers.cuh"

#include "l3g_matvec.cuh"

#include "l3g_attention.cuh"

#include "l3g_attention_fast.cuh"

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
static __global__ void k_tp_reduce(const TpExchange t, float* y, Result* res,
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
static __global__ void k_embed(const uint8_t* emb, int vocab, int cols, const int* io,
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

static __global__ void k_sample(const int* ids, const float* logits, int k, const SampleParams* sp,
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
static __global__ void k_advance(int* io, const Result* res, int* tokens) {
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
static __global__ void k_quantize(const float* x, int n, float* d, int8_t* qs) {
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

__device__ __forceinline__ void bitonic_step(uint64_t* keys, int i, int j, int k) {
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
// Descending bitonic sort of n keys (a power of two) in shared memory by the
// whole block.  When n is a multiple of the block size and each warp's share
// n / warps a multiple of 32, warp w owns the contiguous segment [w * seg,
// (w + 1) * seg): a step whose partner distance j is below seg pairs keys of
// one segment, so only the warp synchronizes; the few steps with j >= seg
// (log2(warps) per merge level) span the block and take block barriers.
// The keys here are unique, so the result is the same whichever order the
// steps run in.
static __device__ void bitonic_desc(uint64_t* keys, int n) {
  const int T = (int)blockDim.x, W = T >> 5;
  const int seg = n / W;
  if (n % T != 0 || seg % 32 != 0) {
    for (int k = 2; k <= n; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < n; i += T) bitonic_step(keys, i, j, k);
        __syncthreads();
      }
    return;
  }
  const int base = (threadIdx.x >> 5) * seg + (threadIdx.x & 31);
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= seg) {
        __syncthreads();  // the warps' last in-segment steps are done
        for (int i = threadIdx.x; i < n; i += T) bitonic_step(keys, i, j, k);
        __syncthreads();
      } else {
        for (int m = 0; m < seg; m += 32) bitonic_step(keys, base + m, j, k);
        __syncwarp();
      }
    }
  __syncthreads();
}

constexpr int TOPK_CHUNK = 2048;
// Phase 1: each CTA sorts one chunk of logits and keeps its best k keys.
static __global__ void k_topk_partial(const float* logits, int n, int k, int id_offset,
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
static __global__ void k_topk_final(const uint64_t* part, int count, int cap, int k,
                             int* out_ids, float* out_logits) {
  L3G_DYNAMIC_SMEM(keys2_raw);
  uint64_t* keys2 = reinterpret_cast<uint64_t*>(keys2_raw);
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

#include "l3g_repack.cuh"


// ---------------------------------------------------------------------------
// Failure-detection self test: a bounded wait on an mbarrier that nothing
// completes must give up and report ERR_TIMEOUT.
// ---------------------------------------------------------------------------
static __global__ void k_selftest_wait(Result* res, unsigned long long timeout_ns) {
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
