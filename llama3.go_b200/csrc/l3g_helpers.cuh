// Device helpers shared by the kernels (included inside namespace l3g, after
// l3g_ptx.cuh): tracing, error reporting, bounded mbarrier waits, warp
// reductions and the Q8_0 activation quantization of QuantizeQ8_0Into.
#pragma once

// Device timeline (off when tr == nullptr): thread 0 of every CTA (up to
// TRACE_CTAS per launch) stamps %globaltimer at a few points; launch `seq` of
// the step owns tr[(seq * TRACE_CTAS + cta) * 8 + event].
enum { TR_ENTRY = 0, TR_WAITED = 1, TR_PROLOGUE = 2, TR_LOOP = 3, TR_EXIT = 4 };
constexpr int TRACE_CTAS = 256;
__device__ __forceinline__ void trace_mark(unsigned long long* tr, int seq, int ev) {
  if (tr == nullptr || threadIdx.x != 0) return;
  const unsigned lin = blockIdx.x + blockIdx.y * gridDim.x;
  if (lin >= (unsigned)TRACE_CTAS) return;
  tr[((size_t)seq * TRACE_CTAS + lin) * 8 + ev] = gtime();
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
  const float inv = __frcp_rn(scale);
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
  const float inv = __frcp_rn(scale);
  char4 q;
  q.x = quant_one(u.x, inv);
  q.y = quant_one(u.y, inv);
  q.z = quant_one(u.z, inv);
  q.w = quant_one(u.w, inv);
  *reinterpret_cast<char4*>(xqs + blk * 32 + sub * 4) = q;
  if (sub == 0) xd[blk] = scale;
}
