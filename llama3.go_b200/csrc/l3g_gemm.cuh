// Batched Q8_0 product on the tcgen05 tensor cores (included by
// l3g_kernels.cuh, inside namespace l3g, after l3g_gemm_layout.h and the
// tensor-core helpers of l3g_tcgen05.cuh).
#pragma once

// An int32 block sum (|v| < 2^22: at most 32 * 128 * 128) as fp32, exactly,
// without the conversion unit: the bits of 1.5 * 2^23 + v, minus 1.5 * 2^23
// (the second step is the caller's packed add of -1.5 * 2^23).
constexpr int GEMM_BIAS_BITS = 0x4B400000;
constexpr float GEMM_BIAS = 12582912.0f;

struct GemmArgs {
  const uint8_t* a;   // weight chunks [row tiles][nk] (gemm::A_CHUNK bytes each)
  const uint8_t* b;   // activation chunks [token tiles][nk] (gemm::b_chunk(NT) each)
  float* out;         // [n_tok][ldo], columns [0, rows) written (ksplit == 1)
  int rows, ldo, n_tok, nk, n_rt, n_tt;
  int ksplit;         // K split into ksplit equal ranges of nk / ksplit chunks
  float* part;        // ksplit > 1: partial sums [ksplit][n_tok][rows]
  int nstages;
  Result* res;
  unsigned long long wait_ns;
};

// Rescale warps: each TMEM lane quarter (weight rows 32q..) is read by one
// warp per group of token columns, so a warp rescales 16 products per row
// and block at 16 and 32 tokens, 32 at 64 (two CTAs per SM, eight warps
// each) and 128: the per-block cost of waiting, loading from tensor memory
// and releasing is paid for at least 16 products, and a scheduler has one
// to four rescale warps.
__host__ __device__ constexpr int gemm_epi_warps(int nt) {
  return nt >= 64 ? (gemm::ctas_per_sm(nt) == 2 ? 8 : 16) : nt / 4;
}
__host__ __device__ constexpr int gemm_threads(int nt) {
  return 32 * (2 + gemm_epi_warps(nt));  // producer, MMA issuer, rescale
}

struct GemmSmem {
  uint64_t full[gemm::MAX_STAGES_G];   // stage landed (A and B copies)
  uint64_t empty[gemm::MAX_STAGES_G];  // stage consumed: 1 MMA commit + every rescale warp
  uint64_t tfull[32];                  // TMEM buffer holds a finished block product
  uint64_t tempty[32];                 // TMEM buffer read by every rescale warp
  uint64_t drain;                      // every MMA issued has completed
  uint32_t tmem_base;
  int abort_flag;
  int issued;
  int producer_done;
};
static_assert(sizeof(GemmSmem) <= gemm::SMEM_HEAD, "gemm smem head");

// out[n][r] = sum over Q8_0 blocks b of fp16(d_w[r,b]) * d_x[n,b] * I_b[r,n]
// for every token n < n_tok and row r < rows: n_tok matvec_q8_c products
// (simd.c:33-110) sharing one pass over the weights.
//
// Roles: warp 0 lane 0 streams (weight chunk, activation chunk) pairs into a
// ring of shared-memory stages with 1-D bulk copies (the weight copies of the
// first stages are issued before griddepcontrol.wait: weights never depend on
// the previous kernel); warp 1 lane 0 issues one kind::i8 MMA per Q8_0 block
// (M = 128 weight rows, N = NT tokens, K = 32) into one of NB tensor-memory
// buffers and commits its completion to that buffer's barrier; warps 2..
// read each block's int32 products back (warp w reads TMEM lanes 32*(w%4)..,
// i.e. weight rows, and the columns of its group of the token tile),
// rescale them by
// d_w * d_x and accumulate in fp32 registers, then release the buffer.  A
// stage is refilled once its four MMAs have completed and every rescale
// warp has read its scales.  Work units (row tile, token tile, K range)
// are dealt round-robin over the grid; after the last chunk of a unit the
// rescale warps store its outputs, or with a split K its partial sums
// (k_gemm_reduce adds them in split order).
template <int NT>
__global__ void __launch_bounds__(gemm_threads(NT), gemm::ctas_per_sm(NT))
    k_gemm_q8(const __grid_constant__ GemmArgs g) {
  using namespace gemm;
  constexpr int NB = tmem_buffers(NT);
  constexpr uint32_t TCOLS = tmem_cols(NT);
  constexpr int EPI = gemm_epi_warps(NT);
  constexpr int CPT = NT / (EPI / 4);  // token columns per rescale thread
  // blocks rescaled per group: 64 (16 warps, or two CTAs per SM: 32)
  // loaded products per thread
  constexpr int LP = EPI >= 16 || ctas_per_sm(NT) == 2 ? 32 : 64;
  constexpr int GB = LP / CPT >= BPC ? BPC : (LP / CPT >= 2 ? LP / CPT : 1);
  static_assert(BPC % GB == 0 && tmem_buffers(NT) >= 2 * GB, "rescale groups");
  constexpr uint32_t IDESC = idesc_i8(TILE_M, NT);
  constexpr int SB = stage_bytes(NT);
  static_assert(NB * NT <= (int)TCOLS && TCOLS <= 512, "tensor memory budget");
  static_assert(CPT % 4 == 0, "tcgen05.ld granularity");
  L3G_DYNAMIC_SMEM(smem);
  GemmSmem* sh = reinterpret_cast<GemmSmem*>(smem);
  uint8_t* ring = smem + SMEM_HEAD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = g.nstages;
  const int nku = g.nk / g.ksplit;  // chunks per unit
  const int n_units = g.n_rt * g.n_tt * g.ksplit;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const int my_units = cta < n_units ? (n_units - cta + G - 1) / G : 0;
  const int nchunks = my_units * nku;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1 + EPI);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&sh->tfull[i], 1);
      mbar_init(&sh->tempty[i], EPI);
    }
    mbar_init(&sh->drain, 1);
    sh->abort_flag = 0;
    sh->issued = 0;
    sh->producer_done = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sh->tmem_base, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---- producer -------------------------------------------------------
    if (lane == 0) {
      // the CTA's c-th chunk: unit cta + (c / nku) * G, chunk (c % nku) of its range
      auto a_src = [&](int c) {
        const int u = cta + (c / nku) * G;
        const int tile = u / g.ksplit, kc = (u % g.ksplit) * nku + c % nku;
        return g.a + ((size_t)(tile % g.n_rt) * g.nk + kc) * A_CHUNK;
      };
      auto b_src = [&](int c) {
        const int u = cta + (c / nku) * G;
        const int tile = u / g.ksplit, kc = (u % g.ksplit) * nku + c % nku;
        return g.b + ((size_t)(tile / g.n_rt) * g.nk + kc) * b_chunk(NT);
      };
      const int pre = nchunks < ns ? nchunks : ns;
      for (int c = 0; c < pre; ++c) {
        mbar_arrive_expect_tx(&sh->full[c], SB);
        bulk_g2s(ring + (size_t)c * SB, a_src(c), A_CHUNK, &sh->full[c]);
      }
      pdl_wait();  // the activations come from the previous kernel
      for (int c = 0; c < pre; ++c)
        bulk_g2s(ring + (size_t)c * SB + A_CHUNK, b_src(c), b_chunk(NT), &sh->full[c]);
      *(volatile int*)&sh->issued = pre;
      for (int c = pre; c < nchunks; ++c) {
        const int s = c % ns;
        if (!mbar_wait(&sh->empty[s], ((c / ns) - 1) & 1, &sh->abort_flag, g.res, 20, g.wait_ns))
          break;
        mbar_arrive_expect_tx(&sh->full[s], SB);
        bulk_g2s(ring + (size_t)s * SB, a_src(c), A_CHUNK, &sh->full[s]);
        bulk_g2s(ring + (size_t)s * SB + A_CHUNK, b_src(c), b_chunk(NT), &sh->full[s]);
        *(volatile int*)&sh->issued = c + 1;
      }
      *(volatile int*)&sh->producer_done = 1;
    }
  } else if (warp == 1) {
    // ---- MMA issuer -----------------------------------------------------
    if (lane == 0) {
      int blk = 0;
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c % ns;
        if (!mbar_wait(&sh->full[s], (c / ns) & 1, &sh->abort_flag, g.res, 21, g.wait_ns)) break;
        const uint32_t a0 = smem_u32(ring + (size_t)s * SB);
        const uint32_t b0 = a0 + A_CHUNK;
#pragma unroll
        for (int j = 0; j < BPC; ++j, ++blk) {
          const int buf = blk % NB, use = blk / NB;
          if (use > 0 &&
              !mbar_wait(&sh->tempty[buf], (use - 1) & 1, &sh->abort_flag, g.res, 22, g.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          mma_i8(tmem + (uint32_t)(buf * NT), a_desc(a0, j), b_desc(b0, j, NT), IDESC, 0u);
          mma_commit(&sh->tfull[buf]);
        }
        if (ok) mma_commit(&sh->empty[s]);
      }
      // every MMA issued has completed before the tensor memory is released
      if (blk > 0) {
        mma_commit(&sh->drain);
        int dummy = 0;
        mbar_wait(&sh->drain, 0, &dummy, g.res, 23, g.wait_ns);
      }
    }
    __syncwarp();
  } else {
    // ---- rescale warps --------------------------------------------------
    const int ep = warp - 2;
    const int quarter = warp & 3;      // TMEM lanes this warp may read
    const int half = ep >> 2;          // column group: token columns [half*CPT, half*CPT+CPT)
    const int m = quarter * 32 + lane; // weight row within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * CPT);
    int c = 0, blk = 0;
    bool ok = true;
    for (int ui = 0; ui < my_units && ok; ++ui) {
      const int u = cta + ui * G;
      const int tile = u / g.ksplit, ks = u % g.ksplit;
      const int rt = tile % g.n_rt, tt = tile / g.n_rt;
      unsigned long long acc2[CPT / 2];  // fp32 pairs (columns 2i, 2i + 1)
#pragma unroll
      for (int i = 0; i < CPT / 2; ++i) acc2[i] = 0ull;
      for (int kc = 0; kc < nku; ++kc, ++c) {
        const int s = c % ns;
        ok = __all_sync(0xffffffffu, mbar_wait(&sh->full[s], (c / ns) & 1, &sh->abort_flag,
                                               g.res, 24, g.wait_ns));
        if (!ok) break;
        const uint8_t* st = ring + (size_t)s * SB;
        const __half* dw = reinterpret_cast<const __half*>(st + A_Q_BYTES);
        const float* dx = reinterpret_cast<const float*>(st + A_CHUNK + b_q_bytes(NT));
        // blocks in groups of GB: every block's products are loaded from
        // tensor memory before one wait for the loads, so the latency of a
        // wait, a load and a release is paid once per group
#pragma unroll 1
        for (int j0 = 0; j0 < BPC; j0 += GB, blk += GB) {
          uint32_t v[GB][CPT];
#pragma unroll
          for (int gi = 0; gi < GB; ++gi) {
            const int buf = (blk + gi) % NB, use = (blk + gi) / NB;
            ok = __all_sync(0xffffffffu, mbar_wait(&sh->tfull[buf], use & 1, &sh->abort_flag,
                                                   g.res, 25, g.wait_ns));
            if (!ok) break;
            tc_fence_after();
            if constexpr (CPT % 8 == 0) {
#pragma unroll
              for (int i = 0; i < CPT / 8; ++i)
                tmem_ld8(t_lane + (uint32_t)(buf * NT + i * 8), v[gi] + i * 8);
            } else {
#pragma unroll
              for (int i = 0; i < CPT / 4; ++i)
                tmem_ld4(t_lane + (uint32_t)(buf * NT + i * 4), v[gi] + i * 4);
            }
          }
          if (!ok) break;
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
#pragma unroll
            for (int gi = 0; gi < GB; ++gi) mbar_arrive(&sh->tempty[(blk + gi) % NB]);
          // acc += float(I) * (d_w * d_x), per column, as fmaf(I, d_w * d_x, acc)
          const unsigned long long nbias2 = pk2(-GEMM_BIAS, -GEMM_BIAS);
#pragma unroll
          for (int gi = 0; gi < GB; ++gi) {
            const int j = j0 + gi;
            const float w = __half2float(dw[j * TILE_M + m]);
            const unsigned long long w2 = pk2(w, w);
            // the column scales of this block: 16-byte loads (NT and CPT are
            // multiples of 4, the stage 128-byte aligned), a pair per product pair
            const float4* dxj = reinterpret_cast<const float4*>(dx + j * NT + half * CPT);
#pragma unroll
            for (int i = 0; i < CPT / 2; ++i) {
              const float4 d4 = dxj[i >> 1];
              const unsigned long long s2 =
                  mul2(w2, (i & 1) ? pk2(d4.z, d4.w) : pk2(d4.x, d4.y));
              const unsigned long long f2 =
                  add2(pk2(__int_as_float((int)v[gi][2 * i] + GEMM_BIAS_BITS),
                           __int_as_float((int)v[gi][2 * i + 1] + GEMM_BIAS_BITS)),
                       nbias2);
              acc2[i] = fma2(f2, s2, acc2[i]);
            }
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->empty[s]);
      }
      if (!ok) break;
      const int row = rt * TILE_M + m;
      if (row < g.rows) {
        float* dst = g.ksplit > 1 ? g.part + (size_t)ks * g.n_tok * g.rows : g.out;
        const int ld = g.ksplit > 1 ? g.rows : g.ldo;
#pragma unroll
        for (int i = 0; i < CPT / 2; ++i) {
          const float2 a2 = upk2(acc2[i]);
          const int n = tt * NT + half * CPT + 2 * i;
          if (n < g.n_tok) dst[(size_t)n * ld + row] = a2.x;
          if (n + 1 < g.n_tok) dst[(size_t)(n + 1) * ld + row] = a2.y;
        }
      }
    }
  }

  // After an abort: wait (bounded) until the producer has stopped issuing,
  // then for the last copy issued to each stage.
  if (*(volatile int*)&sh->abort_flag && threadIdx.x == 0) {
    const uint64_t t_start = gtime();
    while (!*(volatile int*)&sh->producer_done && gtime() - t_start < 100000000ull) {
    }
    const int issued = *(volatile int*)&sh->issued;
    for (int s2 = 0; s2 < ns && s2 < issued; ++s2) {
      const int t = s2 + ((issued - 1 - s2) / ns) * ns;
      int dummy = 0;
      mbar_wait(&sh->full[s2], (t / ns) & 1, &dummy, g.res, 26, 100000000ull);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TCOLS);
  }
}

// out[n][r] = sum over k of part[k][n][r], k in order (deterministic).
static __global__ void k_gemm_reduce(const float* part, int ksplit, int n_tok, int rows, int ldo,
                              float* out) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (long long)n_tok * rows) return;
  const int n = (int)(e / rows), r = (int)(e % rows);
  float v = part[e];
  for (int k = 1; k < ksplit; ++k) v += part[(size_t)k * n_tok * rows + e];
  out[(size_t)n * ldo + r] = v;
}

// QuantizeQ8_0Into (q8_0.go:22-79) of n_tok rows of x [n_tok][cols] into the
// activation chunks of the batched product: one warp per (token, 32-column
// block), one value per lane; tokens n_tok..n_pad-1 and the columns past
// cols up to the chunk boundary are written as zero blocks.  Bit-identical
// to the reference's quantization of each row.
static __global__ void k_gemm_quantize(const float* x, int n_tok, int cols, int nt, int nk,
                                int n_pad, uint8_t* act) {
  using namespace gemm;
  pdl_launch_dependents();
  pdl_wait();
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int nbk = nk * BPC;
  if (gw >= n_pad * nbk) return;
  const int n = gw / nbk, bk = gw % nbk;
  const int k = bk * QBLK + lane;
  const bool live = n < n_tok && bk * QBLK < cols;
  const float v = live ? x[(size_t)n * cols + k] : 0.0f;
  const float mx = warp_max(fabsf(v));
  float scale = __fdiv_rn(mx, 127.0f);
  if (scale == 0.0f) scale = 1e-8f;
  const float inv = __frcp_rn(scale);
  const int8_t q = live ? quant_one(v, inv) : (int8_t)0;
  const int ti = n / nt, nn = n % nt, c = bk / BPC, j = bk % BPC;
  uint8_t* ch = act + ((size_t)ti * nk + c) * b_chunk(nt);
  ch[q_offset(nt, nn, j * QBLK + lane)] = (uint8_t)q;
  if (lane == 0) reinterpret_cast<float*>(ch + b_q_bytes(nt))[j * nt + nn] = live ? scale : 0.0f;
}
