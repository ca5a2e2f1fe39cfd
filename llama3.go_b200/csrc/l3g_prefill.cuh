// Batched prefill kernels (included by l3g_kernels.cuh after l3g_gemm.cuh).
//
// The reference ingests a prompt one ForwardIntoWorkspace per token
// (cmd/go-llama-chat/main.go:276-286, infer.go:21-267).  Batched prefill
// runs the same per-token arithmetic for P tokens at once: the projections
// as batched Q8_0 products on the tensor cores (k_gemm_q8), everything
// between them as row-wise kernels here, and causal attention of the P new
// positions over the cache.  Rows are token-major: X[p][n_emb] etc.
#pragma once

// x[p][i] = f16(d) * q[i] of embedding row ids[p] (infer.go:513-518,
// tensor_read.go:128-147), as k_embed.  grid (ceil(cols / 256), P).
static __global__ void k_pf_embed(const uint8_t* emb, int vocab, int cols, const int* ids, float* X,
                           Result* res) {
  const int p = blockIdx.y;
  const int token = ids[p];
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
  X[(size_t)p * cols + i] = __fmul_rn(d, (float)(int8_t)blk[2 + (i & 31)]);
}

// Store one quantized value group (4 consecutive columns k..k+3 of token n)
// and, from the group's first lane, the block scale, into activation chunks.
__device__ __forceinline__ void pf_store_quad(uint8_t* act, int nt, int nk, int n, int k,
                                              char4 q, float scale, bool first) {
  using namespace gemm;
  const int ti = n / nt, nn = n % nt, c = k / KC, kin = k % KC;
  uint8_t* ch = act + ((size_t)ti * nk + c) * b_chunk(nt);
  *reinterpret_cast<char4*>(ch + q_offset(nt, nn, kin)) = q;
  if (first) reinterpret_cast<float*>(ch + b_q_bytes(nt))[(kin / QBLK) * nt + nn] = scale;
}

// Per token p (one CTA of PF_THREADS): v = X[p] (+ Y[p], written back to
// X[p]: the residual adds infer.go:189-191 / :244-246), rmsNorm (math.go:5-14)
// with weights w, then QuantizeQ8_0Into (q8_0.go:22-79) of the normed row
// into the activation chunks (token tile nt, nk chunks).  The same arithmetic
// as the PRO_RMS prologue of the decode matvecs; cols a multiple of 32, at
// most PF_THREADS * 4 * PF_VK.
constexpr int PF_THREADS = 256;
constexpr int PF_VK = 8;
static __global__ void __launch_bounds__(PF_THREADS) k_pf_rms_quant(float* X, const float* Y,
                                                             const float* w, float eps, int cols,
                                                             int nt, int nk, uint8_t* act) {
  __shared__ float red[PF_THREADS / 32];
  const int p = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nv = cols >> 2;
  float4* x4 = reinterpret_cast<float4*>(X + (size_t)p * cols);
  const float4* y4 = Y ? reinterpret_cast<const float4*>(Y + (size_t)p * cols) : nullptr;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 v[PF_VK];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < PF_VK; ++k) {
    const int i = tid + k * PF_THREADS;
    v[k] = i < nv ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (y4 && i < nv) {
      const float4 y = y4[i];
      v[k].x = __fadd_rn(v[k].x, y.x);
      v[k].y = __fadd_rn(v[k].y, y.y);
      v[k].z = __fadd_rn(v[k].z, y.z);
      v[k].w = __fadd_rn(v[k].w, y.w);
      x4[i] = v[k];
    }
    ss = fmaf(v[k].x, v[k].x, ss);
    ss = fmaf(v[k].y, v[k].y, ss);
    ss = fmaf(v[k].z, v[k].z, ss);
    ss = fmaf(v[k].w, v[k].w, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int q = 0; q < PF_THREADS / 32; ++q) tot += red[q];
  const float scale = (float)(1.0 / sqrt((double)__fadd_rn(__fdiv_rn(tot, (float)cols), eps)));
#pragma unroll
  for (int k = 0; k < PF_VK; ++k) {
    const int i = tid + k * PF_THREADS;
    if (k * PF_THREADS >= nv) break;  // uniform
    const bool live = i < nv;
    float4 u = v[k];
    const float4 wk = live ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    u.x = __fmul_rn(__fmul_rn(u.x, scale), wk.x);
    u.y = __fmul_rn(__fmul_rn(u.y, scale), wk.y);
    u.z = __fmul_rn(__fmul_rn(u.z, scale), wk.z);
    u.w = __fmul_rn(__fmul_rn(u.w, scale), wk.w);
    // the 8 lanes (lane & 7) of an aligned group share one 32-column block
    float m = fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    if (!live) continue;
    float sc = __fdiv_rn(m, 127.0f);
    if (sc == 0.0f) sc = 1e-8f;
    const float inv = __frcp_rn(sc);
    char4 q;
    q.x = quant_one(u.x, inv);
    q.y = quant_one(u.y, inv);
    q.z = quant_one(u.z, inv);
    q.w = quant_one(u.w, inv);
    pf_store_quad(act, nt, nk, p, i * 4, q, sc, (lane & 7) == 0);
  }
}

// act_i = silu(gate_i) * up_i (infer.go:228-230) of the interleaved up/gate
// rows UG[p][2i] = up_i, UG[p][2i+1] = gate_i, quantized (q8_0.go:22-79) into
// the activation chunks for down.  One warp per (token, 32 outputs).
static __global__ void k_pf_swiglu_quant(const float* UG, int P, int ff, int nt, int nk, uint8_t* act) {
  using namespace gemm;
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int nb = ff / QBLK;
  if (gw >= P * nb) return;
  const int p = gw / nb, b = gw % nb;
  const int i = b * QBLK + lane;
  const float2 ug = reinterpret_cast<const float2*>(UG + (size_t)p * 2 * ff)[i];
  const float v = __fmul_rn(silu_ref(ug.y), ug.x);
  const float mx = warp_max(fabsf(v));
  float scale = __fdiv_rn(mx, 127.0f);
  if (scale == 0.0f) scale = 1e-8f;
  const float inv = __frcp_rn(scale);
  const int8_t q = quant_one(v, inv);
  const int ti = p / nt, nn = p % nt, c = i / KC, kin = i % KC;
  uint8_t* ch = act + ((size_t)ti * nk + c) * b_chunk(nt);
  ch[q_offset(nt, nn, kin)] = (uint8_t)q;
  if (lane == 0) reinterpret_cast<float*>(ch + b_q_bytes(nt))[(kin / QBLK) * nt + nn] = scale;
}

// RoPE (rope.go:39-52) on the q and k rows of QKV[p] = [q | k | v] at
// position pos0 + p, q to Q[p], k and v appended to layer `layer` of the
// paged cache (infer.go:122-127), as the EPI_QKV epilogue of the decode
// step.  One thread per adjacent pair; grid covers P * rows/2.
static __global__ void k_pf_qkv_rope(const float* QKV, int P, int pos0, int nq, int nkv, int hd,
                              int rope_half, const float* rope_cos, const float* rope_sin,
                              float* Q, const KvMap kv, int layer, int kv_f16) {
  const int rows = nq + 2 * nkv;
  const int half_rows = rows >> 1;
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (long long)P * half_rows) return;
  const int p = (int)(e / half_rows);
  const int row = (int)(e % half_rows) * 2;
  const int pos = pos0 + p;
  const float2 xv = *reinterpret_cast<const float2*>(QKV + (size_t)p * rows + row);
  float x0 = xv.x, x1 = xv.y;
  const bool is_q = row < nq;
  const bool is_k = !is_q && row < nq + nkv;
  if (is_q || is_k) {
    const int d = (is_q ? row : row - nq) % hd;
    const int i = d >> 1;
    if (i < rope_half) {
      const float c = rope_cos[(size_t)pos * rope_half + i];
      const float s = rope_sin[(size_t)pos * rope_half + i];
      const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
      x0 = y0;
      x1 = y1;
    }
  }
  if (is_q) {
    *reinterpret_cast<float2*>(Q + (size_t)p * nq + row) = make_float2(x0, x1);
  } else {
    const int r2 = is_k ? row - nq : row - nq - nkv;
    const int kvh = r2 / hd, d = r2 % hd;
    const size_t off = (is_k ? 0 : hd) + d;
    uint8_t* base = kv_row(kv, layer, kvh, pos);
    if (kv_f16)
      *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + off) = __floats2half2_rn(x0, x1);
    else
      *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + off) = make_float2(x0, x1);
  }
}

// Causal GQA attention of P new positions pos0..pos0+P-1 over the cache
// positions 0..pos (infer.go:130-175: s_t = dot(q, K_t) * scale, softmax
// with max, out = sum_t softmax_t * V_t; here as an online softmax over key
// tiles, like the decode kernel).  CTA (query block, kv head): the G query
// heads of the kv head times BQ consecutive positions, R = G * BQ <= 64 rows,
// row r = token (r / G), head (r % G); 8 warps of up to 8 rows each.  Key
// tiles of 32 positions are staged in shared memory (K transposed with a
// padded row, so lane = key reads and the transposing stores are free of bank
// conflicts; V row-major, lane j*32+lane = dims).  Dynamic shared memory:
// pf_attention_smem(HD) bytes.
__host__ __device__ constexpr int pf_attention_smem(int hd) {
  return (64 * hd + hd * 33 + 32 * hd) * 4;
}
template <int HD, typename KT>
__global__ void __launch_bounds__(256) k_pf_attention(const float* Q, const KvMap kv, int layer,
                                                      float* out, int P, int pos0, int group,
                                                      int bq, int nq_heads, float scale) {
  constexpr int DPL = HD / 32;  // output dims per lane: lane + 32 j
  constexpr int RW = 8;         // rows per warp
  L3G_DYNAMIC_SMEM(pf_smem_raw);
  float* pf_smem = reinterpret_cast<float*>(pf_smem_raw);
  float(*qs)[HD] = reinterpret_cast<float(*)[HD]>(pf_smem);
  float(*kt)[33] = reinterpret_cast<float(*)[33]>(pf_smem + 64 * HD);
  float(*vs)[HD] = reinterpret_cast<float(*)[HD]>(pf_smem + 64 * HD + HD * 33);
  const int kvh = blockIdx.y;
  const int tok0 = blockIdx.x * bq;
  const int ntok = min(bq, P - tok0);
  const int R = group * ntok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // query rows of this block
  for (int e = threadIdx.x; e < R * HD; e += 256) {
    const int r = e / HD, d = e % HD;
    const int t = r / group, g = r % group;
    qs[r][d] = Q[(size_t)(tok0 + t) * nq_heads * HD + (size_t)(kvh * group + g) * HD + d];
  }
  float o[RW][DPL];
  float mrow[RW], lrow[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[i][j] = 0.0f;
  }
  const int last = pos0 + tok0 + ntok - 1;  // last key any row of the block sees
  for (int kb = 0; kb <= last; kb += 32) {
    __syncthreads();  // previous tile consumed (and, first time, qs written)
    // the tile's 32 keys start at a multiple of 32, which divides KV_PAGE:
    // they are consecutive rows of one page
    const KT* kvp = reinterpret_cast<const KT*>(kv_row(kv, layer, kvh, kb));
    for (int e = threadIdx.x; e < 32 * HD; e += 256) {
      const int key = e / HD, d = e % HD;
      const int kp = kb + key;
      float kval = 0.0f, vval = 0.0f;
      if (kp <= last) {
        kval = (float)kvp[(size_t)key * 2 * HD + d];
        vval = (float)kvp[(size_t)key * 2 * HD + HD + d];
      }
      kt[d][key] = kval;
      vs[key][d] = vval;
    }
    __syncthreads();
    // this warp's rows r0 .. r0 + nr - 1 (warp-uniform); every key and value
    // element read from shared memory serves all of them
    const int r0 = warp * RW;
    const int nr = min(RW, R - r0);
    if (nr > 0) {
      float sdot[RW];
#pragma unroll
      for (int i = 0; i < RW; ++i) sdot[i] = 0.0f;
#pragma unroll 2
      for (int d = 0; d < HD; d += 4) {
        const float k0 = kt[d][lane], k1 = kt[d + 1][lane], k2 = kt[d + 2][lane],
                    k3 = kt[d + 3][lane];
#pragma unroll
        for (int i = 0; i < RW; ++i) {
          if (i < nr) {
            const float4 q4 = *reinterpret_cast<const float4*>(&qs[r0 + i][d]);
            sdot[i] = fmaf(q4.x, k0, sdot[i]);
            sdot[i] = fmaf(q4.y, k1, sdot[i]);
            sdot[i] = fmaf(q4.z, k2, sdot[i]);
            sdot[i] = fmaf(q4.w, k3, sdot[i]);
          }
        }
      }
      const int kp = kb + lane;
      float pe[RW];
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        pe[i] = 0.0f;
        if (i < nr) {
          const int limit = pos0 + tok0 + (r0 + i) / group;  // causal: keys <= own position
          const bool valid = kp <= limit;
          const float sc = valid ? __fmul_rn(sdot[i], scale) : -INFINITY;
          const float mn = fmaxf(mrow[i], warp_max(sc));
          pe[i] = valid ? expf(sc - mn) : 0.0f;
          const float corr = mrow[i] == -INFINITY ? 0.0f : expf(mrow[i] - mn);
          lrow[i] = fmaf(lrow[i], corr, warp_sum(pe[i]));
          mrow[i] = mn;
#pragma unroll
          for (int j = 0; j < DPL; ++j) o[i][j] *= corr;
        }
      }
#pragma unroll 4
      for (int key = 0; key < 32; ++key) {
        float vv[DPL];
#pragma unroll
        for (int j = 0; j < DPL; ++j) vv[j] = vs[key][j * 32 + lane];
#pragma unroll
        for (int i = 0; i < RW; ++i) {
          if (i < nr) {
            const float pk = __shfl_sync(0xffffffffu, pe[i], key);
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[i][j] = fmaf(pk, vv[j], o[i][j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int r = warp * RW + i;
    if (r >= R) break;
    const int t = r / group, g = r % group;
    float* dst = out + (size_t)(tok0 + t) * nq_heads * HD + (size_t)(kvh * group + g) * HD;
    const float inv = 1.0f / lrow[i];
#pragma unroll
    for (int j = 0; j < DPL; ++j) dst[j * 32 + lane] = o[i][j] * inv;
  }
}

// Weight chunks of the batched product from a matrix already resident in
// the decode kernels' tile layout (Q8Tiles: tile (g, s) = int8 q[wr][ck] then
// fp16 d[wr][ck/32]), so the sharded, fused and interleaved row orders of the
// decode step carry over unchanged.  One thread per (row, block); dst must
// be zeroed first (padding rows and blocks stay zero).
static __global__ void k_gemm_from_tiles(const Q8Tiles t, uint8_t* dst) {
  using namespace gemm;
  const int nbc = t.cols / 32;
  const int nk = chunks(t.cols);
  const long long total = (long long)t.rows * nbc;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / nbc), b = (int)(e % nbc);
    const int g = r / t.wr, i = r % t.wr;
    const int bpt = t.ck / 32;
    const int s = b / bpt, bb = b % bpt;
    const uint8_t* tile = t.data + ((size_t)g * t.nslices + s) * t.tile_bytes;
    const uint8_t* q = tile + (size_t)i * t.ck + bb * 32;
    const uint8_t* d = tile + (size_t)t.wr * t.ck + ((size_t)i * bpt + bb) * 2;
    const int rt = r / TILE_M, m = r % TILE_M, c = b / BPC, j = b % BPC;
    uint8_t* ch = dst + ((size_t)rt * nk + c) * A_CHUNK;
    const int4* q4 = reinterpret_cast<const int4*>(q);
    *reinterpret_cast<int4*>(ch + q_offset(TILE_M, m, j * QBLK)) = q4[0];
    *reinterpret_cast<int4*>(ch + q_offset(TILE_M, m, j * QBLK + 16)) = q4[1];
    ch[A_Q_BYTES + (j * TILE_M + m) * 2] = d[0];
    ch[A_Q_BYTES + (j * TILE_M + m) * 2 + 1] = d[1];
  }
}
