// Work schedule of the persistent decode-step kernel (k_layers), shared by
// the device code and the host-side schedule checks.  Plain C++ (host and
// device), no CUDA API.
//
// k_layers runs every layer of one decode step (ForwardIntoWorkspace,
// internal/llama/infer.go:56-246) in one launch of one CTA per SM.  Per
// layer it walks seven phases separated by grid barriers:
//
//   0 QKV     residual add + rmsNorm + act-quant, Q/K/V matvec, RoPE, KV append
//   1 ATT     split-K attention over the KV cache: one (kv head, split) item per CTA
//   2 MERGE   merge of the splits, act-quant of the attention output
//   3 WO      Wo matvec (tensor parallel: rows pushed to every rank, then summed)
//   4 UPGATE  residual add + rmsNorm + act-quant, up/gate matvec, SwiGLU
//   5 QUANT   act-quant of the SwiGLU output
//   6 DOWN    down matvec (tensor parallel: pushed and summed like Wo)
//
// One producer warp per CTA streams every tile the CTA will consume, in
// consumption order and across phase boundaries, through one shared-memory
// ring: the weight tiles of its row groups of the four matrices and the K|V
// stages of its attention item.  Weights and past KV rows never depend on
// the step, so the ring keeps streaming while the consumers wait at a
// barrier; only the stage holding this step's own K/V waits (on the barrier
// after QKV) before it is copied.
//
// Row groups of a matrix (wr rows, all column slices) are dealt round-robin
// over the CTAs, and each phase starts dealing where the previous one
// stopped (a rotation), so the per-CTA bytes of a whole layer stay within
// one group of each other instead of the same CTAs taking every phase's
// remainder.
#pragma once

#include <stdint.h>

#ifndef L3G_HD
#if defined(__CUDACC__)
#define L3G_HD __host__ __device__
#else
#define L3G_HD
#endif
#endif

namespace l3g {

// Geometry of a repacked Q8_0 matrix: rows grouped by wr = nw * rpw, columns
// sliced so that one tile (wr rows x ck columns of int8, then the fp16
// scales, padded to 16 bytes) is about tile_target bytes with a whole
// number of 32-blocks per slice.
struct TileGeom {
  int wr, ck, nslices, tile_bytes, n_groups;
};
L3G_HD inline TileGeom tile_geometry(int rows, int cols, int rpw, int nw, int tile_target) {
  TileGeom t;
  t.wr = nw * rpw;
  const int nb = cols / 32;
  int nsl = (int)(((long long)cols * t.wr + tile_target - 1) / tile_target);
  if (nsl < 1) nsl = 1;
  while (nb % nsl) ++nsl;
  t.nslices = nsl;
  t.ck = cols / nsl;
  t.tile_bytes = (t.wr * t.ck + t.wr * (t.ck / 32) * 2 + 15) / 16 * 16;
  t.n_groups = (rows + t.wr - 1) / t.wr;
  return t;
}

namespace persist {

enum Mat { M_QKV = 0, M_WO = 1, M_UPGATE = 2, M_DOWN = 3, N_MAT = 4 };
// Units dealt round-robin, in layer order: QKV groups, attention items,
// Wo groups, up/gate groups, down groups.
enum Deal { D_QKV = 0, D_ATT = 1, D_WO = 2, D_UPGATE = 3, D_DOWN = 4, N_DEAL = 5 };
constexpr int BARRIERS_PER_LAYER = 7;  // after QKV, ATT, MERGE, WO, UPGATE, QUANT, DOWN
// With the SwiGLU act-quant fused into the up/gate phase the QUANT phase and
// its barrier go; with the split merge fused into the attention phase the
// barrier between ATT and MERGE goes: 7, 6 or 5 barriers per layer.
L3G_HD inline int barriers_per_layer(bool fuse_quant, bool fuse_merge = false) {
  return 7 - (fuse_quant ? 1 : 0) - (fuse_merge ? 1 : 0);
}

struct Plan {
  int grid;       // CTAs (one per SM)
  int n_layers;
  // per matrix (same geometry in every layer)
  int ng[N_MAT];          // row groups
  int nsl[N_MAT];         // column slices per group
  int tile_bytes[N_MAT];  // bytes of one tile (one bulk copy)
  int wr[N_MAT];          // rows per group
  int ck[N_MAT];          // columns per slice
  int rows[N_MAT];
  int cols[N_MAT];
  // attention
  int hkv;        // kv heads of this rank
  int splits;     // splits per kv head (hkv * splits <= grid)
  int P;          // positions per stage
  int row_bytes;  // bytes of one position's K|V row (2 * head_dim * element size)
  int ctx;        // positions per kv head in the cache
};

// Units of each deal per layer.
L3G_HD inline int deal_units(const Plan& p, int d) {
  switch (d) {
    case D_QKV: return p.ng[M_QKV];
    case D_ATT: return p.hkv * p.splits;
    case D_WO: return p.ng[M_WO];
    case D_UPGATE: return p.ng[M_UPGATE];
    default: return p.ng[M_DOWN];
  }
}

// First CTA of deal d in layer l: where the previous deal stopped.
L3G_HD inline int deal_rot(const Plan& p, int l, int d) {
  int per_layer = 0;
  for (int i = 0; i < N_DEAL; ++i) per_layer += deal_units(p, i) % p.grid;
  int r = (int)(((long long)l * per_layer) % p.grid);
  for (int i = 0; i < d; ++i) r = (r + deal_units(p, i)) % p.grid;
  return r;
}

// CTA b's position in deal d of layer l: it takes units vb, vb + grid, ...
L3G_HD inline int deal_vrank(const Plan& p, int l, int d, int b) {
  return (b - deal_rot(p, l, d) + p.grid) % p.grid;
}

L3G_HD inline int mat_deal(int m) {
  return m == M_QKV ? D_QKV : m == M_WO ? D_WO : m == M_UPGATE ? D_UPGATE : D_DOWN;
}

// Row groups of matrix m that CTA b takes in layer l.
L3G_HD inline int my_groups(const Plan& p, int l, int m, int b) {
  const int vb = deal_vrank(p, l, mat_deal(m), b);
  return vb < p.ng[m] ? (p.ng[m] - vb + p.grid - 1) / p.grid : 0;
}
// Its k-th row group.
L3G_HD inline int my_group(const Plan& p, int l, int m, int b, int k) {
  return deal_vrank(p, l, mat_deal(m), b) + k * p.grid;
}
// Byte offset of tile (group g, slice s) in a matrix stored group-major.
L3G_HD inline long long tile_offset(const Plan& p, int m, int g, int s) {
  return ((long long)g * p.nsl[m] + s) * p.tile_bytes[m];
}

// Attention item of CTA b in layer l: kv head and split, or false.
L3G_HD inline bool my_item(const Plan& p, int l, int b, int* kvh, int* split) {
  const int it = deal_vrank(p, l, D_ATT, b);
  if (it >= p.hkv * p.splits) return false;
  *kvh = it / p.splits;
  *split = it % p.splits;
  return true;
}
// Positions [t0, t1) of split `split` when positions 0..n-1 are live: a
// chunk of whole stages per split, the last splits possibly empty.
L3G_HD inline void item_range(const Plan& p, int split, int n, int* t0, int* t1) {
  const int per = (n + p.splits - 1) / p.splits;
  const int chunk = (per + p.P - 1) / p.P * p.P;
  const long long a = (long long)split * chunk;
  *t0 = a < n ? (int)a : n;
  *t1 = *t0 + chunk < n ? *t0 + chunk : n;
}
L3G_HD inline int item_stages(const Plan& p, int t0, int t1) { return (t1 - t0 + p.P - 1) / p.P; }
// Byte offset, in one layer's cache, of stage st of kv head kvh from t0.
L3G_HD inline long long stage_offset(const Plan& p, int kvh, int t0, int st) {
  return ((long long)kvh * p.ctx + t0 + (long long)st * p.P) * p.row_bytes;
}

// Global index of barrier j of layer l, bpl barriers per layer (the last
// layer's last barrier is never run: the kernel ends).  Arrivals are spread over
// nsub counters (1 to BAR_MAX_SUB, each on its own 128-byte line): CTA b adds
// one to counter b % nsub, and barrier k is complete when every counter i
// holds (k + 1) * sub_count(grid, nsub, i).  One counter makes every
// arrival an atomic on the same address; several let the arrivals proceed
// in parallel at the cost of one load per counter when polling.
L3G_HD inline int barrier_index(int l, int j, int bpl) { return l * bpl + j; }
constexpr int BAR_STRIDE = 32;                      // 32-bit words between counters
constexpr int BAR_MAX_SUB = 16;
constexpr int BAR_ABORT = BAR_MAX_SUB * BAR_STRIDE;  // the step's abort word
constexpr int BAR_WORDS = BAR_ABORT + 1;
// After them: one arrival counter per Q8_0 block of the SwiGLU output (the
// fused act-quant's handshake between the two 32-row groups of a block),
// then one per kv head of the rank (the fused merge's split arrivals).
constexpr int BAR_QCNT = BAR_WORDS;
L3G_HD inline int sub_count(int grid, int nsub, int i) {
  return grid / nsub + (i < grid % nsub ? 1 : 0);
}

// Tiles CTA b consumes in layer l (weights and attention stages) when n
// positions are live; the producer and the consumers walk the same list.
L3G_HD inline int layer_tiles(const Plan& p, int l, int b, int n) {
  int t = 0;
  for (int m = 0; m < N_MAT; ++m) t += my_groups(p, l, m, b) * p.nsl[m];
  int kvh, split;
  if (my_item(p, l, b, &kvh, &split)) {
    int t0, t1;
    item_range(p, split, n, &t0, &t1);
    t += item_stages(p, t0, t1);
  }
  return t;
}

// The plan for one rank: the four layer matrices (rows x cols of this
// rank's shard, in phase order) tiled with four rows per warp, hkv kv heads
// whose caches hold positions of row_bytes, stages of P positions, splits
// per kv head as many as fill the grid (at most one per P positions of the
// workspace's context), the same count as the per-kernel step's global
// merge.  ctx (the state's cache length) is filled per state.  Needs
// grid >= hkv (one item per CTA at least per kv head).
L3G_HD inline Plan make_plan(int grid, int n_layers, const int rows[N_MAT], const int cols[N_MAT],
                             int hkv, int P, int row_bytes, int ws_ctx, int nw, int tile_target) {
  Plan p{};
  p.grid = grid;
  p.n_layers = n_layers;
  for (int m = 0; m < N_MAT; ++m) {
    const TileGeom g = tile_geometry(rows[m], cols[m], 4, nw, tile_target);
    p.ng[m] = g.n_groups;
    p.nsl[m] = g.nslices;
    p.tile_bytes[m] = g.tile_bytes;
    p.wr[m] = g.wr;
    p.ck[m] = g.ck;
    p.rows[m] = rows[m];
    p.cols[m] = cols[m];
  }
  p.hkv = hkv;
  p.P = P;
  p.row_bytes = row_bytes;
  const int by_grid = grid / hkv, by_ctx = (ws_ctx + P - 1) / P;
  p.splits = by_grid < by_ctx ? by_grid : by_ctx;
  if (p.splits < 1) p.splits = 1;
  p.ctx = ws_ctx;
  return p;
}

}  // namespace persist
}  // namespace l3g
