// Host build of libl3g's device kernels under the SIMT emulator, with a C
// entry point per kernel for the CPU tests (ctypes).  Test infrastructure.
#include "simt.h"

#include "simt_tcgen05.h"

// every device kernel of the library, on the emulator's PTX layer
#define L3G_PTX_HEADER "simt_l3g_ptx.h"
#include "l3g_kernels.cuh"

// ---------------------------------------------------------------------------
// C entry points (ctypes).  Pointers named "device" come from emu_malloc.
// Each returns 0, or -1 with the message in emu_error().
// ---------------------------------------------------------------------------
namespace {
std::string g_err;

template <typename F>
int guarded_call(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}
// An identity page table over a contiguous cache [n_layers][hkv][ctx][K|V]
// (ctx a multiple of KV_PAGE): page j of (layer, kv head) h is pool page
// h * pps + j, as the library's private pools map them.  The table lives in
// emulated device memory kept in `keep`.
l3g::KvMap contiguous_kv(void* kv, int n_layers, int hkv, int ctx, int row_bytes,
                         std::vector<void*>& keep) {
  if (ctx % l3g::KV_PAGE) simt::fail("cache length not a multiple of KV_PAGE");
  const int pps = ctx / l3g::KV_PAGE;
  const size_t n = (size_t)n_layers * hkv * pps;
  int* pages = static_cast<int*>(simt::dmalloc(n * sizeof(int)));
  keep.push_back(pages);
  for (size_t i = 0; i < n; ++i) pages[i] = (int)i;
  l3g::KvMap m{};
  m.pool = static_cast<uint8_t*>(kv);
  m.pages = pages;
  m.pps = pps;
  m.hkv = hkv;
  m.row_bytes = row_bytes;
  return m;
}
}  // namespace

extern "C" {

const char* emu_error() { return g_err.c_str(); }

// randomize = 0: round-robin schedule, bulk copies land after one round;
// else a seeded random permutation per round and copy delays up to
// max_copy_delay rounds-ish.
void emu_schedule(int randomize, unsigned long long seed, int max_copy_delay) {
  simt::rt().randomize = randomize != 0;
  simt::rt().rng.seed(seed);
  simt::rt().max_copy_delay = max_copy_delay;
}

void* emu_malloc(unsigned long long bytes) {
  void* p = nullptr;
  guarded_call([&] { p = simt::dmalloc(bytes); });
  return p;
}
void emu_free(void* p) { guarded_call([&] { simt::dfree(p); }); }

// wr, ck, nslices, tile_bytes, n_groups of a matrix tiled with rpw rows per warp
void emu_tile_geometry(int rows, int cols, int rpw, int* out) {
  const l3g::TileGeom g = l3g::tile_geometry(rows, cols, rpw, l3g::NW, l3g::TILE_TARGET);
  out[0] = g.wr;
  out[1] = g.ck;
  out[2] = g.nslices;
  out[3] = g.tile_bytes;
  out[4] = g.n_groups;
}

// k_repack of GGUF Q8_0 rows (device) into the tiled layout (device `out`).
int emu_repack(const void* const* src, const int* src_row0, const int* seg_rows, int nseg,
               int interleave2, int src_blocks, int blk0, int rows, int cols, int rpw, void* out) {
  return guarded_call([&] {
    l3g::RepackArgs a{};
    for (int i = 0; i < nseg && i < 3; ++i) {
      a.src[i] = static_cast<const uint8_t*>(src[i]);
      a.src_row0[i] = src_row0[i];
      a.seg_rows[i] = seg_rows[i];
    }
    a.nseg = nseg;
    a.interleave2 = interleave2;
    a.src_blocks = src_blocks;
    a.blk0 = blk0;
    const l3g::TileGeom g = l3g::tile_geometry(rows, cols, rpw, l3g::NW, l3g::TILE_TARGET);
    a.dst = l3g::Q8Tiles{nullptr, rows, cols, g.wr, g.ck, g.nslices, g.tile_bytes, g.n_groups};
    a.out = static_cast<uint8_t*>(out);
    simt::launch(dim3(4), dim3(128), 0, [&] { l3g::k_repack(a); });
  });
}

// The top-K path's fastExp attention of one layer: k_attf_scores,
// k_attf_values, k_attf_merge as the runtime launches them.
int emu_attf(const float* q, const void* kv, int ctx, int hd, int group, int hkv, int splits,
             int kv_f16, const int* io, float* scores, float* pmax, float* psum, float* po,
             float* out, float* out_d, int8_t* out_q) {
  std::vector<void*> keep;
  const int rc = guarded_call([&] {
    l3g::AttfArgs a{};
    a.q = q;
    a.kv = contiguous_kv(const_cast<void*>(kv), 1, hkv, ctx, 2 * hd * (kv_f16 ? 2 : 4), keep);
    a.layer = 0;
    a.ctx = ctx;
    a.hd = hd;
    a.group = group;
    a.splits = splits;
    a.n_blocks = hkv * group * hd / 32;
    a.scale = (float)(1.0 / sqrt((double)hd));
    a.io = io;
    a.scores = scores;
    a.pmax = pmax;
    a.psum = psum;
    a.po = po;
    a.out = out;
    a.out_d = out_d;
    a.out_q = out_q;
    const dim3 grid(hkv, splits), blk(l3g::ATTF_THREADS);
    const int dpl = hd / 32;
    auto run = [&](auto dpl_c, auto kt) {
      constexpr int D = decltype(dpl_c)::value;
      using KT = decltype(kt);
      simt::launch(grid, blk, sizeof(l3g::AttfScoresSmem), [&] { l3g::k_attf_scores<D, KT>(a); });
      simt::launch(grid, blk, sizeof(l3g::AttfValuesSmem), [&] { l3g::k_attf_values<D, KT>(a); });
    };
    if (kv_f16) {
      if (dpl == 2) run(std::integral_constant<int, 2>{}, __half{});
      else if (dpl == 4) run(std::integral_constant<int, 4>{}, __half{});
      else simt::fail("head dim");
    } else {
      if (dpl == 1) run(std::integral_constant<int, 1>{}, float{});
      else if (dpl == 2) run(std::integral_constant<int, 2>{}, float{});
      else if (dpl == 4) run(std::integral_constant<int, 4>{}, float{});
      else simt::fail("head dim");
    }
    simt::launch(dim3((a.n_blocks + l3g::NW - 1) / l3g::NW), blk, 0, [&] { l3g::k_attf_merge(a); });
  });
  for (void* p : keep) guarded_call([&] { simt::dfree(p); });
  return rc;
}

// One decode step's layers through the persistent kernel, set up as the
// runtime's persist_setup / persist_args do.  Under tensor parallelism each
// rank's record carries its shard's local sizes (hq, hkv, n_ff) and weights.
struct EmuLayers {
  int grid, n_layers, n_emb, n_ff, hq, hkv, hd, rope_half, ctx, kv_f16;
  int fuse_quant, nsub, max_stages, max_splits;
  int launch_grid;           // CTAs actually launched (0: the plan's grid)
  int fuse_merge;            // the split merge in the attention phase
  unsigned long long wait_ns;  // bound of every wait in emulated ns (0: the library's)
  float eps;
  const void* const* w;      // [n_layers * 4] tiled QKV, Wo, up/gate, down (device)
  const float* const* norm;  // [n_layers * 2] attn_norm, ffn_norm (device)
  float* xa;                 // residual stream; the embedding row on entry (device)
  float* xb;                 // residual after the attention block (device)
  float* y;                  // Wo / down output (device)
  float* attn;               // attention output of the last layer (device)
  float* act;                // SwiGLU output of the last layer (device)
  void* kv;                  // cache [n_layers][hkv][ctx][2][hd] (device)
  const float* rope_cos;     // [ctx][rope_half] (device)
  const float* rope_sin;
  int token, pos;
  int step_count;            // the step counter k_embed leaves (tensor-parallel epochs)
  int err, where;            // out: the step's result word
  int splits, stages;        // out: the plan's attention splits and ring slots
};

}  // extern "C"

namespace {
struct RankRun {
  l3g::PersistArgs a{};
  size_t smem = 0;
  std::vector<void*> scratch;
  l3g::Result* res = nullptr;
};

void setup_rank(EmuLayers* e, int world, int rank, unsigned* step,
                unsigned long long* const* recv, RankRun& rr) {
  using namespace l3g;
  const int G = e->hq / e->hkv;
  const int es = e->kv_f16 ? 2 : 4;
  int rows[persist::N_MAT] = {(e->hq + 2 * e->hkv) * e->hd, e->n_emb, 2 * e->n_ff, e->n_emb};
  int cols[persist::N_MAT] = {e->n_emb, e->hq * e->hd, e->n_emb, e->n_ff};
  int P = NW;  // the runtime's stage size: a power of two dividing KV_PAGE
  while (P * 2 <= std::min(KV_PAGE, 32768 / (2 * e->hd * es))) P *= 2;
  persist::Plan p = persist::make_plan(e->grid, e->n_layers, rows, cols, e->hkv, P,
                                       2 * e->hd * es, e->ctx, NW, TILE_TARGET);
  if (e->max_splits >= 1) p.splits = std::min(p.splits, e->max_splits);
  int slot = p.P * p.row_bytes, max_cols = 0;
  for (int m = 0; m < persist::N_MAT; ++m) {
    slot = std::max(slot, p.tile_bytes[m]);
    max_cols = std::max(max_cols, cols[m]);
  }
  PersistArgs& a = rr.a;
  a.plan = p;
  a.slot_bytes = align_up(slot, 128);
  a.xq_off = ps_xq_off(max_cols);
  a.union_bytes = ps_union_bytes(max_cols, G, e->hd, p.splits);
  a.nstages = std::min(MAX_STAGES, (227 * 1024 - PS_HEAD - a.union_bytes) / a.slot_bytes);
  if (e->max_stages >= 2) a.nstages = std::min(a.nstages, e->max_stages);
  if (a.nstages < 2) simt::fail("ring of fewer than two slots");
  rr.smem = PS_HEAD + a.union_bytes + (size_t)a.nstages * a.slot_bytes;
  e->splits = p.splits;
  e->stages = a.nstages;
  auto dm = [&](size_t bytes) {
    void* q = simt::dmalloc(bytes);
    rr.scratch.push_back(q);
    return q;
  };
  auto* layers = static_cast<PersistLayer*>(dm(sizeof(PersistLayer) * e->n_layers));
  for (int l = 0; l < e->n_layers; ++l) {
    for (int m = 0; m < persist::N_MAT; ++m)
      layers[l].w[m] = static_cast<const uint8_t*>(e->w[l * 4 + m]);
    layers[l].attn_norm = e->norm[l * 2];
    layers[l].ffn_norm = e->norm[l * 2 + 1];
  }
  int* io = static_cast<int*>(dm(16));
  io[0] = e->token;
  io[1] = e->pos;
  const int bar_words = persist::BAR_QCNT + e->n_ff / 32 + e->hkv;
  auto* bar = static_cast<unsigned*>(dm(bar_words * 4));  // zeroed, as k_embed leaves it
  rr.res = static_cast<Result*>(dm(sizeof(Result)));
  a.layers = layers;
  a.eps = e->eps;
  a.scale = (float)(1.0 / sqrt((double)e->hd));
  a.n_emb = e->n_emb;
  a.n_ff = e->n_ff;
  a.hq = e->hq;
  a.head_dim = e->hd;
  a.group = G;
  a.rope_half = e->rope_half;
  a.xa = e->xa;
  a.xb = e->xb;
  a.y = e->y;
  a.q = static_cast<float*>(dm((size_t)e->hq * e->hd * 4));
  a.attn = e->attn;
  a.attn_d = static_cast<float*>(dm((size_t)e->hq * e->hd / 32 * 4));
  a.attn_q = static_cast<int8_t*>(dm((size_t)e->hq * e->hd));
  a.act = e->act;
  a.act_d = static_cast<float*>(dm((size_t)e->n_ff / 32 * 4));
  a.act_q = static_cast<int8_t*>(dm((size_t)e->n_ff));
  a.part_o = static_cast<float*>(dm((size_t)e->hkv * p.splits * G * e->hd * 4));
  a.part_ml = static_cast<float*>(dm((size_t)e->hkv * p.splits * G * 2 * 4));
  a.rope_cos = e->rope_cos;
  a.rope_sin = e->rope_sin;
  a.io = io;
  a.kv = contiguous_kv(e->kv, e->n_layers, e->hkv, e->ctx, 2 * e->hd * es, rr.scratch);
  a.bar = bar;
  a.nsub = std::max(1, std::min({e->nsub, (int)persist::BAR_MAX_SUB, p.grid}));
  a.fuse_quant = e->fuse_quant && p.wr[persist::M_UPGATE] == 32 &&
                 p.rows[persist::M_UPGATE] % 64 == 0;
  a.fuse_merge = e->fuse_merge ? 1 : 0;
  a.bpl = persist::barriers_per_layer(a.fuse_quant != 0, a.fuse_merge != 0);
  a.res = rr.res;
  a.wait_ns = e->wait_ns ? e->wait_ns : (world > 1 ? WAIT_TIMEOUT_PEER_NS : WAIT_TIMEOUT_NS);
  a.tp = TpExchange{};
  a.tp.world = world;
  if (world > 1) {  // tp_exchange(ws, 0) of the runtime
    a.tp.rank = rank;
    a.tp.n = e->n_emb;
    a.tp.nphase = 2 * e->n_layers;
    a.tp.phase = 0;
    a.tp.step = step;
    for (int r = 0; r < world; ++r) a.tp.recv[r] = recv[r];
    a.tp.my_recv = recv[rank];
  }
  a.stamps = nullptr;
}

template <int D, typename KT>
void launch_layers(int gp, dim3 grid, size_t smem, std::vector<RankRun>& rr) {
  const bool fm = rr[0].a.fuse_merge != 0;
  auto go = [&](auto gp_c) {
    constexpr int GPc = decltype(gp_c)::value;
    simt::launch(grid, dim3(l3g::NTHREADS), smem, [&] {
      if (fm)
        l3g::k_layers<D, KT, GPc, true>(rr[simt::block_idx().z].a);
      else
        l3g::k_layers<D, KT, GPc, false>(rr[simt::block_idx().z].a);
    });
  };
  switch (gp) {
    case 1: go(std::integral_constant<int, 1>{}); break;
    case 2: go(std::integral_constant<int, 2>{}); break;
    case 4: go(std::integral_constant<int, 4>{}); break;
    case 8: go(std::integral_constant<int, 8>{}); break;
    default: simt::fail("group");
  }
}
}  // namespace

extern "C" {

// `world` ranks (one record each) as one emulated launch whose z index is the
// rank: every rank's CTAs run concurrently, the Wo / down rows pushed into
// every rank's receive buffer and summed in rank order, as on `world` GPUs.
int emu_layers_tp(EmuLayers* ranks, int world) {
  return guarded_call([&] {
    if (world < 1 || world > l3g::MAX_WORLD) simt::fail("world size");
    std::vector<RankRun> rr(world);
    std::vector<void*> shared;
    auto cleanup = [&] {
      for (auto& r : rr)
        for (void* q : r.scratch) simt::dfree(q);
      for (void* q : shared) simt::dfree(q);
    };
    try {
      std::vector<unsigned long long*> recv(world, nullptr);
      std::vector<unsigned*> step(world, nullptr);
      for (int r = 0; r < world; ++r) {
        recv[r] = static_cast<unsigned long long*>(
            simt::dmalloc((size_t)2 * world * ranks[0].n_emb * 8));
        step[r] = static_cast<unsigned*>(simt::dmalloc(4));
        *step[r] = (unsigned)ranks[r].step_count;
        shared.push_back(recv[r]);
        shared.push_back(step[r]);
      }
      size_t smem = 0;
      for (int r = 0; r < world; ++r) {
        setup_rank(&ranks[r], world, r, step[r], recv.data(), rr[r]);
        smem = std::max(smem, rr[r].smem);
      }
      const EmuLayers& e = ranks[0];
      int gp = 1;
      while (gp < e.hq / e.hkv) gp <<= 1;
      const int launched = e.launch_grid > 0 ? e.launch_grid : e.grid;
      const dim3 grid(launched, 1, world);
      const int dpl = e.hd / 32;
      if (e.kv_f16) {
        if (dpl == 2) launch_layers<2, __half>(gp, grid, smem, rr);
        else if (dpl == 4) launch_layers<4, __half>(gp, grid, smem, rr);
        else simt::fail("head dim");
      } else {
        if (dpl == 1) launch_layers<1, float>(gp, grid, smem, rr);
        else if (dpl == 2) launch_layers<2, float>(gp, grid, smem, rr);
        else if (dpl == 4) launch_layers<4, float>(gp, grid, smem, rr);
        else simt::fail("head dim");
      }
      for (int r = 0; r < world; ++r) {
        ranks[r].err = rr[r].res->err;
        ranks[r].where = rr[r].res->where;
      }
    } catch (...) {
      cleanup();
      throw;
    }
    cleanup();
  });
}

int emu_layers(EmuLayers* e) { return emu_layers_tp(e, 1); }

// The runtime's gemm_ksplit: with fewer (row tile, token tile) tiles than
// SMs, split K over a divisor of the chunk count that fits `part_floats`.
static int emu_ksplit(int rows, int cols, int n_tok, int nsm, size_t part_floats) {
  using namespace l3g;
  const int nt = gemm::token_tile(n_tok), nk = gemm::chunks(cols);
  const long long tiles = (long long)gemm::row_tiles(rows) * ((n_tok + nt - 1) / nt);
  if (part_floats == 0 || tiles >= nsm) return 1;
  const long long want = nsm / tiles;
  int best = 1;
  for (int d = 2; d <= nk && d <= want; ++d)
    if (nk % d == 0 && (size_t)d * n_tok * rows <= part_floats) best = d;
  return best;
}

// One product as the runtime's launch_gemm issues it (ldo = rows).
static void run_gemm(const uint8_t* w, int rows, int cols, const uint8_t* act, int n_tok,
                     float* out, int ksplit, float* part, int grid, int nstages, l3g::Result* res,
                     int nsm = 148) {
  using namespace l3g;
  const int nt = gemm::token_tile(n_tok);
  GemmArgs g{};
  g.a = w;
  g.b = act;
  g.out = out;
  g.rows = rows;
  g.ldo = rows;
  g.n_tok = n_tok;
  g.nk = gemm::chunks(cols);
  g.n_rt = gemm::row_tiles(rows);
  g.n_tt = (n_tok + nt - 1) / nt;
  g.ksplit = ksplit > 1 ? ksplit : 1;
  if (g.nk % g.ksplit) simt::fail("ksplit must divide the chunk count");
  g.part = part;
  g.nstages = nstages > 0 ? std::min(nstages, gemm::stages(nt)) : gemm::stages(nt);
  g.res = res;
  g.wait_ns = WAIT_TIMEOUT_NS;
  const long long units = (long long)g.n_rt * g.n_tt * g.ksplit;
  const int G = grid > 0 ? grid : (int)std::max<long long>(1, std::min<long long>(nsm, units));
  const size_t smem = gemm::SMEM_HEAD + (size_t)g.nstages * gemm::stage_bytes(nt);
  auto go = [&](auto nt_c) {
    constexpr int NT = decltype(nt_c)::value;
    simt::launch(dim3(G), dim3(gemm_threads(NT)), smem, [&] { k_gemm_q8<NT>(g); });
  };
  switch (nt) {
    case 16: go(std::integral_constant<int, 16>{}); break;
    case 32: go(std::integral_constant<int, 32>{}); break;
    case 64: go(std::integral_constant<int, 64>{}); break;
    default: go(std::integral_constant<int, 128>{}); break;
  }
  if (g.ksplit > 1) {
    const long long n = (long long)n_tok * rows;
    simt::launch(dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                 [&] { k_gemm_reduce(part, g.ksplit, n_tok, rows, rows, out); });
  }
}

// k_gemm_quantize of x [n_tok][cols] (device) into activation chunks for a
// token tile of token_tile(n_tok) (device `act`, l3g_gemm_act_bytes bytes).
int emu_gemm_quantize(const float* x, int n_tok, int cols, uint8_t* act) {
  return guarded_call([&] {
    using namespace l3g;
    const int nt = gemm::token_tile(n_tok), nk = gemm::chunks(cols);
    const int n_pad = (n_tok + nt - 1) / nt * nt;
    const long long warps = (long long)n_pad * nk * gemm::BPC;
    simt::launch(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
                 [&] { k_gemm_quantize(x, n_tok, cols, nt, nk, n_pad, act); });
  });
}

// The batched Q8_0 product as the runtime's launch_gemm issues it: weight
// chunks w (device, rows x cols repacked), activation chunks act, out
// [n_tok][rows]; ksplit > 1 splits K over CTAs into `part` and reduces.
// grid 0 takes min(148, units); nstages 0 the layout's ring depth.
int emu_gemm(const uint8_t* w, int rows, int cols, const uint8_t* act, int n_tok, float* out,
             int ksplit, float* part, int grid, int nstages, int* err, int* where) {
  return guarded_call([&] {
    auto* res = static_cast<l3g::Result*>(simt::dmalloc(sizeof(l3g::Result)));
    try {
      run_gemm(w, rows, cols, act, n_tok, out, ksplit, part, grid, nstages, res);
    } catch (...) {
      simt::dfree(res);
      throw;
    }
    *err = res->err;
    *where = res->where;
    simt::dfree(res);
  });
}

// k_gemm_from_tiles: weight chunks (device dst, zeroed) of a matrix held in
// the decode kernels' tile layout with rpw rows per warp (device src).
int emu_gemm_from_tiles(const uint8_t* src, int rows, int cols, int rpw, uint8_t* dst) {
  return guarded_call([&] {
    const l3g::TileGeom g = l3g::tile_geometry(rows, cols, rpw, l3g::NW, l3g::TILE_TARGET);
    const l3g::Q8Tiles t{src, rows, cols, g.wr, g.ck, g.nslices, g.tile_bytes, g.n_groups};
    simt::launch(dim3(8), dim3(256), 0, [&] { l3g::k_gemm_from_tiles(t, dst); });
  });
}

// One batched prefill pass of P tokens at positions pos0.. as the runtime's
// enqueue_prefill_pass issues it on one GPU.
struct EmuPrefillLayer {
  const uint8_t* g[4];  // weight chunks of QKV, Wo, up/gate (interleaved), down (device)
  const float* attn_norm;
  const float* ffn_norm;
};
struct EmuPrefill {
  int n_layers, n_emb, n_ff, hq, hkv, hd, rope_half, ctx, kv_f16, vocab;
  float eps;
  const EmuPrefillLayer* layers;  // host array of n_layers
  const uint8_t* emb;             // raw GGUF token_embd (device)
  void* kv;                       // cache [n_layers][hkv][ctx][2][hd] (device)
  const float* rope_cos;          // [ctx][rope_half] (device)
  const float* rope_sin;
  const int* ids;                 // P token ids (device)
  int P, pos0, nsm;
  int err, where;
};

int emu_prefill(EmuPrefill* e) {
  return guarded_call([&] {
    using namespace l3g;
    const int ne = e->n_emb, hd = e->hd, P = e->P;
    const int nq = e->hq * hd, nkv = e->hkv * hd, ff = e->n_ff, G = e->hq / e->hkv;
    const int es = e->kv_f16 ? 2 : 4;
    const int nt = gemm::token_tile(P);
    const int rows[4] = {nq + 2 * nkv, ne, 2 * ff, ne}, cols[4] = {ne, nq, ne, ff};
    std::vector<void*> scratch;
    auto dm = [&](size_t bytes) {
      void* q = simt::dmalloc(bytes);
      scratch.push_back(q);
      return q;
    };
    try {
      const int cap = P;
      const int max_cols = std::max(std::max(ne, nq), ff);
      const int ntc = gemm::token_tile(cap);
      const size_t act_bytes =
          (size_t)((cap + ntc - 1) / ntc) * gemm::chunks(max_cols) * gemm::b_chunk(ntc);
      auto* X = static_cast<float*>(dm((size_t)cap * ne * 4));
      auto* Y = static_cast<float*>(dm((size_t)cap * ne * 4));
      auto* QKV = static_cast<float*>(dm((size_t)cap * (nq + 2 * nkv) * 4));
      auto* Q = static_cast<float*>(dm((size_t)cap * nq * 4));
      auto* ATT = static_cast<float*>(dm((size_t)cap * nq * 4));
      auto* UG = static_cast<float*>(dm((size_t)cap * 2 * ff * 4));
      auto* act = static_cast<uint8_t*>(dm(act_bytes));
      size_t part_floats = 0;  // gemm_part_bound over the matrices
      for (int m = 0; m < 4; ++m) {
        const long long d = std::min<long long>(
            gemm::chunks(cols[m]), std::max(1, e->nsm / std::max(1, gemm::row_tiles(rows[m]))));
        if (d > 1) part_floats = std::max(part_floats, (size_t)d * cap * rows[m]);
      }
      auto* part = static_cast<float*>(dm(std::max<size_t>(1, part_floats) * 4));
      auto* res = static_cast<Result*>(dm(sizeof(Result)));
      const KvMap kvm = contiguous_kv(e->kv, e->n_layers, e->hkv, e->ctx, 2 * hd * es, scratch);
      auto gemm = [&](int l, int m, float* out) {
        const int ks = emu_ksplit(rows[m], cols[m], P, e->nsm, part_floats);
        run_gemm(e->layers[l].g[m], rows[m], cols[m], act, P, out, ks, part, 0, 0, res, e->nsm);
      };
      simt::launch(dim3((ne + 255) / 256, P), dim3(256), 0,
                   [&] { k_pf_embed(e->emb, e->vocab, ne, e->ids, X, res); });
      for (int l = 0; l < e->n_layers; ++l) {
        const EmuPrefillLayer& L = e->layers[l];
        const KvMap kv = kvm;
        simt::launch(dim3(P), dim3(PF_THREADS), 0, [&] {
          k_pf_rms_quant(X, l ? Y : nullptr, L.attn_norm, e->eps, ne, nt, gemm::chunks(ne), act);
        }, true);
        gemm(l, 0, QKV);
        const long long pairs = (long long)P * ((nq + 2 * nkv) / 2);
        simt::launch(dim3((unsigned)((pairs + 255) / 256)), dim3(256), 0, [&] {
          k_pf_qkv_rope(QKV, P, e->pos0, nq, nkv, hd, e->rope_half, e->rope_cos, e->rope_sin, Q,
                        kv, l, e->kv_f16);
        });
        if (l == e->n_layers - 1) break;
        {
          const int bq = std::max(1, 64 / G);
          const dim3 grid((P + bq - 1) / bq, e->hkv);
          const float scale = (float)(1.0 / sqrt((double)hd));
          auto att = [&](auto hd_c) {
            constexpr int HD = decltype(hd_c)::value;
            if (e->kv_f16)
              simt::launch(grid, dim3(256), pf_attention_smem(HD), [&] {
                k_pf_attention<HD, __half>(Q, kv, l, ATT, P, e->pos0, G, bq, e->hq, scale);
              });
            else
              simt::launch(grid, dim3(256), pf_attention_smem(HD), [&] {
                k_pf_attention<HD, float>(Q, kv, l, ATT, P, e->pos0, G, bq, e->hq, scale);
              });
          };
          switch (hd) {
            case 32: att(std::integral_constant<int, 32>{}); break;
            case 64: att(std::integral_constant<int, 64>{}); break;
            case 128: att(std::integral_constant<int, 128>{}); break;
            default: simt::fail("head dim");
          }
        }
        {
          const int n_pad = (P + nt - 1) / nt * nt;
          const long long warps = (long long)n_pad * gemm::chunks(nq) * gemm::BPC;
          simt::launch(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, [&] {
            k_gemm_quantize(ATT, P, nq, nt, gemm::chunks(nq), n_pad, act);
          });
        }
        gemm(l, 1, Y);
        simt::launch(dim3(P), dim3(PF_THREADS), 0, [&] {
          k_pf_rms_quant(X, Y, L.ffn_norm, e->eps, ne, nt, gemm::chunks(ne), act);
        }, true);
        gemm(l, 2, UG);
        {
          const long long warps = (long long)P * (ff / 32);
          simt::launch(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
                       [&] { k_pf_swiglu_quant(UG, P, ff, nt, gemm::chunks(ff), act); });
        }
        gemm(l, 3, Y);
      }
      e->err = res->err;
      e->where = res->where;
    } catch (...) {
      for (void* q : scratch) simt::dfree(q);
      throw;
    }
    for (void* q : scratch) simt::dfree(q);
  });
}

// One batched decode step of n sessions as the runtime's l3g_batch_step
// issues it on one GPU (embedding, per layer RMSNorm + act-quant, QKV
// product, RoPE + KV append per session, split-K attention over each
// session's cache and its merge, Wo, FFN; final norm, logits product,
// top-K and SampleTopK per session).
struct EmuBatch {
  int n_layers, n_emb, n_ff, hq, hkv, hd, rope_half, kv_f16, vocab;
  float eps;
  const EmuPrefillLayer* layers;  // host array of n_layers (weight chunks)
  const uint8_t* glogits;         // logits matrix as weight chunks (device)
  const float* out_norm;          // (device)
  const uint8_t* emb;             // raw GGUF token_embd (device)
  l3g::SeqInfo* seqs;             // [n] (device)
  int n, max_splits, top_k, nsm;
  float* logits;                  // out: [n][vocab] (device)
  l3g::Result* out;               // out: [n] sampled token and its logit (device)
  int err, where;
};

int emu_batch_step(EmuBatch* e) {
  return guarded_call([&] {
    using namespace l3g;
    const int ne = e->n_emb, hd = e->hd, n = e->n;
    const int nq = e->hq * hd, nkv = e->hkv * hd, ff = e->n_ff, G = e->hq / e->hkv;
    const int nt = gemm::token_tile(n), n_pad = (n + nt - 1) / nt * nt;
    const int rows[5] = {nq + 2 * nkv, ne, 2 * ff, ne, e->vocab};
    const int cols[5] = {ne, nq, ne, ff, ne};
    std::vector<void*> scratch;
    auto dm = [&](size_t bytes) {
      void* q = simt::dmalloc(bytes);
      scratch.push_back(q);
      return q;
    };
    try {
      int max_pos = 0;
      for (int i = 0; i < n; ++i) max_pos = std::max(max_pos, e->seqs[i].pos);
      const int splits = (max_pos + 1 + BD_SPLIT - 1) / BD_SPLIT;
      if (splits > e->max_splits) simt::fail("max_splits too small");
      const int max_cols = std::max(std::max(ne, nq), ff);
      const size_t act_bytes = (size_t)(n_pad / nt) * gemm::chunks(max_cols) * gemm::b_chunk(nt);
      auto* X = static_cast<float*>(dm((size_t)n * ne * 4));
      auto* Y = static_cast<float*>(dm((size_t)n * ne * 4));
      auto* QKV = static_cast<float*>(dm((size_t)n * (nq + 2 * nkv) * 4));
      auto* Q = static_cast<float*>(dm((size_t)n * nq * 4));
      auto* ATT = static_cast<float*>(dm((size_t)n * nq * 4));
      auto* UG = static_cast<float*>(dm((size_t)n * 2 * ff * 4));
      auto* part_o = static_cast<float*>(dm((size_t)n * e->hq * e->max_splits * hd * 4));
      auto* part_ml = static_cast<float*>(dm((size_t)n * e->hq * e->max_splits * 2 * 4));
      auto* act = static_cast<uint8_t*>(dm(act_bytes));
      size_t part_floats = 0;
      for (int m = 0; m < 5; ++m) {
        const long long d = std::min<long long>(
            gemm::chunks(cols[m]), std::max(1, e->nsm / std::max(1, gemm::row_tiles(rows[m]))));
        if (d > 1) part_floats = std::max(part_floats, (size_t)d * n * rows[m]);
      }
      auto* part = static_cast<float*>(dm(std::max<size_t>(1, part_floats) * 4));
      const int tk_chunks = (e->vocab + TOPK_CHUNK - 1) / TOPK_CHUNK;
      auto* tk_part = static_cast<uint64_t*>(dm((size_t)n * tk_chunks * MAX_TOPK * 8));
      auto* tk_ids = static_cast<int*>(dm((size_t)n * MAX_TOPK * 4));
      auto* tk_logits = static_cast<float*>(dm((size_t)n * MAX_TOPK * 4));
      auto* res = static_cast<Result*>(dm(sizeof(Result)));
      auto gemm = [&](const uint8_t* w, int m, float* out) {
        const int ks = emu_ksplit(rows[m], cols[m], n, e->nsm, part_floats);
        run_gemm(w, rows[m], cols[m], act, n, out, ks, part, 0, 0, res, e->nsm);
      };
      const float scale = (float)(1.0 / sqrt((double)hd));
      simt::launch(dim3((ne + 255) / 256, n), dim3(256), 0,
                   [&] { k_bd_embed(e->emb, e->vocab, ne, e->seqs, X, res); });
      for (int l = 0; l < e->n_layers; ++l) {
        const EmuPrefillLayer& L = e->layers[l];
        simt::launch(dim3(n), dim3(PF_THREADS), 0, [&] {
          k_pf_rms_quant(X, l ? Y : nullptr, L.attn_norm, e->eps, ne, nt, gemm::chunks(ne), act);
        }, true);
        gemm(L.g[0], 0, QKV);
        const long long pairs = (long long)n * ((nq + 2 * nkv) / 2);
        simt::launch(dim3((unsigned)((pairs + 255) / 256)), dim3(256), 0, [&] {
          k_bd_qkv_rope(QKV, n, e->seqs, l, nq, nkv, hd, e->rope_half, Q, e->kv_f16);
        });
        {
          const dim3 grid(splits, e->hkv, n);
          const int gp = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
          auto att = [&](auto hd_c, auto gp_c, auto kt) {
            constexpr int HD = decltype(hd_c)::value, GPc = decltype(gp_c)::value;
            using KT = decltype(kt);
            simt::launch(grid, dim3(BD_THREADS), bd_smem_bytes(HD, (int)sizeof(KT), GPc), [&] {
              k_bd_attention<HD, GPc, KT>(Q, e->seqs, l, G, e->hq, scale, part_o, part_ml,
                                          e->max_splits, BD_SPLIT, res, WAIT_TIMEOUT_NS);
            });
          };
          auto by_gp = [&](auto hd_c, auto kt) {
            switch (gp) {
              case 1: att(hd_c, std::integral_constant<int, 1>{}, kt); break;
              case 2: att(hd_c, std::integral_constant<int, 2>{}, kt); break;
              case 4: att(hd_c, std::integral_constant<int, 4>{}, kt); break;
              default: att(hd_c, std::integral_constant<int, 8>{}, kt); break;
            }
          };
          auto by_kt = [&](auto hd_c) {
            if (e->kv_f16) by_gp(hd_c, __half{});
            else by_gp(hd_c, float{});
          };
          switch (hd) {
            case 32: by_kt(std::integral_constant<int, 32>{}); break;
            case 64: by_kt(std::integral_constant<int, 64>{}); break;
            case 128: by_kt(std::integral_constant<int, 128>{}); break;
            default: simt::fail("head dim");
          }
          simt::launch(dim3(e->hq, n), dim3(128), 0, [&] {
            k_bd_merge(part_o, part_ml, e->seqs, e->hq, hd, e->max_splits, BD_SPLIT, ATT);
          });
        }
        {
          const long long warps = (long long)n_pad * gemm::chunks(nq) * gemm::BPC;
          simt::launch(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, [&] {
            k_gemm_quantize(ATT, n, nq, nt, gemm::chunks(nq), n_pad, act);
          });
        }
        gemm(L.g[1], 1, Y);
        simt::launch(dim3(n), dim3(PF_THREADS), 0, [&] {
          k_pf_rms_quant(X, Y, L.ffn_norm, e->eps, ne, nt, gemm::chunks(ne), act);
        }, true);
        gemm(L.g[2], 2, UG);
        {
          const long long warps = (long long)n * (ff / 32);
          simt::launch(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
                       [&] { k_pf_swiglu_quant(UG, n, ff, nt, gemm::chunks(ff), act); });
        }
        gemm(L.g[3], 3, Y);
      }
      simt::launch(dim3(n), dim3(PF_THREADS), 0, [&] {
        k_pf_rms_quant(X, Y, e->out_norm, e->eps, ne, nt, gemm::chunks(ne), act);
      }, true);
      gemm(e->glogits, 4, e->logits);
      simt::launch(dim3(tk_chunks, n), dim3(256), 0, [&] {
        k_bd_topk_partial(e->logits, n, e->vocab, e->vocab, e->top_k, tk_part);
      }, true);
      {
        const int count = tk_chunks * e->top_k;
        int cap2 = 1;
        while (cap2 < count) cap2 <<= 1;
        simt::launch(dim3(n), dim3(256), (size_t)cap2 * 8, [&] {
          k_bd_topk_final(tk_part, count, cap2, e->top_k, tk_ids, tk_logits);
        });
      }
      simt::launch(dim3(n), dim3(32), 0,
                   [&] { k_bd_sample(tk_ids, tk_logits, e->top_k, e->seqs, e->out); }, true);
      e->err = res->err;
      e->where = res->where;
    } catch (...) {
      for (void* q : scratch) simt::dfree(q);
      throw;
    }
    for (void* q : scratch) simt::dfree(q);
  });
}

// The decode step's Q8_0 matvec as the per-op entry l3g_matvec_q8 launches
// it (k_matvec, pre-quantized activation, plain store of rows [row_lo,
// row_hi)) on tiles with rpw rows per warp; ring depth as the runtime's
// finish_plan picks it; grid min(row groups, nsm).
int emu_matvec(const uint8_t* tiles, int rows, int cols, int rpw, const float* xd,
               const int8_t* xq, float* out, int row_lo, int row_hi, int nsm) {
  return guarded_call([&] {
    using namespace l3g;
    const TileGeom g = tile_geometry(rows, cols, rpw, NW, TILE_TARGET);
    MatvecArgs a{};
    a.w = Q8Tiles{tiles, rows, cols, g.wr, g.ck, g.nslices, g.tile_bytes, g.n_groups};
    const int fixed = mv_smem_bytes(cols, 0, g.tile_bytes);
    a.nstages = std::max(2, std::min(MAX_STAGES, (CTA_SMEM_SHARE - fixed) / g.tile_bytes));
    const size_t smem = mv_smem_bytes(cols, a.nstages, g.tile_bytes);
    a.row_lo = row_lo;
    a.row_hi = row_hi;
    a.xd_in = xd;
    a.xqs_in = xq;
    a.out = out;
    auto* res = static_cast<Result*>(simt::dmalloc(sizeof(Result)));
    a.res = res;
    a.wait_ns = WAIT_TIMEOUT_NS;
    const int gl = row_lo / g.wr, ng = (row_hi + g.wr - 1) / g.wr - gl;
    const dim3 grid(std::max(1, std::min(ng, nsm)));
    try {
      auto go = [&](auto r_c) {
        constexpr int R = decltype(r_c)::value;
        simt::launch(grid, dim3(NTHREADS), smem, [&] { k_matvec<PRO_PREQ, EPI_STORE, R, 1>(a); });
      };
      switch (rpw) {
        case 1: go(std::integral_constant<int, 1>{}); break;
        case 2: go(std::integral_constant<int, 2>{}); break;
        case 4: go(std::integral_constant<int, 4>{}); break;
        case 8: go(std::integral_constant<int, 8>{}); break;
        default: simt::fail("rows per warp");
      }
      if (res->err) simt::fail("k_matvec reported an error");
    } catch (...) {
      simt::dfree(res);
      throw;
    }
    simt::dfree(res);
  });
}

// k_matvec with a fused epilogue on a pre-quantized activation, grid CTAs:
//  epi 0 (EPI_STORE): out[r];
//  epi 3 (EPI_LOGITS): out[r] (or no store when out is null) and the argmax
//    through per-CTA slots am_val / am_idx and the arrival counter
//    am_counter, into *result (index, value, status, detail), as
//    l3g_matvec_q8_argmax_static runs it on its static scratch.
int emu_matvec_epi(const uint8_t* tiles, int rows, int cols, int rpw, const float* xd,
                   const int8_t* xq, float* out, int epi, float* am_val, int* am_idx,
                   unsigned* am_counter, int* result, int grid) {
  return guarded_call([&] {
    using namespace l3g;
    const TileGeom g = tile_geometry(rows, cols, rpw, NW, TILE_TARGET);
    MatvecArgs a{};
    a.w = Q8Tiles{tiles, rows, cols, g.wr, g.ck, g.nslices, g.tile_bytes, g.n_groups};
    const int fixed = mv_smem_bytes(cols, 0, g.tile_bytes);
    a.nstages = std::max(2, std::min(MAX_STAGES, (CTA_SMEM_SHARE - fixed) / g.tile_bytes));
    const size_t smem = mv_smem_bytes(cols, a.nstages, g.tile_bytes);
    a.row_lo = 0;
    a.row_hi = rows;
    a.xd_in = xd;
    a.xqs_in = xq;
    a.out = out;
    a.am_val = am_val;
    a.am_idx = am_idx;
    a.am_counter = am_counter;
    a.res = reinterpret_cast<Result*>(result);
    a.wait_ns = WAIT_TIMEOUT_NS;
    auto go = [&](auto r_c, auto e_c) {
      constexpr int R = decltype(r_c)::value;
      constexpr int E = decltype(e_c)::value;
      simt::launch(dim3(grid), dim3(NTHREADS), smem, [&] { k_matvec<PRO_PREQ, E, R, 1>(a); });
    };
    auto by_rpw = [&](auto e_c) {
      switch (rpw) {
        case 1: go(std::integral_constant<int, 1>{}, e_c); break;
        case 2: go(std::integral_constant<int, 2>{}, e_c); break;
        case 4: go(std::integral_constant<int, 4>{}, e_c); break;
        case 8: go(std::integral_constant<int, 8>{}, e_c); break;
        default: simt::fail("rows per warp");
      }
    };
    if (epi == EPI_LOGITS) by_rpw(std::integral_constant<int, EPI_LOGITS>{});
    else if (epi == EPI_STORE) by_rpw(std::integral_constant<int, EPI_STORE>{});
    else simt::fail("epilogue");
  });
}

// bitonic_desc (the top-K kernels' sort) of n keys by one block of `threads`
// threads, in shared memory; keys sorted in place (device).
int emu_bitonic(unsigned long long* keys, int n, int threads) {
  return guarded_call([&] {
    using namespace l3g;
    simt::launch(dim3(1), dim3(threads), (size_t)n * 8, [&] {
      L3G_DYNAMIC_SMEM(raw);
      uint64_t* k = reinterpret_cast<uint64_t*>(raw);
      for (int i = threadIdx.x; i < n; i += blockDim.x) k[i] = keys[i];
      __syncthreads();
      bitonic_desc(k, n);
      for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = k[i];
    });
  });
}

// The decode step's split-K attention (k_attention, global merge through
// partials in device memory, the CTAs of a kv head waiting on each other's
// arrival counters) for one layer, set up as l3g_workspace_new and
// enqueue_step do: P positions per stage, nstages stages (the runtime's 4 at
// one GPU, 6 under tensor parallelism), splits filling nsm.
int emu_attention(const float* q, const void* kv, int ctx, int hd, int group, int hkv, int kv_f16,
                  const int* io, float* out, float* out_d, int8_t* out_q, int nsm, int nstages,
                  int* splits_out) {
  return guarded_call([&] {
    using namespace l3g;
    const int es = kv_f16 ? 2 : 4;
    AttnArgs a{};
    a.P = NW;  // the runtime's stage size: a power of two dividing KV_PAGE
    while (a.P * 2 <= std::min(KV_PAGE, (int)(32768 / (2 * hd * es)))) a.P *= 2;
    a.stage_bytes = 2 * a.P * hd * es;
    if (nstages < 2 || nstages > 6) simt::fail("stages outside 2..6");
    a.nstages = nstages;
    a.n_splits = std::max(1, std::min(nsm / hkv, (ctx + a.P - 1) / a.P));
    *splits_out = a.n_splits;
    int gp = 1;
    while (gp < group) gp <<= 1;
    const int scratch = std::max(at_scratch_floats(group, hd) * 4, NW * align_up(a.n_splits, 32) * 4);
    const size_t smem = at_ring_offset() + std::max(a.nstages * a.stage_bytes, scratch);
    std::vector<void*> sc;
    auto dm = [&](size_t bytes) {
      void* p = simt::dmalloc(bytes);
      sc.push_back(p);
      return p;
    };
    a.wait_ns = WAIT_TIMEOUT_NS;
    a.q = q;
    a.kv = contiguous_kv(const_cast<void*>(kv), 1, hkv, ctx, 2 * hd * es, sc);
    a.layer = 0;
    a.hd = hd;
    a.group = group;
    a.scale = (float)(1.0 / sqrt((double)hd));
    a.io = io;
    a.part_o = static_cast<float*>(dm((size_t)hkv * a.n_splits * group * hd * 4));
    a.part_ml = static_cast<float*>(dm((size_t)hkv * a.n_splits * group * 2 * 4));
    a.counters = static_cast<unsigned*>(dm((size_t)hkv * 2 * 4));
    a.out = out;
    a.out_d = out_d;
    a.out_q = out_q;
    a.res = static_cast<Result*>(dm(sizeof(Result)));
    const dim3 grid(hkv, a.n_splits);
    try {
      auto go = [&](auto dpl_c, auto kt, auto gp_c) {
        constexpr int D = decltype(dpl_c)::value, GPc = decltype(gp_c)::value;
        using KT = decltype(kt);
        simt::launch(grid, dim3(NTHREADS), smem, [&] { k_attention<D, KT, GPc, false>(a); });
      };
      auto by_gp = [&](auto dpl_c, auto kt) {
        switch (gp) {
          case 1: go(dpl_c, kt, std::integral_constant<int, 1>{}); break;
          case 2: go(dpl_c, kt, std::integral_constant<int, 2>{}); break;
          case 4: go(dpl_c, kt, std::integral_constant<int, 4>{}); break;
          default: go(dpl_c, kt, std::integral_constant<int, 8>{}); break;
        }
      };
      const int dpl = hd / 32;
      if (kv_f16) {
        if (dpl == 2) by_gp(std::integral_constant<int, 2>{}, __half{});
        else by_gp(std::integral_constant<int, 4>{}, __half{});
      } else {
        if (dpl == 1) by_gp(std::integral_constant<int, 1>{}, float{});
        else if (dpl == 2) by_gp(std::integral_constant<int, 2>{}, float{});
        else by_gp(std::integral_constant<int, 4>{}, float{});
      }
      if (a.res->err) simt::fail("k_attention reported an error");
      for (int i = 0; i < 2 * hkv; ++i)
        if (a.counters[i]) simt::fail("k_attention left its counters non-zero");
    } catch (...) {
      for (void* p : sc) simt::dfree(p);
      throw;
    }
    for (void* p : sc) simt::dfree(p);
  });
}

}  // extern "C"
