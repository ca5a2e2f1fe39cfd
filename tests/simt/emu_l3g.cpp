// Host build of libl3g's device kernels under the SIMT emulator, with a C
// entry point per kernel for the CPU tests (ctypes).  Test infrastructure.
#include "simt.h"

#include "l3g_persist_plan.h"

namespace l3g {
#include "l3g_base.cuh"

#include "simt_ptx.h"

#include "l3g_helpers.cuh"

#include "l3g_matvec.cuh"

#include "l3g_attention.cuh"

#include "l3g_attention_fast.cuh"

#include "l3g_persist.cuh"

#include "l3g_repack.cuh"
}  // namespace l3g

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
  return guarded_call([&] {
    l3g::AttfArgs a{};
    a.q = q;
    a.kv = kv;
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
}

// One decode step's layers through the persistent kernel, set up as the
// runtime's persist_setup / persist_args do.  Under tensor parallelism each
// rank's record carries its shard's local sizes (hq, hkv, n_ff) and weights.
struct EmuLayers {
  int grid, n_layers, n_emb, n_ff, hq, hkv, hd, rope_half, ctx, kv_f16;
  int fuse_quant, nsub, max_stages, max_splits;
  int launch_grid;           // CTAs actually launched (0: the plan's grid)
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
  const int P = std::max(NW, 32768 / (2 * e->hd * es));
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
  const int bar_words = persist::BAR_QCNT + e->n_ff / 32;
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
  a.kv = static_cast<uint8_t*>(e->kv);
  a.kv_layer_bytes = (size_t)e->hkv * e->ctx * 2 * e->hd * es;
  a.bar = bar;
  a.nsub = std::max(1, std::min({e->nsub, (int)persist::BAR_MAX_SUB, p.grid}));
  a.fuse_quant = e->fuse_quant && p.wr[persist::M_UPGATE] == 32 &&
                 p.rows[persist::M_UPGATE] % 64 == 0;
  a.bpl = persist::barriers_per_layer(a.fuse_quant != 0);
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
  auto go = [&](auto gp_c) {
    constexpr int GPc = decltype(gp_c)::value;
    simt::launch(grid, dim3(l3g::NTHREADS), smem,
                 [&] { l3g::k_layers<D, KT, GPc>(rr[simt::block_idx().z].a); });
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

}  // extern "C"
