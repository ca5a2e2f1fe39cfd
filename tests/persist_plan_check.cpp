// Host-only check of the persistent layer kernel's work schedule
// (llama3.go_b200/csrc/l3g_persist_plan.h), compiled with g++ by
// tests/test_persist_plan.py.  For each shape, rank count, grid size and KV
// element size it builds the plan exactly as the library does (make_plan)
// and checks, for several layers and live position counts:
//   - every tile (row group, column slice) of the four layer matrices is
//     taken by exactly one CTA, and every tile lies inside its matrix;
//   - every (kv head, split) attention item is taken by exactly one CTA,
//     and the splits of a kv head cover positions [0, n) in order without
//     gaps or overlap, in stages of at most P positions that stay inside
//     that kv head's cache rows;
//   - the per-CTA tile counts (layer_tiles) add up to the matrices' tiles
//     plus the attention stages;
//   - the barrier targets fit 32 bits.
// It prints one line per plan (tiles per CTA per layer: min, mean, max) and
// exits non-zero on the first failure.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "l3g_persist_plan.h"

using namespace l3g;
using namespace l3g::persist;

namespace {

int g_fail = 0;
#define CHECK(cond, ...)                       \
  do {                                         \
    if (!(cond)) {                             \
      std::fprintf(stderr, "FAIL %s: ", #cond); \
      std::fprintf(stderr, __VA_ARGS__);       \
      std::fprintf(stderr, "\n");              \
      g_fail = 1;                              \
      return false;                            \
    }                                          \
  } while (0)

struct Shape {
  const char* name;
  int n_emb, n_layers, heads, kv_heads, n_ff;
};

bool check_plan(const Plan& p, const char* tag) {
  const int G = p.grid;
  CHECK(p.hkv * p.splits <= G, "%s: %d items on %d CTAs", tag, p.hkv * p.splits, G);
  CHECK((long long)(BARRIERS_PER_LAYER * p.n_layers + 1) * G < (1ll << 32), "%s: barrier count", tag);
  CHECK(barrier_index(p.n_layers - 1, barriers_per_layer(false) - 1, barriers_per_layer(false)) <
            BARRIERS_PER_LAYER * p.n_layers, "%s: barrier index", tag);
  const int layers[3] = {0, p.n_layers > 1 ? 1 : 0, p.n_layers - 1};
  const int ns[5] = {1, p.P, p.P + 1, p.ctx / 2 + 3, p.ctx};
  for (int li = 0; li < 3; ++li) {
    const int l = layers[li];
    long long mat_tiles = 0;
    for (int m = 0; m < N_MAT; ++m) {
      std::vector<int> seen(p.ng[m], 0);
      for (int b = 0; b < G; ++b) {
        const int k_n = my_groups(p, l, m, b);
        for (int k = 0; k < k_n; ++k) {
          const int g = my_group(p, l, m, b, k);
          CHECK(g >= 0 && g < p.ng[m], "%s: layer %d mat %d cta %d group %d of %d", tag, l, m, b, g,
                p.ng[m]);
          ++seen[g];
          const long long end = tile_offset(p, m, g, p.nsl[m] - 1) + p.tile_bytes[m];
          CHECK(end <= (long long)p.ng[m] * p.nsl[m] * p.tile_bytes[m], "%s: tile past matrix", tag);
        }
      }
      for (int g = 0; g < p.ng[m]; ++g)
        CHECK(seen[g] == 1, "%s: layer %d mat %d group %d taken %d times", tag, l, m, g, seen[g]);
      mat_tiles += (long long)p.ng[m] * p.nsl[m];
      CHECK(p.wr[m] * ((p.rows[m] + p.wr[m] - 1) / p.wr[m]) >= p.rows[m], "%s: rows", tag);
      CHECK(p.ck[m] * p.nsl[m] == p.cols[m] && p.ck[m] % 32 == 0, "%s: slices", tag);
    }
    std::vector<int> item_seen(p.hkv * p.splits, 0);
    std::vector<int> item_cta(p.hkv * p.splits, -1);
    for (int b = 0; b < G; ++b) {
      int kvh, split;
      if (my_item(p, l, b, &kvh, &split)) {
        CHECK(kvh >= 0 && kvh < p.hkv && split >= 0 && split < p.splits, "%s: item", tag);
        ++item_seen[kvh * p.splits + split];
        item_cta[kvh * p.splits + split] = b;
      }
    }
    for (int i = 0; i < p.hkv * p.splits; ++i)
      CHECK(item_seen[i] == 1, "%s: layer %d item %d taken %d times", tag, l, i, item_seen[i]);
    for (int n : ns) {
      if (n < 1 || n > p.ctx) continue;
      long long att_tiles = 0;
      for (int kvh = 0; kvh < p.hkv; ++kvh) {
        int next = 0;
        for (int s = 0; s < p.splits; ++s) {
          int t0, t1;
          item_range(p, s, n, &t0, &t1);
          CHECK(t0 == next || t0 == t1, "%s: n %d kvh %d split %d starts %d, want %d", tag, n, kvh,
                s, t0, next);
          CHECK(t1 >= t0 && t1 <= n, "%s: range", tag);
          if (t1 > t0) next = t1;
          const int nst = item_stages(p, t0, t1);
          att_tiles += nst;
          for (int st = 0; st < nst; ++st) {
            const int ta = t0 + st * p.P;
            const int tb = ta + p.P < t1 ? ta + p.P : t1;
            CHECK(tb > ta && tb - ta <= p.P, "%s: stage size", tag);
            const long long off = stage_offset(p, kvh, t0, st);
            CHECK(off == ((long long)kvh * p.ctx + ta) * p.row_bytes, "%s: stage offset", tag);
            CHECK(off + (long long)(tb - ta) * p.row_bytes <= (long long)(kvh + 1) * p.ctx * p.row_bytes,
                  "%s: stage past its kv head", tag);
          }
        }
        CHECK(next == n, "%s: n %d kvh %d covered up to %d", tag, n, kvh, next);
      }
      long long per_cta = 0;
      for (int b = 0; b < G; ++b) per_cta += layer_tiles(p, l, b, n);
      CHECK(per_cta == mat_tiles + att_tiles, "%s: per-CTA tiles %lld != %lld", tag, per_cta,
            mat_tiles + att_tiles);
    }
  }
  // balance at the full context, layer 0
  int mn = 1 << 30, mx = 0;
  long long sum = 0;
  for (int b = 0; b < G; ++b) {
    const int t = layer_tiles(p, 0, b, p.ctx);
    mn = t < mn ? t : mn;
    mx = t > mx ? t : mx;
    sum += t;
  }
  std::printf("%s grid %d splits %d P %d tiles/cta min %d mean %.2f max %d\n", tag, G, p.splits,
              p.P, mn, (double)sum / G, mx);
  return true;
}

}  // namespace

int main() {
  const Shape shapes[] = {
      {"llama3.2-1b", 2048, 16, 32, 8, 8192},
      {"llama3.2-3b", 3072, 28, 24, 8, 8192},
      {"llama3.1-8b", 4096, 32, 32, 8, 14336},
      {"small-gqa3", 384, 2, 6, 2, 1024},
  };
  const int grids[] = {148, 132, 9};  // at least one CTA per kv head (the runtime's condition)
  const int ctxs[] = {4352, 300};
  int plans = 0;
  for (const Shape& sh : shapes) {
    const int hd = sh.n_emb / sh.heads;
    for (int world : {1, 2, 4, 8}) {
      if (sh.kv_heads % world || (sh.n_ff / world) % 32 || (sh.heads / world * hd) % 32) continue;
      const int hq = sh.heads / world, hkv = sh.kv_heads / world, ff = sh.n_ff / world;
      const int rows[N_MAT] = {(hq + 2 * hkv) * hd, sh.n_emb, 2 * ff, sh.n_emb};
      const int cols[N_MAT] = {sh.n_emb, hq * hd, sh.n_emb, ff};
      for (int es : {4, 2}) {
        if (es == 2 && hd < 64) continue;
        const int P = 32768 / (2 * hd * es) > 8 ? 32768 / (2 * hd * es) : 8;  // the workspace's att_P
        for (int grid : grids) {
          for (int ctx : ctxs) {
            Plan p = make_plan(grid, sh.n_layers, rows, cols, hkv, P, 2 * hd * es, ctx, 8, 32 * 1024);
            char tag[160];
            std::snprintf(tag, sizeof tag, "%s tp%d kv%s ctx %d", sh.name, world, es == 4 ? "f32" : "f16",
                          ctx);
            if (!check_plan(p, tag)) return 1;
            ++plans;
          }
        }
      }
    }
  }
  std::printf("ok %d plans\n", plans);
  return g_fail;
}
