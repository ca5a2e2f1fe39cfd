"""Schedule of the persistent layer kernel, checked on the CPU (no GPU).

tests/persist_plan_check.cpp builds the plans the library builds
(l3g_persist_plan.h make_plan) for the 1B, 3B and 8B shapes and a small GQA
shape, at 1 to 8 ranks, f32 and f16 KV caches and several grid sizes, and
checks that every weight tile and every attention item is taken by exactly
one CTA, that the splits of each kv head cover the live positions in order
in stages inside the head's cache rows, and that the per-CTA tile counts the
producer and the consumers walk add up.  The tile geometry it uses is the
library's own (tile_geometry, also behind make_tiles), pinned here against
the 8B shapes' known layout.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "llama3.go_b200", "csrc")


@pytest.fixture(scope="module")
def check_output(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    exe = str(tmp_path_factory.mktemp("persist") / "persist_plan_check")
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-I", CSRC,
                    os.path.join(HERE, "persist_plan_check.cpp"), "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout[-2000:]
    return r.stdout


def test_schedule_covers_every_tile_and_item(check_output):
    lines = check_output.strip().splitlines()
    assert lines[-1].startswith("ok ")
    assert int(lines[-1].split()[1]) >= 100


def test_8b_layer_is_balanced(check_output):
    """Single GPU, 8B shape, 148 SMs, all 4352 positions live: the busiest
    CTA's share of a layer (weight tiles + attention stages, ~34 KB each) is
    within 8 tiles of the mean (45 weight tiles + 7.35 stages per CTA)."""
    line = next(l for l in check_output.splitlines()
                if l.startswith("llama3.1-8b tp1 kvf32 ctx 4352 grid 148 "))
    f = line.split()
    mean, mx = float(f[f.index("mean") + 1]), int(f[f.index("max") + 1])
    assert abs(mean - (6656 + 8 * 4352 / 32) / 148) < 0.01, line
    assert mx - mean < 8, line


def test_tile_geometry_matches_the_8b_layout():
    """The 8B up/gate shard at four rows per warp: 32-row groups, 1024-column
    slices, 34,816-byte tiles, 896 groups (the layout the decode step's
    measurements were taken on)."""
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    src = r'''
#include <cstdio>
#include "l3g_persist_plan.h"
int main() {
  const l3g::TileGeom g = l3g::tile_geometry(28672, 4096, 4, 8, 32 * 1024);
  const l3g::TileGeom d = l3g::tile_geometry(4096, 14336, 4, 8, 32 * 1024);
  std::printf("%d %d %d %d %d %d %d %d %d %d\n", g.wr, g.ck, g.nslices, g.tile_bytes, g.n_groups,
              d.wr, d.ck, d.nslices, d.tile_bytes, d.n_groups);
}
'''
    import tempfile
    with tempfile.TemporaryDirectory() as td:
        cpp = os.path.join(td, "g.cpp")
        with open(cpp, "w") as f:
            f.write(src)
        exe = os.path.join(td, "g")
        subprocess.run([gxx, "-std=c++17", "-I", CSRC, cpp, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    assert [int(v) for v in out] == [32, 1024, 4, 34816, 896, 32, 1024, 14, 34816, 128]


def test_tile_geometry_matches_the_python_statement(tmp_path):
    """The shared tile_geometry (used by make_tiles for every decode matrix)
    equals the independent statement of the layout in
    test_batched_index_math.make_tiles for 480 shapes and every rows-per-warp
    choice."""
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    from test_batched_index_math import make_tiles
    rows_l = [1, 7, 32, 100, 513, 1024, 2050, 4096, 6144, 14336, 28672, 128256]
    cols_l = [32, 96, 288, 512, 1792, 2048, 3072, 4096, 8192, 14336]
    src = tmp_path / "g.cpp"
    src.write_text("#include <cstdio>\n#include \"l3g_persist_plan.h\"\nint main() {\n"
                   + "".join(f"  {{ l3g::TileGeom g = l3g::tile_geometry({r}, {c}, {k}, 8, 32768);"
                             f" std::printf(\"%d %d %d %d %d\\n\", g.wr, g.ck, g.nslices, g.tile_bytes,"
                             f" g.n_groups); }}\n"
                             for r in rows_l for c in cols_l for k in (1, 2, 4, 8))
                   + "}\n")
    exe = str(tmp_path / "g")
    subprocess.run([gxx, "-std=c++17", "-I", CSRC, str(src), "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.splitlines()
    i = 0
    for r in rows_l:
        for c in cols_l:
            for k in (1, 2, 4, 8):
                t = make_tiles(r, c, k)
                want = [t["wr"], t["ck"], t["nslices"], t["tile_bytes"], t["n_groups"]]
                assert [int(v) for v in out[i].split()] == want, (r, c, k)
                i += 1

