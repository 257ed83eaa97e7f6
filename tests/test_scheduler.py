"""Tile scheduling (CPU only): the kernel's tile_to_bmn (compiled from
hopper-lab_b200/csrc/gemm_sm100.cuh as host code) against the reference's
group-M formula (src/08_persistent/gemm_fp8_persist.cu:56-66), and coverage of the
static persistent schedule (every tile exactly once)."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CASES = [(64, 32, 1), (64, 32, 8), (64, 32, 16), (7, 5, 3), (1, 64, 8), (33, 1, 8), (32, 32, 8),
         (2, 64, 8), (5, 9, 5), (100, 3, 7)]


def ref_tile_to_bmn(tile, num_bm, num_bn, G):
    """The reference's group-M mapping, stated directly."""
    tiles_per_group = G * num_bn
    g = tile // tiles_per_group
    first_bm = g * G
    gsize = min(num_bm - first_bm, G)
    t = tile - g * tiles_per_group
    return first_bm + t % gsize, t // gsize


@pytest.fixture(scope="module")
def kernel_mapping(tmp_path_factory):
    d = tmp_path_factory.mktemp("sched")
    src = d / "map.cu"
    src.write_text('''#include <cstdio>
#include "gemm_sm100.cuh"
int main(int argc, char** argv) {
  const unsigned cases[][3] = {%s};
  for (auto& c : cases) {
    for (unsigned t = 0; t < c[0] * c[1]; ++t) {
      unsigned bm, bn;
      b200::tile_to_bmn(t, c[0], c[1], c[2], bm, bn);
      std::printf("%%u %%u %%u %%u %%u %%u\\n", c[0], c[1], c[2], t, bm, bn);
    }
  }
  return 0;
}
''' % ", ".join("{%d,%d,%d}" % c for c in CASES))
    exe = d / "map"
    subprocess.run(["nvcc", "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{ROOT / 'hopper-lab_b200' / 'csrc'}",
                    f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    rows = [tuple(map(int, line.split())) for line in out.splitlines()]
    return rows


def test_kernel_mapping_equals_reference_formula(kernel_mapping):
    for nbm, nbn, G, t, bm, bn in kernel_mapping:
        assert (bm, bn) == ref_tile_to_bmn(t, nbm, nbn, G)


@pytest.mark.parametrize("nbm,nbn,G", CASES)
def test_group_m_is_a_bijection(nbm, nbn, G):
    seen = {ref_tile_to_bmn(t, nbm, nbn, G) for t in range(nbm * nbn)}
    assert seen == {(m, n) for m in range(nbm) for n in range(nbn)}


def test_group1_is_row_wave_order():
    assert [ref_tile_to_bmn(t, 3, 4, 1) for t in range(12)] == [(m, n) for m in range(3) for n in range(4)]


@pytest.mark.parametrize("tiles,ctas", [(2048, 148), (1024, 74), (5, 148), (148, 148), (149, 148)])
def test_static_persistent_schedule_covers_each_tile_once(tiles, ctas):
    """Cluster c takes tiles c, c + G, c + 2G, ... with G = number of clusters."""
    grid = min(tiles, ctas)
    taken = [t for c in range(grid) for t in range(c, tiles, grid)]
    assert sorted(taken) == list(range(tiles))


def test_group_m_window_limits_distinct_rows():
    """With G = 8 the first 148 tiles touch at most 8 block-rows (the L2 window)."""
    rows = {ref_tile_to_bmn(t, 64, 32, 8)[0] for t in range(148)}
    assert len(rows) <= 8
