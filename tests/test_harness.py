"""The drop-in host harness include/common/*.h (CPU only): same API as the
reference's harness (include/common/{tensor,checker,bench}.h), checked by compiling
a small program against it and comparing with the oracle."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]

PROG = r'''
#include <cstdio>
#include <vector>
#include "common/bench.h"
#include "common/checker.h"
#include "common/tensor.h"
int main(int argc, char** argv) {
  const char* csv = argv[1];
  auto u = hopper::make_random_vector(1000, 601, -1.f, 1.f);
  auto n = hopper::make_normal_vector(1000, 605, 0.f, 0.1f);
  for (float x : u) std::printf("%a\n", x);
  for (float x : n) std::printf("%a\n", x);
  std::vector<float> g = {1.f, 2.f, 3.001f, 4.1f};
  std::vector<float> e = {1.f, 2.0005f, 3.f, 4.f};
  auto r = hopper::check_close(g, e, 1e-3, 1e-3);
  std::printf("%d %zu %a %a\n", int(r.pass), r.mismatches, r.max_abs_err, r.max_rel_err);
  hopper::print_report(r, "harness");
  std::printf("%a\n", hopper::norm_rel_error(g, e));
  std::printf("%a %a\n", hopper::tflops(2e12, 1.0), hopper::bandwidth_gbps(1e9, 2.0));
  { hopper::CsvWriter w(csv, {"a", "b"}); w.row({"1", "2"}); }
  { hopper::CsvWriter w(csv, {"a", "b"}); w.row({"3", "4"}); }
  return 0;
}
'''


@pytest.fixture(scope="module")
def harness_out(tmp_path_factory):
    d = tmp_path_factory.mktemp("harness")
    (d / "h.cpp").write_text(PROG)
    exe = d / "h"
    subprocess.run(["g++", "-std=c++17", "-O2", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
                    str(d / "h.cpp"), "-o", str(exe), "-L/usr/local/cuda/lib64", "-lcudart"],
                   check=True)
    csv = d / "out.csv"
    out = subprocess.run([str(exe), str(csv)], capture_output=True, text=True, check=True).stdout
    return out.splitlines(), csv.read_text()


def test_make_random_vector_matches_oracle(harness_out, oracle):
    lines, _ = harness_out
    u = np.array([float.fromhex(x) for x in lines[:1000]], np.float32)
    assert np.array_equal(u, oracle.uniform(601, 1000))


def test_make_normal_vector_matches_oracle(harness_out, oracle):
    lines, _ = harness_out
    n = np.array([float.fromhex(x) for x in lines[1000:2000]], np.float32)
    assert np.array_equal(n, oracle.normal(605, 1000, 0.0, 0.1))


def test_check_close_and_report(harness_out, oracle):
    lines, _ = harness_out
    p, mm, ma, mr = lines[2000].split()
    r = oracle.check_close(np.array([1, 2, 3.001, 4.1], np.float32),
                           np.array([1, 2.0005, 3, 4], np.float32), 1e-3, 1e-3)
    assert int(p) == 0 and int(mm) == r.mismatches == 1
    assert float.fromhex(ma) == r.max_abs_err and float.fromhex(mr) == r.max_rel_err
    assert lines[2001].startswith("[CHECK ] harness") and "FAIL" in lines[2001]


def test_bench_helpers(harness_out):
    lines, _ = harness_out
    tf, bw = (float.fromhex(x) for x in lines[2003].split())
    assert tf == pytest.approx(2000.0) and bw == pytest.approx(500.0)


def test_csv_header_written_once(harness_out):
    _, csv = harness_out
    assert csv == "a,b\n1,2\n3,4\n"
