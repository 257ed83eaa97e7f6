"""The per-experiment executables (hopper-lab_b200/experiments/*.cu): each mirrors
one of the reference's experiment mains, prints [CHECK ] / [BENCH ] / [GEMM  ]
lines and appends results/*.csv. CPU: they are built and answer --help. GPU: each
runs its --quick set and every [CHECK ] line passes."""
import importlib.util
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "hopper-lab_b200" / "bin"


def _experiments():
    spec = importlib.util.spec_from_file_location("b200_build", ROOT / "hopper-lab_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return sorted(mod.EXPERIMENTS)


EXPERIMENTS = _experiments()


def test_every_experiment_source_is_built():
    srcs = sorted(p.stem for p in (ROOT / "hopper-lab_b200" / "experiments").glob("*.cu"))
    assert srcs == EXPERIMENTS


@pytest.mark.parametrize("name", EXPERIMENTS)
def test_experiment_answers_help_without_gpu(name):
    exe = BIN / name
    if not exe.exists():
        pytest.skip("executables not built (python hopper-lab_b200/build.py)")
    r = subprocess.run([str(exe), "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "usage" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("name", EXPERIMENTS)
def test_experiment_quick_run_passes(name, tmp_path):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = BIN / name
    args = [str(exe), "--quick"]
    if name == "gemm_multi_gpu":
        args += ["--gpus", "1"]
    r = subprocess.run(args, capture_output=True, text=True, timeout=900, cwd=tmp_path,
                       env={**os.environ})
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    checks = [line for line in out.splitlines() if line.startswith("[CHECK ]")]
    assert all("FAIL" not in line for line in checks), out[-3000:]
    if name not in ("peak_tcgen05",):
        assert checks, out[-3000:]
    assert list((tmp_path / "results").glob("*.csv")), "no CSV written"
