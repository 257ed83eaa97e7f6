"""bench.py's reference arm (--impl reference) on CPU: the reference's host GEMM
loop (oracle port) on row bands of the 8192^3 fp16 problem, printing the one JSON
line the driver reads. Also the roofline traffic lookup in profiles/."""
import importlib.util
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3", "--cpu-budget", "0.3"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOPS" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
    assert d["config"]["workload"] == "gemm_tn_f16_8192x8192x8192_per_gpu"


def test_reference_arm_non_zero_rank_exits_quietly():
    env = {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1", "PATH": "/usr/bin:/bin"}
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference"],
                       capture_output=True, text=True, timeout=120, cwd=ROOT, env=env)
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_roofline_traffic_comes_from_profiles():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.profile_traffic("f16_8192") > 402653184  # above the compulsory bytes
    assert m.profile_traffic("e4m3_8192") > 268435456
    assert m.profile_traffic("nonexistent") is None


def test_measurement_modes_parse_and_size_helper():
    """The profile / power / sweep helpers parse their arguments (positional arguments may
    be mixed with options) and sizes like 8192, 8192x1024 and 256x16384x8192."""
    spec = importlib.util.spec_from_file_location("bench_mod2", ROOT / "bench.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m._parse_size("8192") == (8192, 8192, 8192)
    assert m._parse_size("8192x1024") == (8192, 8192, 1024)
    assert m._parse_size("256x16384x8192") == (256, 16384, 8192)
    for args in (["--mode", "power", "e4m3", "--shape", "256x16384x8192", "cublas", "--help"],
                 ["--mode", "sweep", "--dtypes", "f16", "--help"],
                 ["--mode", "profile", "f16", "ours", "--help"]):
        r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                           text=True, timeout=120, cwd=ROOT)
        assert r.returncode == 0 and "--mode" in r.stdout, (args, r.stderr[-500:])
