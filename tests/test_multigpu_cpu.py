"""Multi-GPU host logic on CPU: column sharding, the all-gather + re-layout of C
slabs with world_size-2 gloo process groups, and failure detection when a rank
dies before a collective (the failure is made on the host; no GPU involved).

Inside the worker processes the oracle stands in for each rank's GPU GEMM."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests"))


def _pkg():
    from conftest import _load_pkg

    return _load_pkg()


def _mg():
    import importlib.util

    spec = importlib.util.spec_from_file_location("b200_multigpu", ROOT / "hopper-lab_b200" / "multigpu.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.mark.parametrize("n,world", [(65536, 8), (8192, 3), (100, 4), (16, 4), (0, 2), (65536, 1)])
def test_shards_tile_the_columns(n, world):
    mg = _mg()
    ranges = [mg.shard_columns(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 <= a1
    for a0, _ in ranges:
        assert a0 % 16 == 0
    sizes = mg.shard_sizes(n, world)
    assert sum(sizes) == n and all(s <= -(-n // world) + 16 for s in sizes)


def test_config5_shape_splits_evenly():
    mg = _mg()
    for g in (1, 2, 4, 8):
        assert set(mg.shard_sizes(65536, g)) == {65536 // g}


def test_bad_rank_rejected():
    mg = _mg()
    with pytest.raises(ValueError):
        mg.shard_columns(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta

        sys.path.insert(0, str(ROOT))
        import oracle as O

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        mg = _mg()
        M, N, K = 48, 64, 40
        A = O.f16_bits_to_f32(O.f32_to_f16_bits(O.uniform(601, M * K))).reshape(M, K)
        B = O.f16_bits_to_f32(O.f32_to_f16_bits(O.uniform(602, N * K))).reshape(N, K)
        n0, n1 = mg.shard_columns(N, world, rank)
        if mode == "die" and rank == 1:
            os._exit(3)  # leaves between steps, before any collective
        c_slab = torch.from_numpy(O.gemm_tn(A, B[n0:n1]))
        full = mg.all_gather_columns(c_slab, world)
        ref = O.gemm_tn(A, B)
        q.put((rank, "ok", bool(np.array_equal(full.numpy(), ref))))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 — reported to the parent
        q.put((rank, "error", type(e).__name__ + ": " + str(e)[:200]))


def _spawn(world, mode):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    for p in ps:
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return out, [p.exitcode for p in ps]


def test_sharded_gemm_all_gather_equals_full_gemm():
    out, codes = _spawn(2, "ok")
    assert codes == [0, 0]
    assert sorted(out) == [(0, "ok", True), (1, "ok", True)]


def test_dead_rank_surfaces_as_error_not_hang():
    out, codes = _spawn(2, "die")
    assert codes[1] == 3
    assert len(out) == 1 and out[0][0] == 0 and out[0][1] == "error"
