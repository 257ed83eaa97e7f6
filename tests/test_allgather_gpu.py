"""Fused GEMM + all-gather of C (b200_gemm_allgather) on 2+ GPUs of one node.

Every rank computes its N-column slab of C = A.B^T and the GEMM epilogue stores each
finished tile into a symmetric M x N buffer on every rank: through the NVSwitch with
multimem stores when the node supports NVLink multicast, and with peer stores
otherwise (both modes are run), on the static and the cluster-launch-control pair
schedules. Checked on every rank:
- the gathered buffer holds, bit for bit, each rank's locally written slab;
- the gathered buffers of all ranks are identical;
and on rank 0 the gathered M x N result against the CPU oracle (seeded row bands
against all N columns plus one full column slab). Needs at least two GPUs; skipped
otherwise.
"""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, shapes, queue):
    import importlib.util
    import sys
    from datetime import timedelta
    from pathlib import Path

    import torch.distributed as dist

    root = Path(__file__).resolve().parents[1]
    for d in (str(root), str(root / "tests")):
        if d not in sys.path:
            sys.path.insert(0, d)
    import oracle as O
    from gemm_check import TOL_16, check_big, make_inputs, to_device

    spec = importlib.util.spec_from_file_location("hopper_lab_b200", root / "hopper-lab_b200" / "__init__.py")
    b200 = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b200)
    spec = importlib.util.spec_from_file_location("b200_multigpu", root / "hopper-lab_b200" / "multigpu.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    out = []
    try:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=dev)
        for (m, n, k, dt) in shapes:
            # the same seeded inputs on every rank (the oracle's generator)
            inp = make_inputs(O, m, n, k, dt, 1234, 1235)
            a, b, _, _ = to_device(inp, torch)
            tdt = a.dtype
            gc = mg.GatheredC(m, n, tdt, dev)
            n0, n1 = gc.slab()
            modes = [False, True] if gc.multicast else [True]
            for variant in ("auto", "2cta", "2cta_clc"):
                for force_peers in modes:
                    gc.buf.fill_(float("nan"))
                    torch.cuda.synchronize()
                    dist.barrier(device_ids=[rank])
                    c_slab = torch.empty((m, n1 - n0), dtype=tdt, device=dev)
                    gc.gemm(b200, a, b[n0:n1], c_slab, force_peers=force_peers, variant=variant)
                    gc.sync()
                    torch.cuda.synchronize()
                    rc, bits = b200.status()
                    full = gc.buf.clone()
                    own_ok = torch.equal(full[:, n0:n1], c_slab)
                    # every rank's gathered buffer is identical: compare against rank 0's
                    r0 = full.clone()
                    dist.broadcast(r0, src=0)
                    same = torch.equal(r0, full)
                    fails = None
                    if rank == 0:
                        fails = check_big(O, inp, full.float().cpu().numpy(), TOL_16, seed=m + n,
                                          rows=64, band=16, slab=256)
                    out.append({"shape": (m, n, k, dt), "variant": variant,
                                "mode": "peers" if force_peers else "multicast",
                                "status": rc, "bits": bits, "own": own_ok, "same": same,
                                "oracle_fails": fails,
                                "finite": bool(torch.isfinite(full.float()).all())})
                    dist.barrier(device_ids=[rank])
            del gc
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        queue.put((rank, out, None))
    except Exception as e:  # report to the parent instead of hanging it
        queue.put((rank, out, repr(e)))


def test_gemm_allgather_on_every_gpu(b200):
    n_gpu = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n_gpu < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n_gpu, 4)
    import torch.multiprocessing as mp

    shapes = [(1024, 2048, 512, "f16"), (520, 1056, 264, "bf16"), (4096, 8192, 2048, "f16")]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, out, err = queue.get(timeout=600)
        results[rank] = (out, err)
    for p in procs:
        p.join(timeout=120)
    for rank, (out, err) in sorted(results.items()):
        assert err is None, (rank, err)
        assert out, rank
        print(f"rank {rank}: modes run {sorted({r['mode'] for r in out})}")
        for r in out:
            assert r["status"] == 0, (rank, r)
            assert r["own"] and r["same"] and r["finite"], (rank, r)
            assert not r["oracle_fails"], (rank, r)


@pytest.mark.parametrize("variant,tile_n", [("auto", 0), ("2cta", 0), ("persistent", 0), ("1cta", 0),
                                            ("2cta_clc", 0), ("clc", 0), ("2cta", 128), ("2cta_clc", 512)])
def test_gather_epilogue_on_one_gpu_peer_mode(b200, variant, tile_n):
    """The gather stores of the epilogue on a single GPU (peer mode with one base: this
    GPU's own buffer): the gathered columns equal C bit for bit, the rest of each row
    is untouched."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda")
    g.manual_seed(81)
    m, n, k = 1000, 1040, 520
    a = (torch.rand((m, k), generator=g, device="cuda") * 2 - 1).half()
    b = (torch.rand((n, k), generator=g, device="cuda") * 2 - 1).half()
    c = torch.empty((m, n), dtype=torch.float16, device="cuda")
    ldg, col = 3 * 1040 + 24, 1040 + 8
    gathered = torch.full((m, ldg), float("nan"), dtype=torch.float16, device="cuda")
    bases = torch.tensor([gathered.data_ptr()], dtype=torch.int64, device="cuda")
    b200.gemm_allgather(a, b, c, bases.data_ptr(), b200.GATHER_PEERS, 1, ldg, col, variant=variant,
                        tile_n=tile_n)
    torch.cuda.synchronize()
    rc, bits = b200.status()
    assert rc == 0, hex(bits)
    assert torch.equal(gathered[:, col:col + n], c)
    assert torch.isnan(gathered[:, :col].float()).all() and torch.isnan(gathered[:, col + n:].float()).all()


def test_gather_refuses_streamk(b200):
    """The gather entry point takes no workspace, so the stream-K schedule (the only one
    that needs one) is refused; AUTO never resolves to it there."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    a = torch.zeros((256, 256), dtype=torch.float16, device="cuda")
    c = torch.empty((256, 256), dtype=torch.float16, device="cuda")
    dst = torch.empty((256, 512), dtype=torch.float16, device="cuda")
    with pytest.raises(b200.B200Error) as e:
        b200.gemm_allgather(a, a, c, dst.data_ptr(), b200.GATHER_MULTICAST, 0, 512, 0, variant="2cta_streamk")
    assert e.value.code == b200.ERR_UNSUPPORTED
