"""Column split across GPUs through the C ABI and NCCL (busfill_b200/tp.py).
Needs two or more GPUs; each rank is a spawned process on its own GPU."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fmt, n, k, m, q):
    from datetime import timedelta

    import torch.distributed as dist

    import busfill_b200 as bf
    from busfill_b200 import tp
    from oracle import q4_oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        s0, s1 = tp.shard_rows(n, world, rank)
        a = orc.gen_activations(m, k, seed=11)
        at = torch.from_numpy(a).to(dev)
        if fmt == "q4k":
            blocks = orc.gen_q4k(n, k, seed=12)
            c = tp.gemm_q4k_tp(torch.from_numpy(blocks[s0:s1]).to(dev), at, n)
            ref = orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k))
        else:
            wq, ws = orc.gen_q4_0(n, k, seed=12)
            c = tp.gemm_q4_0_tp(torch.from_numpy(wq[s0:s1]).to(dev), torch.from_numpy(ws[s0:s1]).to(dev), at, n)
            ref = orc.gemm_ref(a, orc.dequant_q4_0_planes_f32(wq, ws))
        torch.cuda.synchronize(dev)
        status = bf.stream_status()
        max_abs, rel, finite = orc.gemm_errors(c.float().cpu().numpy(), ref)
        q.put((rank, status, bool(finite), float(max_abs), float(rel)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fmt,n", [("q4k", 5120), ("q4k", 1408), ("q4_0", 2048)])
def test_column_split_matches_oracle(fmt, n):
    import torch.multiprocessing as mp

    from oracle import q4_oracle as orc

    world = min(torch.cuda.device_count(), 4)
    k, m = 2048, 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fmt, n, k, m, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, status, finite, max_abs, rel in results:
        assert status == 0 and finite, rank
        assert max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2, (rank, max_abs, rel)
