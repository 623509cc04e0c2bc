"""Column split across ranks (busfill_b200/tp.py) on CPU: the shard arithmetic,
and the gather/assembly with world_size 2 and 3 over gloo, the local GEMM
replaced by the oracle. The CUDA path of the same functions is exercised by
tests/test_tp_gpu.py on machines with two or more GPUs."""
import os
import socket

import numpy as np
import pytest

from busfill_b200 import tp
from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("n", [1, 127, 128, 129, 640, 5120, 17408, 10000])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition(n, world):
    spans = [tp.shard_rows(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0                           # contiguous, in rank order
    for s0, s1 in spans:
        assert s0 % tp.TILE_ROWS == 0 or s0 == n  # whole tiles (an empty shard sits at the end)
        assert s1 - s0 >= 0
    sizes = [s1 - s0 for s0, s1 in spans]
    assert max(sizes) - min(sizes) <= tp.TILE_ROWS  # balanced to within a tile
    assert tp.max_shard_rows(n, world) == max(sizes)


def test_shard_rows_rejects_bad_args():
    with pytest.raises(ValueError):
        tp.shard_rows(128, 2, 2)
    with pytest.raises(ValueError):
        tp.shard_rows(128, 0, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fmt, n, k, m, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a = orc.gen_activations(m, k, seed=7)
        s0, s1 = tp.shard_rows(n, world, rank)
        at = torch.from_numpy(a)
        if fmt == "q4k":
            blocks = orc.gen_q4k(n, k, seed=5)
            local = lambda b, a_: torch.from_numpy(
                orc.gemm_ref(a_.numpy(), orc.dequant_q4k_f32(b.numpy(), k)).astype(np.float16))
            c = tp.gemm_q4k_tp(torch.from_numpy(blocks[s0:s1]), at, n, local_gemm=local)
            # per-slice products computed exactly as the ranks compute them (BLAS
            # rounding depends on the matrix shape), concatenated in rank order
            want = np.concatenate([local(torch.from_numpy(blocks[r0:r1]), at).numpy()
                                   for r0, r1 in (tp.shard_rows(n, world, r) for r in range(world))], axis=1)
        else:
            wq, ws = orc.gen_q4_0(n, k, seed=5)
            local = lambda w, s, a_: torch.from_numpy(
                orc.gemm_ref(a_.numpy(), orc.dequant_q4_0_planes_f32(w.numpy(), s.numpy())).astype(np.float16))
            c = tp.gemm_q4_0_tp(torch.from_numpy(wq[s0:s1]), torch.from_numpy(ws[s0:s1]), at, n, local_gemm=local)
            want = np.concatenate([local(torch.from_numpy(wq[r0:r1]), torch.from_numpy(ws[r0:r1]), at).numpy()
                                   for r0, r1 in (tp.shard_rows(n, world, r) for r in range(world))], axis=1)
        full = orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k) if fmt == "q4k" else orc.dequant_q4_0_planes_f32(wq, ws))
        _, rel, _ = orc.gemm_errors(c.numpy().astype(np.float32), full)
        same = bool(np.array_equal(c.numpy().view(np.uint16), want.view(np.uint16))) and rel < 1e-3
        q.put((rank, same, tuple(c.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,world,n", [("q4k", 2, 512), ("q4k", 2, 640), ("q4_0", 2, 384),
                                         ("q4k", 3, 640), ("q4_0", 3, 256)])
def test_gather_assembles_column_slices(fmt, world, n):
    import torch.multiprocessing as mp

    k, m = 512, 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fmt, n, k, m, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, shape in results:
        assert shape == (m, n)
        assert same, f"rank {rank}: assembled C differs from the unsplit product"
