"""Column split across GPUs through the C ABI and NCCL (busfill_b200/tp.py).
Each rank is a spawned process on its own GPU; the multi-rank tests need two
or more GPUs, the single-rank run of the gathered GEMMs one."""
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


def _worker_gather(rank, world, port, q, m=8):
    """Two chained column-split GEMMs whose all-gathers run in the GEMM
    epilogues (peer stores + flags, no NCCL on the data path), and a fused
    SwiGLU site reading the first one's gathered output too; first eagerly,
    then replayed from a CUDA graph with new activations each time
    (device-resident flag generations). Activations are scaled so that the
    unnormalised synthetic weights keep every stage inside fp16."""
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
    space = None
    try:
        k0, n1, n2, n3 = 2048, 1280, 768, 384
        w1 = orc.gen_q4k(n1, k0, seed=21)
        w2 = orc.gen_q4k(n2, n1, seed=22)
        wg = orc.gen_q4k(n3, n1, seed=23)
        wu = orc.gen_q4k(n3, n1, seed=24)

        def shard(w, n):
            s0, s1 = tp.shard_rows(n, world, rank)
            return torch.from_numpy(w[s0:s1]).to(dev)

        w1l, w2l, wgl, wul = shard(w1, n1), shard(w2, n2), shard(wg, n3), shard(wu, n3)
        space = tp.GatherSpace([(m, n1), (m, n2), (m, n3)])
        a = torch.empty((m, k0), dtype=torch.float16, device=dev)
        st = torch.cuda.Stream(device=dev)

        def chain():
            o1 = tp.gemm_q4k_gather(w1l, a, space, 0, stream=st)
            o2 = tp.gemm_q4k_gather(w2l, o1, space, 1, wait_site=0, stream=st)
            # a second consumer of site 0's gathered output, with its own wait count
            return o1, o2, tp.gemm_q4k_swiglu_gather(wgl, wul, o1, space, 2, wait_site=0, stream=st)

        def check(an, o1, o2, o3):
            # each stage against the oracle on the previous stage's gathered (fp16) output
            r1 = orc.gemm_ref(an, orc.dequant_q4k_f32(w1, k0))
            x1 = o1.cpu().numpy()
            r2 = orc.gemm_ref(x1, orc.dequant_q4k_f32(w2, n1))
            x2 = o2.cpu().numpy()
            r3 = orc.swiglu_ref(x1, orc.dequant_q4k_f32(wg, n1), orc.dequant_q4k_f32(wu, n1))
            errs = []
            for got, ref in ((o1, r1), (o2, r2), (o3, r3)):
                g = got.float().cpu().numpy().astype(np.float64)
                errs.append(float(np.linalg.norm(g - ref) / max(np.linalg.norm(ref), 1e-30)))
            return errs

        results = []
        an = (orc.gen_activations(m, k0, seed=30) / 4096).astype(np.float16)
        a.copy_(torch.from_numpy(an))
        with torch.cuda.stream(st):
            o1, o2, o3 = chain()
        st.synchronize()
        results.append(check(an, o1, o2, o3))
        dist.barrier()  # no rank writes the next outputs while another still reads these
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            chain()
        for rep in range(3):
            an = (orc.gen_activations(m, k0, seed=40 + rep) / 4096).astype(np.float16)
            a.copy_(torch.from_numpy(an))
            torch.cuda.synchronize(dev)
            with torch.cuda.stream(st):
                g.replay()
            st.synchronize()
            results.append(check(an, space.output(0), space.output(1), space.output(2)))
            dist.barrier()
        del g
        status = bf.stream_status(st)
        q.put((rank, status, results))
    except Exception as e:  # report instead of leaving the parent waiting on the queue
        q.put((rank, "error", repr(e)))
        raise
    finally:
        torch.cuda.synchronize(dev)
        dist.barrier()
        if space is not None:
            space.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m", [8, 40])  # 40 rows: two launches per call (the first waits, the last signals)
def test_gather_fused_into_epilogue(m):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_gather, args=(r, world, port, q, m)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, status, runs in results:
        assert status == 0, (rank, status, runs)
        for errs in runs:
            assert all(e <= 1e-3 for e in errs), (rank, runs)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("m", [8, 40])
def test_gather_fused_single_rank(m):
    """The gathered GEMMs in a process group of one: every peer store and
    flag is the rank's own, and each consuming GEMM waits only on a GEMM
    issued before it on the same stream (already resident when it starts),
    so the whole epilogue-gather path, its tile counters, its call counting
    and graph replays run on a single GPU."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_worker_gather, args=(0, 1, _free_port(), q, m))
    p.start()
    rank, status, runs = q.get(timeout=240)
    p.join(timeout=60)
    assert p.exitcode == 0
    assert status == 0, (rank, status, runs)
    for errs in runs:
        assert all(e <= 1e-3 for e in errs), runs
