#!/usr/bin/env python
"""Benchmark of the batched dequant-fused Q4 GEMM (BASELINE metric: "Q4_K GEMM
tokens/s & HBM GB/s (% of ~8 TB/s) at M=1/8/32, K=N=5120").

Headline workload (N=1): Q4_K, M=32, K=N=5120. A *step* is one pass over R
distinct weight matrices (R rotating copies, together larger than 2x the L2
cache, so every GEMM streams its weights from HBM): R GEMM launches on the
same fp16 activations. ``value`` = tokens/s = M * R * steps / elapsed, i.e.
M / (average GEMM time) -- the reference's own definition (t/s = B / step
time, kernels/busfill_v1a.cu:172). Inputs are synthetic (seeded torch RNG, the
BASELINE config distributions), generated on the device.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl busfill|reference]

N > 1 (launched by torchrun): every weight matrix is split by output columns
across the ranks (rank r owns rows [r*N/g, (r+1)*N/g)); each GEMM is followed
by an NCCL all-gather of the [M, N/g] output slices and the re-interleave to
[M, N] (strong scaling: total work fixed). Timing is the max over ranks.

--impl reference: the CPU dequantize-then-fp32-matmul path (the reference's
own correctness path, kernels/q4k_batched.py:75,100, restated by the oracle)
on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["busfill", "reference"], default="busfill")
    ap.add_argument("--fmt", choices=["q4k", "q4_0"], default="q4k")
    ap.add_argument("--m", type=int, default=32)
    ap.add_argument("--n", type=int, default=5120)
    ap.add_argument("--k", type=int, default=5120)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-extras", action="store_true", help="skip sweep / cuBLAS / e2e / CPU / layer-set legs")
    ap.add_argument("--layers", type=int, default=64, help="layers in the BASELINE config-3 layer-set sweep")
    ap.add_argument("--layerset-only", action="store_true",
                    help="after the headline, run the layer-set leg alone (profiling the layer-sweep kernel)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def metric_name(fmt, K, N):
    return (f"{'Q4_K' if fmt == 'q4k' else 'Q4_0'} GEMM tokens/s (M / avg GEMM time) at "
            + (f"K=N={K}" if K == N else f"K={K}, N={N}"))


def alg_bytes(m, n, k):
    return n * k * 18 // 32 + 2 * m * k + 2 * m * n


def profiled_traffic(workload, world=1):
    """dram bytes per launch from a committed ncu summary of this exact
    per-rank workload (profiles/<workload>.md for one GPU,
    profiles/<workload>_tp<world>.md for a column split), else None."""
    name = workload if world == 1 else f"{workload}_tp{world}"
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().split()[0])
    except Exception:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                bits = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, name in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons - {"gpu_idle"})}


# ---------------------------------------------------------------------------
# synthetic inputs on the device (BASELINE config distributions)
# ---------------------------------------------------------------------------
def make_q4k_weights(torch, n, k, gen, dev):
    s = k // 256
    blocks = torch.randint(0, 256, (n, s, 144), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.rand((n, s), device=dev, generator=gen) * 0.009 + 0.001).half()
    dmin = (torch.rand((n, s), device=dev, generator=gen) * 0.005).half()
    blocks[:, :, 0:2] = d.view(torch.uint8).view(n, s, 2)
    blocks[:, :, 2:4] = dmin.view(torch.uint8).view(n, s, 2)
    return blocks.view(n, s * 144).contiguous()


def make_q5k_weights(torch, n, k, gen, dev):
    """block_q5_K rows [N, K/256*176] with config-2-like d / dmin; other bytes random."""
    s = k // 256
    blocks = torch.randint(0, 256, (n, s, 176), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.rand((n, s), device=dev, generator=gen) * 0.009 + 0.001).half()
    dmin = (torch.rand((n, s), device=dev, generator=gen) * 0.005).half()
    blocks[:, :, 0:2] = d.view(torch.uint8).view(n, s, 2)
    blocks[:, :, 2:4] = dmin.view(torch.uint8).view(n, s, 2)
    return blocks.view(n, s * 176).contiguous()


def make_q6k_weights(torch, bf, n, k, gen, dev):
    """Q6_K in the GEMM's layout (busfill_repack_q6k of random block_q6_K rows):
    body [N, K/256*208] random bytes, d [K/256, N] ~ U(0.0001, 0.0005)."""
    s = k // 256
    blocks = torch.randint(0, 256, (n, s, 210), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.rand((n, s), device=dev, generator=gen) * 0.0004 + 0.0001).half()
    blocks[:, :, 208:210] = d.view(torch.uint8).view(n, s, 2)
    return bf.repack_q6k(blocks.view(n, s * 210).contiguous(), k)


def make_q4_0_ggml_weights(torch, n, k, gen, dev):
    """llama.cpp block_q4_0 rows [N, K/32*18] with config-0 scales (U(0.001, 0.02))."""
    nb = k // 32
    blocks = torch.randint(0, 256, (n, nb, 18), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.rand((n, nb), device=dev, generator=gen) * 0.019 + 0.001).half()
    blocks[:, :, 0:2] = d.view(torch.uint8).view(n, nb, 2)
    return blocks.view(n, nb * 18).contiguous()


def make_q4_0_weights(torch, n, k, gen, dev):
    wq = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=gen)
    ws = (torch.rand((n, k // 32), device=dev, generator=gen) * 0.019 + 0.001).half()
    return wq, ws


# ---------------------------------------------------------------------------
# parity of the timed path (device reference, outside the timed region)
# ---------------------------------------------------------------------------
GATE_MAX_ABS = 0.6      # the reference's gate, kernels/q4k_batched.py:102
GATE_REL_L2 = 1e-3


def _errors(torch, c, ref):
    d = (c.double() - ref.double())
    finite = bool(torch.isfinite(c).all())
    return (float(d.abs().max()) if finite else float("inf"),
            float(d.norm() / ref.double().norm()), finite)


def parity_check(torch, bf, tp, dev, world, rank, args, space=None):
    """One call of the timed path on seeded inputs, checked on every rank
    against fp32 matmuls (torch, on the device) of the weights dequantized by
    busfill_dequant_q4k / _q4_0 (bit-exact to the CPU dequant in the test
    suite): the plain GEMM on one GPU; over several GPUs the gathered GEMM
    of one call site and a second site that consumes it (its wait on the
    first site's tile counters included), every rank's full gathered output
    against the all-gathered reference columns. Gates: max abs <= 0.6,
    rel-L2 <= 1e-3; the worst rank is reported."""
    import torch.distributed as dist
    torch.backends.cuda.matmul.allow_tf32 = False     # the reference is a true fp32 product
    M, N, K = args.m, args.n, args.k
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 7 + rank)
    r0, r1 = tp.shard_rows(N, world, rank)
    a = torch.randn((M, K), device=dev, generator=gen).half()
    if world > 1:
        dist.broadcast(a, 0)
    errs = []
    if args.fmt == "q4k":
        w1 = make_q4k_weights(torch, r1 - r0, K, gen, dev)
        ref1 = a.float() @ bf.dequant_q4k(w1, K).float().t()
    else:
        wq, ws = make_q4_0_weights(torch, r1 - r0, K, gen, dev)
        ref1 = a.float() @ bf.dequant_q4_0(wq, ws).float().t()
    if world == 1:
        c = bf.gemm_q4k(w1, a) if args.fmt == "q4k" else bf.gemm_q4_0(wq, ws, a)
        errs.append(_errors(torch, c.float(), ref1))
    elif space is None:
        c = tp.gemm_q4_0_tp(wq, ws, a, N)
        errs.append(_errors(torch, c.float(), tp.gather_columns(ref1.contiguous(), N)))
    else:
        # site 0: the timed call's shape on the config-scale activations;
        # site 1 on the activations scaled by 2^-12 (exact), whose output
        # site 2 (K' = N) consumes after its device-side wait on site 1's
        # counters (the scaling keeps the chained product near the
        # magnitudes the absolute gate is for)
        w2 = make_q4k_weights(torch, r1 - r0, N, gen, dev)
        a_small = (a.float() / 4096).half()
        st = torch.cuda.current_stream()
        c0 = tp.gemm_q4k_gather(w1, a, space, 0, stream=st)
        c1 = tp.gemm_q4k_gather(w1, a_small, space, 1, stream=st)
        c2 = tp.gemm_q4k_gather(w2, c1, space, 2, wait_site=1, stream=st)
        space.wait(0, stream=st)
        space.wait(2, stream=st)
        assert bf.stream_status(st) == 0
        ref0_full = tp.gather_columns(ref1.contiguous(), N)
        ref1s = a_small.float() @ bf.dequant_q4k(w1, K).float().t()
        ref1_full = tp.gather_columns(ref1s.contiguous(), N)
        ref2 = c1.float() @ bf.dequant_q4k(w2, N).float().t()
        ref2_full = tp.gather_columns(ref2.contiguous(), N)
        errs.append(_errors(torch, c0.float(), ref0_full))
        errs.append(_errors(torch, c1.float(), ref1_full))
        errs.append(_errors(torch, c2.float(), ref2_full))
        dist.barrier()
    torch.cuda.synchronize(dev)
    max_abs = max(e[0] for e in errs)
    rel = max(e[1] for e in errs)
    finite = all(e[2] for e in errs)
    if world > 1:
        t = torch.tensor([max_abs, rel, 0.0 if finite else 1.0], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        max_abs, rel, finite = float(t[0]), float(t[1]), t[2].item() == 0.0
    ok = finite and max_abs <= GATE_MAX_ABS and rel <= GATE_REL_L2
    what = ("plain GEMM" if world == 1 else
            "gathered GEMMs at 3 call sites, one consuming another's output" if space is not None else
            "GEMM + NCCL all-gather")
    return {"ok": ok, "max_abs": round(max_abs, 6), "rel_l2": float(f"{rel:.4g}"), "finite": finite,
            "checked": f"{what}, M={M}, N={N}, K={K}, worst rank of {world}",
            "reference": "fp32 torch matmul on the device of busfill_dequant_* weights (bit-exact dequant)",
            "gates": {"max_abs": GATE_MAX_ABS, "rel_l2": GATE_REL_L2}}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_busfill(args):
    import torch
    import torch.distributed as dist

    import busfill_b200 as bf
    from busfill_b200 import tp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    bf.load_library()
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    hbm_peak, tc_peak, peak_src = measured_peaks()

    M, N, K = args.m, args.n, args.k
    row0, row1 = tp.shard_rows(N, world, rank)    # this rank's weight rows (whole 128-row tiles)
    n_loc = row1 - row0
    if n_loc == 0:
        raise SystemExit(f"N={N} leaves rank {rank} of {world} without rows")
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + rank)
    wbytes = n_loc * K * 18 // 32
    R = max(2, math.ceil(2.2 * l2 / wbytes))
    if args.fmt == "q4k":
        base = make_q4k_weights(torch, n_loc, K, gen, dev)
        weights = [base] + [base.clone() for _ in range(R - 1)]
    else:
        wq, ws = make_q4_0_weights(torch, n_loc, K, gen, dev)
        weights = [(wq, ws)] + [(wq.clone(), ws.clone()) for _ in range(R - 1)]
    a = torch.randn((M, K), device=dev, generator=gen).half()
    a_full = a
    c_loc = torch.empty((M, n_loc), dtype=torch.float16, device=dev)
    c_full = torch.empty((M, N), dtype=torch.float16, device=dev) if world > 1 else None
    # Q4_K over several GPUs: the all-gather runs in the GEMM epilogue (peer
    # stores into every rank's output, one call site per weight copy);
    # Q4_0: NCCL all-gather after the GEMM
    space = tp.GatherSpace([(M, N)] * R) if (world > 1 and args.fmt == "q4k") else None
    pspace = tp.GatherSpace([(M, N)] * 3) if (world > 1 and args.fmt == "q4k") else None
    parity = parity_check(torch, bf, tp, dev, world, rank, args, pspace)
    if pspace is not None:
        torch.cuda.synchronize(dev)
        dist.barrier()
        pspace.close()
    if not parity["ok"]:
        if rank == 0:
            print(json.dumps({"error": "parity check failed", "parity": parity}))
        if world > 1:
            dist.destroy_process_group()
        raise SystemExit(3)

    def gemm(w, stream, i=0):
        if world == 1:
            if args.fmt == "q4k":
                bf.gemm_q4k(w, a, out=c_loc, stream=stream)
            else:
                bf.gemm_q4_0(w[0], w[1], a, out=c_loc, stream=stream)
        elif space is not None:
            tp.gemm_q4k_gather(w, a_full, space, i, stream=stream)
        else:
            tp.gemm_q4_0_tp(w[0], w[1], a, N, out=c_full, local_out=c_loc)

    def one_step(stream):
        for i, w in enumerate(weights):
            gemm(w, stream, i)

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        gemm(weights[0], stream)                  # one call first: fail fast on a device-side error
    st0, bits0 = bf.stream_status_bits(stream)
    if st0 != 0:
        raise SystemExit(f"device-side error on the first call: status {st0}, error bits {bits0:#x}")
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):      # W untimed warm-up steps (also sizes the workspace)
            one_step(stream)
    stream.synchronize()
    if bf.stream_status(stream) != 0:
        raise SystemExit("device-side error during warm-up")

    def capture(nsteps, fn=one_step):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(nsteps):
                fn(stream)
        return g

    def time_graph(g, replays=1, sampler=None):
        with torch.cuda.stream(stream):            # CUDAGraph.replay() launches on the current stream
            g.replay()                             # upload / first-replay cost, untimed
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        ctx = sampler if sampler is not None else _Null()
        with ctx, torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(replays):
                g.replay()
            e1.record(stream)
            e1.synchronize()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    steps = args.steps
    spg = max(d for d in range(1, min(steps, 100) + 1) if steps % d == 0)   # steps per graph
    g_main = capture(spg)
    sampler = ClockSampler(local)
    ms = time_graph(g_main, steps // spg, sampler)
    del g_main
    if bf.stream_status(stream) != 0:
        raise SystemExit("device-side error in the timed region")
    launches = steps * R
    us_per_gemm = ms * 1e3 / launches
    tok_s = M * launches / (ms / 1e3)
    b_launch = alg_bytes(M, n_loc, K)
    achieved = b_launch / (us_per_gemm * 1e-6) / 1e9
    # over several GPUs each rank also stores its [M, n_loc] slice into the
    # other ranks' outputs (NVLink)
    peer_bytes = 2 * M * n_loc * (world - 1) if space is not None else 0
    workload = f"{args.fmt}_gemm_m{M}_k{K}_n{N}"
    # this library's kernels per GEMM call (the gathered path is the decode kernel)
    k_per_gemm = ((M + 31) // 32 if space is not None else
                  bf.gemm_launches(M, n_loc, K, props.multi_processor_count))
    out = {
        "metric": metric_name(args.fmt, K, N),
        "value": round(tok_s, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms / steps, 6),
        "us_per_gemm": round(us_per_gemm, 4),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "fp16 (fp32 accumulate)",
        "data": "synthetic (seeded torch RNG, BASELINE config distributions)",
        "config": {
            "workload": workload, "format": args.fmt, "M": M, "N": N, "K": K,
            "parallelism": (f"tp{world} (N-split, all-gather fused into the GEMM epilogue: NVLink peer stores)"
                            if space is not None else f"tp{world} (N-split + NCCL all-gather)") if world > 1
                           else "single GPU",
            "weight_copies": R, "weight_set_bytes": R * wbytes,
            "l2": f"inputs larger than L2: {R} rotating weight copies, {R * wbytes / 1e6:.0f} MB > 2x L2 "
                  f"({l2 / 1e6:.0f} MB)",
            "timing": f"CUDA graph of {spg} steps x {R} back-to-back GEMM launches (PDL on), replayed "
                      f"{steps // spg}x; CUDA events on the launching stream, max over ranks",
        },
        "gpu_launches": launches * k_per_gemm,
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_src,
            "alg_bytes_per_launch": b_launch, "traffic": profiled_traffic(workload, world),
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this per-rank "
                               f"workload (profiles/)" if profiled_traffic(workload, world) is not None
                               else "no ncu capture of this per-rank workload"),
            **({"peer_store_bytes_per_launch": peer_bytes,
                "achieved_with_peer_stores": round((b_launch + peer_bytes) / (us_per_gemm * 1e-6) / 1e9, 1)}
               if world > 1 else {}),
        },
        "parity": parity,
        "clocks": sampler.summary(),
    }

    if not args.no_extras:
        out["layerset"] = layerset(torch, bf, tp, dev, world, rank, args, hbm_peak)
    if world == 1 and not args.no_extras and not args.layerset_only:
        out["isolated_no_pdl"] = isolated_no_pdl(bf, capture, time_graph, min(steps, 50), R, M)
        out["sweep"] = sweep(torch, bf, dev, l2, hbm_peak, args)
        out["cublas_fp16"] = cublas_comparator(torch, bf, dev, l2, weights, a, args)
        out["config4_prefill"] = config4(torch, bf, dev, args, hbm_peak, tc_peak, peak_src)
        out["e2e"] = e2e(torch, bf, dev, weights, a, args, max(10, steps // 10))
        out["cpu_baseline"] = cpu_baseline(args)
    elif world > 1:
        out["e2e"] = e2e_tp(torch, bf, tp, dev, weights, a, args, N, max(10, steps // 10), space)

    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        if space is not None:
            space.close()
        dist.destroy_process_group()


def _time_on(torch, g, st):
    """Replay graph g on stream st once untimed, then once between CUDA events on st."""
    with torch.cuda.stream(st):
        g.replay()
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        g.replay()
        e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *e):
        return False


def isolated_no_pdl(bf, capture, time_graph, steps, R, M):
    bf.set_pdl(False)
    try:
        g = capture(steps)
        ms = time_graph(g, 1)
        del g
    finally:
        bf.set_pdl(True)
    us = ms * 1e3 / (steps * R)
    return {"us_per_gemm": round(us, 4), "tokens_per_s": round(M / (us * 1e-6), 1),
            "note": "same graph with programmatic dependent launch disabled"}


def sweep(torch, bf, dev, l2, hbm_peak, args):
    rows = []
    cases = [("q4k", 1, 5120, 5120), ("q4k", 8, 5120, 5120), ("q4k", 32, 5120, 5120), ("q4k", 32, 17408, 5120),
             ("q4_0", 1, 5120, 5120), ("q4_0", 8, 5120, 5120), ("q4_0", 32, 5120, 5120),
             ("q4_0_ggml", 32, 5120, 5120), ("q5k", 32, 5120, 5120), ("q6k", 32, 5120, 5120),
             ("q4k_swiglu", 32, 17408, 5120)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 99)
    for fmt, m, n, k in cases:
        wbytes = n * k * {"q5k": 22, "q6k": 26.25}.get(fmt, 18) // 32 * (2 if fmt == "q4k_swiglu" else 1)
        wbytes = int(wbytes)
        R = max(2, math.ceil(2.2 * l2 / wbytes))
        if fmt == "q4k":
            w0 = make_q4k_weights(torch, n, k, gen, dev)
            ws = [w0] + [w0.clone() for _ in range(R - 1)]
        elif fmt == "q4k_swiglu":
            g0, u0 = make_q4k_weights(torch, n, k, gen, dev), make_q4k_weights(torch, n, k, gen, dev)
            ws = [(g0, u0)] + [(g0.clone(), u0.clone()) for _ in range(R - 1)]
        elif fmt == "q5k":
            w0 = make_q5k_weights(torch, n, k, gen, dev)
            ws = [w0] + [w0.clone() for _ in range(R - 1)]
        elif fmt == "q6k":
            b0, d0 = make_q6k_weights(torch, bf, n, k, gen, dev)
            ws = [(b0, d0)] + [(b0.clone(), d0.clone()) for _ in range(R - 1)]
        elif fmt == "q4_0_ggml":
            w0 = make_q4_0_ggml_weights(torch, n, k, gen, dev)
            ws = [w0] + [w0.clone() for _ in range(R - 1)]
        else:
            q, s = make_q4_0_weights(torch, n, k, gen, dev)
            ws = [(q, s)] + [(q.clone(), s.clone()) for _ in range(R - 1)]
        a = torch.randn((m, k), device=dev, generator=gen).half()
        c = torch.empty((m, n), dtype=torch.float16, device=dev)
        st = torch.cuda.Stream(device=dev)

        def step():
            for w in ws:
                if fmt == "q4k":
                    bf.gemm_q4k(w, a, out=c, stream=st)
                elif fmt == "q4k_swiglu":
                    bf.gemm_q4k_swiglu(w[0], w[1], a, out=c, stream=st)
                elif fmt == "q5k":
                    bf.gemm_q5k(w, a, out=c, stream=st)
                elif fmt == "q6k":
                    bf.gemm_q6k(w[0], w[1], a, out=c, stream=st)
                elif fmt == "q4_0_ggml":
                    bf.gemm_q4_0_ggml(w, a, out=c, stream=st)
                else:
                    bf.gemm_q4_0(w[0], w[1], a, out=c, stream=st)

        with torch.cuda.stream(st):
            for _ in range(3):
                step()
        st.synchronize()
        nsteps = max(4, min(40, 4000 // R))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for _ in range(nsteps):
                step()
        ms = _time_on(torch, g, st)
        assert bf.stream_status(st) == 0
        us = ms * 1e3 / (nsteps * R)
        gbs = (wbytes + 2 * m * k + 2 * m * n) / (us * 1e-6) / 1e9
        rows.append({"format": fmt, "M": m, "N": n, "K": k, "us_per_gemm": round(us, 3),
                     "tokens_per_s": round(m / (us * 1e-6), 1), "GB_s": round(gbs, 1),
                     "hbm_frac": round(gbs / hbm_peak, 4)})
        del g, ws
        torch.cuda.empty_cache()
    return rows


def layerset(torch, bf, tp, dev, world, rank, args, hbm_peak, m=32, sweeps=10):
    """a 27B-class dense decoder layer set in Q4_K at M = 32,
    `args.layers` distinct layers streamed back to back: fused QKV 5120 ->
    10240, O 8192 -> 5120, gate/up 5120 -> 2 x 17408 as one fused SwiGLU GEMM,
    down 17408 -> 5120. Attention itself is outside the path: a fixed [32,
    8192] tensor stands in for its output. Over `world` GPUs every weight is
    column-split (tp.shard_rows) and each output all-gathered (NCCL), so every
    rank holds the full activations for the next GEMM. Timed as a CUDA graph of
    one sweep over all layers, CUDA events, max over ranks."""
    import torch.distributed as dist
    L = args.layers
    shapes = {"qkv": (10240, 5120), "o": (5120, 8192), "gate": (17408, 5120), "up": (17408, 5120),
              "down": (5120, 17408)}
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 1000 + rank)
    layers = []
    local_bytes = 0
    for _ in range(L):
        lw = {}
        for name, (n, k) in shapes.items():
            r0, r1 = tp.shard_rows(n, world, rank)
            lw[name] = make_q4k_weights(torch, r1 - r0, k, gen, dev)
            local_bytes += (r1 - r0) * k * 18 // 32
        layers.append(lw)
    total_bytes = sum(n * k * 18 // 32 for n, k in shapes.values()) * L
    x = (torch.randn((m, 5120), device=dev, generator=gen) / 64).half()
    attn = (torch.randn((m, 8192), device=dev, generator=gen) / 64).half()
    full = {name: torch.empty((m, n), dtype=torch.float16, device=dev) for name, (n, _) in shapes.items()}
    st = torch.cuda.Stream(device=dev)
    # over several GPUs every GEMM's all-gather runs in its epilogue: one call
    # site (output buffer, flags) per layer and projection
    ops = ("qkv", "o", "gate", "down")
    space = (tp.GatherSpace([(m, shapes[name][0]) for _ in range(L) for name in ops]) if world > 1 else None)

    def site(layer, name):
        return layer * len(ops) + ops.index(name)

    def sweep():
        h, h_site = x, None
        for li, lw in enumerate(layers):
            if space is None:
                bf.gemm_q4k(lw["qkv"], h, out=full["qkv"], stream=st)   # would feed attention (outside the path)
                o = bf.gemm_q4k(lw["o"], attn, out=full["o"], stream=st)
                g = bf.gemm_q4k_swiglu(lw["gate"], lw["up"], o, out=full["gate"], stream=st)
                h = bf.gemm_q4k(lw["down"], g, out=full["down"], stream=st)
            else:
                tp.gemm_q4k_gather(lw["qkv"], h, space, site(li, "qkv"), wait_site=h_site, stream=st)
                o = tp.gemm_q4k_gather(lw["o"], attn, space, site(li, "o"), stream=st)
                g = tp.gemm_q4k_swiglu_gather(lw["gate"], lw["up"], o, space, site(li, "gate"),
                                              wait_site=site(li, "o"), stream=st)
                h = tp.gemm_q4k_gather(lw["down"], g, space, site(li, "down"), wait_site=site(li, "gate"), stream=st)
                h_site = site(li, "down")

    with torch.cuda.stream(st):
        sweep()
        st.synchronize()
        assert bf.stream_status(st) == 0
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            sweep()
        g.replay()
        st.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(sweeps):
            g.replay()
        e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / sweeps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del g
    fused = None
    if world == 1:
        # the same layers through busfill_gemm_q4k_sweep, two layers (eight
        # ops) per launch, ordered so that no op directly follows the op whose
        # output it reads: O1, O2, QKV1, gate/up1 (after O1), gate/up2 (after
        # O2), down1, down2, QKV2 (after down1); an odd last layer runs alone
        # (O, QKV, gate/up, down). Outputs never overlap an input of their own
        # launch: the second layer's down output alternates between two
        # buffers from launch to launch.
        o2 = [full["o"], torch.empty_like(full["o"])]
        gu = [full["gate"], torch.empty_like(full["gate"])]
        q2 = [full["qkv"], torch.empty_like(full["qkv"])]
        d1 = torch.empty_like(full["down"])
        dl = [full["down"], torch.empty_like(full["down"])]

        def sweep_fused():
            h = x
            for j in range(0, L - 1, 2):
                la, lb = layers[j], layers[j + 1]
                dn = dl[(j // 2) & 1]
                bf.gemm_q4k_sweep([{"w": la["o"], "a": attn, "out": o2[0]},
                                   {"w": lb["o"], "a": attn, "out": o2[1]},
                                   {"w": la["qkv"], "a": h, "out": q2[0]},
                                   {"w": la["gate"], "w_up": la["up"], "a": o2[0], "out": gu[0], "dep": 0},
                                   {"w": lb["gate"], "w_up": lb["up"], "a": o2[1], "out": gu[1], "dep": 1},
                                   {"w": la["down"], "a": gu[0], "out": d1, "dep": 3},
                                   {"w": lb["down"], "a": gu[1], "out": dn, "dep": 4},
                                   {"w": lb["qkv"], "a": d1, "out": q2[1], "dep": 5}], stream=st)
                h = dn
            if L % 2:
                lw = layers[L - 1]
                dn = dl[((L - 1) // 2) & 1]
                bf.gemm_q4k_sweep([{"w": lw["o"], "a": attn, "out": o2[0]},
                                   {"w": lw["qkv"], "a": h, "out": q2[0]},
                                   {"w": lw["gate"], "w_up": lw["up"], "a": o2[0], "out": gu[0], "dep": 0},
                                   {"w": lw["down"], "a": gu[0], "out": d1, "dep": 2}],
                                  stream=st)

        with torch.cuda.stream(st):
            sweep_fused()
            st.synchronize()
            assert bf.stream_status(st) == 0
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=st):
                sweep_fused()
            g2.replay()
            st.synchronize()
            e0.record(st)
            for _ in range(sweeps):
                g2.replay()
            e1.record(st)
        e1.synchronize()
        assert bf.stream_status(st) == 0
        ms2 = e0.elapsed_time(e1) / sweeps
        del g2
        fused = {"ms_per_sweep": round(ms2, 4), "us_per_layer": round(ms2 * 1e3 / L, 2),
                 "tokens_per_s": round(m / (ms2 * 1e-3), 1),
                 "hbm_frac_per_gpu": round(local_bytes / (ms2 * 1e-3) / 1e9 / hbm_peak, 4),
                 "kernels": "busfill_gemm_q4k_sweep x1 per two layers (8 ops, stream-K over all SMs)"}
    del layers
    if space is not None:
        torch.cuda.synchronize(dev)
        dist.barrier()
        space.close()
    torch.cuda.empty_cache()
    return {"layers": L, "M": m, "ms_per_sweep": round(ms, 4), "tokens_per_s": round(m / (ms * 1e-3), 1),
            "weight_bytes_total": total_bytes, "weight_bytes_per_gpu": local_bytes,
            "GB_s_total": round(total_bytes / (ms * 1e-3) / 1e9, 1),
            "hbm_frac_per_gpu": round(local_bytes / (ms * 1e-3) / 1e9 / hbm_peak, 4),
            "n_gpus": world, "parallelism": (f"tp{world} column split, all-gather fused into every GEMM's epilogue "
                                             f"(NVLink peer stores + flags)") if world > 1 else "single GPU", "kernels": "busfill_gemm_q4k x3 + busfill_gemm_q4k_swiglu per layer",
            "timing": f"CUDA graph of one {L}-layer sweep, {sweeps} replays, CUDA events, max over ranks",
            **({"layer_sweep_kernel": fused} if fused else {})}


def config4(torch, bf, dev, args, hbm_peak, tc_peak, peak_src):
    """Q4_K down-proj (K=17408, N=5120) and up-proj
    (K=5120, N=17408) at M in {1, 128, 512, 2048}, through the default
    dispatch (prefill kernel for large batches, decode kernel otherwise),
    against the tensor roofline (2 M N K flops) and the HBM roofline
    (algorithmic bytes), with cuBLAS fp16 on the dequantized weights beside it.
    Each GEMM is timed alone (CUDA events around 5 back-to-back calls after 2
    warm-up calls; the weights, 50 MB, are re-read every call)."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 4)
    rows = []
    st = torch.cuda.Stream(device=dev)

    def timed(fn, it=5):
        with torch.cuda.stream(st):
            for _ in range(2):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(it):
                fn()
            e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / it

    for k, n in ((17408, 5120), (5120, 17408)):
        w = make_q4k_weights(torch, n, k, gen, dev)
        w16 = bf.dequant_q4k(w, k, stream=st)
        for m in (1, 128, 512, 2048):
            a = torch.randn((m, k), device=dev, generator=gen).half()
            c = torch.empty((m, n), dtype=torch.float16, device=dev)
            us = timed(lambda: bf.gemm_q4k(w, a, out=c, stream=st))
            assert bf.stream_status(st) == 0
            us_cb = timed(lambda: torch.matmul(a, w16.t(), out=c))
            fl = 2.0 * m * n * k
            tf = fl / (us * 1e-6) / 1e12
            gbs = alg_bytes(m, n, k) / (us * 1e-6) / 1e9
            rows.append({"M": m, "N": n, "K": k, "kernel": "prefill" if bf.uses_prefill(m, n, k) else "decode",
                         "us": round(us, 2), "tflops": round(tf, 1), "tensor_frac": round(tf / tc_peak, 4),
                         "GB_s": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 4),
                         "cublas_fp16_us": round(us_cb, 2)})
        del w, w16
        torch.cuda.empty_cache()
    return {"rows": rows, "tensor_peak_tflops": tc_peak, "hbm_peak_gbs": hbm_peak, "peak_source": peak_src,
            "note": "tensor_frac against the measured dense bf16 cuBLAS peak (burst); fp16 runs at the same rate"}


def cublas_comparator(torch, bf, dev, l2, weights, a, args):
    """torch.matmul (cuBLAS) on the same weights dequantized to fp16
    (kernels/q4k_batched.py:111-113, bench/baseline_torch.py:19-25)."""
    n, k = (weights[0].shape[0] if args.fmt == "q4k" else weights[0][0].shape[0]), args.k
    if args.fmt == "q4k":
        w16 = bf.dequant_q4k(weights[0], k)
    else:
        w16 = bf.dequant_q4_0(weights[0][0], weights[0][1])
    R = max(2, math.ceil(2.2 * l2 / (n * k * 2)))
    ws = [w16] + [w16.clone() for _ in range(R - 1)]
    st = torch.cuda.Stream(device=dev)
    c = torch.empty((a.shape[0], n), dtype=torch.float16, device=dev)

    def step():
        for w in ws:
            torch.matmul(a, w.t(), out=c)

    with torch.cuda.stream(st):
        for _ in range(3):
            step()
    st.synchronize()
    nsteps = max(4, min(50, 1000 // R))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for _ in range(nsteps):
            step()
    us = _time_on(torch, g, st) * 1e3 / (nsteps * R)
    del g, ws
    torch.cuda.empty_cache()
    m = a.shape[0]
    return {"us_per_gemm": round(us, 4), "tokens_per_s": round(m / (us * 1e-6), 1),
            "fp16_weight_bytes": n * k * 2, "copies": R}


def e2e(torch, bf, dev, weights, a, args, steps):
    """The same metric through the public API with HOST buffers: every step
    copies its calls' activations from pinned host memory, runs the C-ABI
    GEMMs and reads their outputs back to pinned host memory; every call has
    its own host and device buffers. Three measurements:

    * value: the calls of a step (one per weight copy) captured once as a
      CUDA graph, their transfers grouped `group` calls at a time (one
      host-to-device copy of the group's activations, one device-to-host
      copy of its outputs, on their own streams) so that group g+1's input
      copy and group g-1's output copy overlap group g's GEMMs, as a serving
      loop batches its transfers: a 327 KB copy each way per call is bound
      by PCIe at ~16 us a call on B200 boxes (both directions at once),
      more than the GEMM; the graph is replayed `steps` times, CUDA events
      around the replays.
    * per_call_copies: the same with one copy each way per call.
    * eager_serial: the calls issued one by one from Python on a single
      stream (copy, GEMM, copy), host overheads included.
    """
    m, k = a.shape
    n = weights[0].shape[0] if args.fmt == "q4k" else weights[0][0].shape[0]
    R = len(weights)
    h_a = torch.empty((R, m, k), dtype=torch.float16).pin_memory()
    h_a.copy_(a.cpu().expand(R, m, k))
    h_c = torch.empty((R, m, n), dtype=torch.float16).pin_memory()
    d_a = torch.empty((R, m, k), dtype=torch.float16, device=dev)
    d_c = torch.empty((R, m, n), dtype=torch.float16, device=dev)
    s_cmp, s_in, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))

    def gemm(i, w, st):
        if args.fmt == "q4k":
            bf.gemm_q4k(w, d_a[i], out=d_c[i], stream=st)
        else:
            bf.gemm_q4_0(w[0], w[1], d_a[i], out=d_c[i], stream=st)

    def serial_step():
        for i, w in enumerate(weights):
            d_a[i].copy_(h_a[i], non_blocking=True)
            gemm(i, w, s_cmp)
            h_c[i].copy_(d_c[i], non_blocking=True)

    def transfer_groups(group):
        """Calls per transfer: `group` at a time, ramping up from and down to
        one call at the step's ends, where a copy has no GEMM to hide behind."""
        if group == 1:
            return [1] * R
        ramp = [1, group - 1]
        sizes = ramp[:]
        left = R - 2 * sum(ramp)
        while left > 0:
            sizes.append(min(group, left))
            left -= sizes[-1]
        sizes += ramp[::-1]
        assert sum(sizes) == R
        return sizes

    def pipelined_step(group):
        fork = torch.cuda.Event()
        fork.record(s_cmp)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        g1 = 0
        for size in transfer_groups(group):
            g0, g1 = g1, g1 + size
            e_in, e_cmp = torch.cuda.Event(), torch.cuda.Event()
            with torch.cuda.stream(s_in):
                d_a[g0:g1].copy_(h_a[g0:g1], non_blocking=True)
                e_in.record(s_in)
            s_cmp.wait_event(e_in)
            for i in range(g0, g1):
                gemm(i, weights[i], s_cmp)
            e_cmp.record(s_cmp)
            s_out.wait_event(e_cmp)
            with torch.cuda.stream(s_out):
                h_c[g0:g1].copy_(d_c[g0:g1], non_blocking=True)
        join_in, join_out = torch.cuda.Event(), torch.cuda.Event()
        join_in.record(s_in)
        join_out.record(s_out)
        s_cmp.wait_event(join_in)
        s_cmp.wait_event(join_out)

    def timed(fn):
        with torch.cuda.stream(s_cmp):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s_cmp)
            for _ in range(steps):
                fn()
            e1.record(s_cmp)
        e1.synchronize()
        return e0.elapsed_time(e1)

    # warm-up, eager (also makes the library's per-stream words before capture)
    group = 4 if R >= 12 else 1
    with torch.cuda.stream(s_cmp):
        for _ in range(2):
            serial_step()
            pipelined_step(group)
            pipelined_step(1)
    torch.cuda.synchronize(dev)
    ms_serial = timed(serial_step)

    def graph_ms(grp):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s_cmp):
            pipelined_step(grp)
        with torch.cuda.stream(s_cmp):
            g.replay()
        torch.cuda.synchronize(dev)
        h_c.zero_()
        t = timed(g.replay)
        assert bf.stream_status(s_cmp) == 0
        # every call's output reached the host
        assert torch.equal(h_c[R - 1], d_c[R - 1].cpu()) and torch.equal(h_c[0], d_c[0].cpu())
        del g
        return t

    ms = graph_ms(group)
    ms_1 = graph_ms(1)
    calls = steps * R
    return {"value": round(m * calls / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": R * m * k * 2, "d2h_bytes_per_step": R * m * n * 2,
            "us_per_call": round(ms * 1e3 / calls, 3), "steps": steps, "calls_per_step": R,
            "calls_per_transfer": transfer_groups(group),
            "path": "pinned host A -> cudaMemcpyAsync of a group of calls' activations (stream 2) -> busfill_gemm_* "
                    "(C ABI via ctypes, stream 1) -> cudaMemcpyAsync of their outputs (stream 3) -> pinned host C; "
                    "one step's calls captured as a CUDA graph",
            "per_call_copies": {"value": round(m * calls / (ms_1 / 1e3), 1), "unit": "tokens/s",
                                "us_per_call": round(ms_1 * 1e3 / calls, 3),
                                "path": "the same with one copy each way per call"},
            "eager_serial": {"value": round(m * calls / (ms_serial / 1e3), 1), "unit": "tokens/s",
                             "us_per_call": round(ms_serial * 1e3 / calls, 3),
                             "path": "the same calls from Python, one stream, no graph"}}


def e2e_tp(torch, bf, tp, dev, weights, a, args, n_total, steps, space=None):
    """e2e with the weight rows split over the ranks: every call copies the
    activations from pinned host memory, runs this rank's rows through the C
    ABI with the all-gather in the GEMM epilogue (Q4_K; NCCL after the GEMM for
    Q4_0), waits for the gathered output and reads the full C back to pinned
    host memory. Max over ranks."""
    import torch.distributed as dist

    m, k = a.shape
    h_a = torch.empty((m, k), dtype=torch.float16).pin_memory()
    h_a.copy_(a.cpu())
    h_c = torch.empty((m, n_total), dtype=torch.float16).pin_memory()
    d_a = torch.empty_like(a)
    d_c = torch.empty((m, n_total), dtype=torch.float16, device=dev)
    st = torch.cuda.Stream(device=dev)

    def step():
        for i, w in enumerate(weights):
            d_a.copy_(h_a, non_blocking=True)
            if space is not None:
                out = tp.gemm_q4k_gather(w, d_a, space, i, stream=st)
                space.wait(i, stream=st)
                h_c.copy_(out, non_blocking=True)
            else:
                tp.gemm_q4_0_tp(w[0], w[1], d_a, n_total, out=d_c)
                h_c.copy_(d_c, non_blocking=True)

    with torch.cuda.stream(st):
        for _ in range(2):
            step()
        st.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            step()
        e1.record(st)
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    assert bf.stream_status(st) == 0
    calls = steps * len(weights)
    return {"value": round(m * calls / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": len(weights) * m * k * 2, "d2h_bytes_per_step": len(weights) * m * n_total * 2,
            "us_per_call": round(ms * 1e3 / calls, 3), "steps": steps,
            "path": ("pinned host A -> cudaMemcpyAsync -> busfill_gemm_q4k_gather on this rank's rows (C ABI; "
                     "all-gather in the epilogue) -> busfill_gather_wait -> pinned host C (every rank), max over "
                     "ranks") if space is not None else
                    ("pinned host A -> cudaMemcpyAsync -> busfill_gemm_* on this rank's rows (C ABI) -> "
                     "NCCL all-gather -> pinned host C (every rank), max over ranks")}


# ---------------------------------------------------------------------------
# CPU legs (the only places bench.py runs the oracle)
# ---------------------------------------------------------------------------
def _cpu_dequant_gemm(orc, fmt, w, a, k, pool, nchunks):
    import numpy as np
    import torch
    n = w.shape[0] if fmt == "q4k" else w[0].shape[0]
    bounds = [(i * n // nchunks, (i + 1) * n // nchunks) for i in range(nchunks)]
    t0 = time.perf_counter()
    if fmt == "q4k":
        parts = list(pool.map(lambda b: orc.dequant_q4k_f32(w[b[0]:b[1]], k), bounds))
    else:
        parts = list(pool.map(lambda b: orc.dequant_q4_0_planes_f32(w[0][b[0]:b[1]], w[1][b[0]:b[1]]), bounds))
    wf = np.concatenate(parts)
    t1 = time.perf_counter()
    c = torch.from_numpy(a).float() @ torch.from_numpy(wf).T          # kernels/q4k_batched.py:100
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1, c


def cpu_baseline(args, reps=5):
    from concurrent.futures import ThreadPoolExecutor

    import torch

    from oracle import q4_oracle as orc
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    m, n, k = args.m, args.n, args.k
    w = orc.gen_q4k(n, k, seed=args.seed) if args.fmt == "q4k" else orc.gen_q4_0(n, k, seed=args.seed)
    a = orc.gen_activations(m, k, seed=args.seed + 1)
    with ThreadPoolExecutor(cores) as pool:
        _cpu_dequant_gemm(orc, args.fmt, w, a, k, pool, 4 * cores)
        ts = [_cpu_dequant_gemm(orc, args.fmt, w, a, k, pool, 4 * cores) for _ in range(reps)]
    deq = statistics.median(t[0] for t in ts)
    mm = statistics.median(t[1] for t in ts)
    return {"value": round(m / (deq + mm), 2), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{reps} full GEMMs (M={m}, K={k}, N={n}): oracle dequant (numpy, {cores} threads) + "
                      f"torch fp32 matmul ({cores} threads), median",
            "dequant_s": round(deq, 4), "matmul_s": round(mm, 4)}


def run_reference(args, budget_s=90.0):
    """The reference's CPU dequantize-then-matmul path, timed on the host
    cores: each step is one full GEMM (M x N x K) through the same code and
    chunking as cpu_baseline (the oracle's dequant in 4 x cores row chunks on
    a thread pool, then one torch fp32 matmul), so the two CPU numbers measure
    the same thing. Up to --steps steps, stopping early once `budget_s` of
    timed work has run (the count timed is reported)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor

    import torch

    from oracle import q4_oracle as orc
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    m, n, k = args.m, args.n, args.k
    w = orc.gen_q4k(n, k, seed=args.seed) if args.fmt == "q4k" else orc.gen_q4_0(n, k, seed=args.seed)
    a = orc.gen_activations(m, k, seed=args.seed + 1)
    times = []
    with ThreadPoolExecutor(cores) as pool:
        for _ in range(max(args.warmup, 1)):
            _cpu_dequant_gemm(orc, args.fmt, w, a, k, pool, 4 * cores)
        t_start = time.perf_counter()
        for _ in range(args.steps):
            d, mm, _c = _cpu_dequant_gemm(orc, args.fmt, w, a, k, pool, 4 * cores)
            times.append(d + mm)
            if time.perf_counter() - t_start > budget_s:
                break
    el = sum(times)
    value = m * len(times) / el
    out = {"metric": metric_name(args.fmt, k, n),
           "value": round(value, 2), "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
           "steps": len(times), "steps_requested": args.steps, "warmup": max(args.warmup, 1),
           "ms_per_step": round(el / len(times) * 1e3, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic (seeded numpy RNG, BASELINE config distributions)",
           "config": {"workload": f"{args.fmt}_gemm_m{m}_k{k}_n{n}", "format": args.fmt, "M": m, "N": n, "K": k,
                      "parallelism": "host CPU"},
           "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
                            "sample": f"{len(times)} full GEMMs (M={m}, K={k}, N={n}): oracle dequant (numpy, "
                                      f"{cores} threads, {4 * cores} row chunks) + torch fp32 matmul ({cores} "
                                      f"threads), the cpu_baseline code path"},
           "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_busfill(args)


if __name__ == "__main__":
    main()
