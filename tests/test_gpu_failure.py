"""Failure detection on the GPU without a GPU fault: a bounded device-side wait
that runs out. A gathered GEMM is told to wait for a flag word that nothing
ever sets; its activation producer gives up after the 1 s bound, records the
error, and the kernel winds down. busfill_stream_status must report
BUSFILL_ERR_DEVICE_TIMEOUT (with the activation-producer bit), and the same
context must then run a normal GEMM correctly. No trap, no bad address, no
unbounded loop: only a wait whose partner never comes.
"""
import ctypes

import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402
from busfill_b200 import tp  # noqa: E402

DEV = "cuda:0"
TIMEOUT = -7  # BUSFILL_ERR_DEVICE_TIMEOUT
ACT_PRODUCER_BIT = 2


def test_wait_that_runs_out_reports_timeout_and_context_survives():
    m, n, k = 8, 256, 512
    blocks = torch.from_numpy(orc.gen_q4k(n, k, seed=5)).to(DEV)
    a_np = orc.gen_activations(m, k, seed=6)
    a = torch.from_numpy(a_np).to(DEV)
    out = torch.zeros((m, n), dtype=torch.float16, device=DEV)
    words = torch.zeros(16, dtype=torch.int32, device=DEV)   # tile counter, the never-raised wait word, wait count
    base = words.data_ptr()
    g = tp.Gather()
    g.npeers = 1
    g.col_off = 0
    g.ldc = n
    g.out[0] = out.data_ptr()
    g.flag[0] = base
    g.wait = base + 32          # stays 0: the wait for 2 tiles never completes
    g.wait_gen = base + 48
    g.nwait = 1
    g.wait_tiles[0] = n // 128
    lib = bf.load_library()
    st = lib.busfill_gemm_q4k_gather(ctypes.c_void_p(blocks.data_ptr()), ctypes.c_void_p(a.data_ptr()), m, n, k,
                                     ctypes.byref(g), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0                                           # the launch itself is fine
    status, bits = bf.stream_status_bits()
    assert status == TIMEOUT, status
    assert bits & ACT_PRODUCER_BIT, bits
    assert lib.busfill_last_failure_detail() & 0x80000000     # a failure record names the waiting warp
    # the context is still usable: a plain GEMM right after is correct
    c = bf.gemm_q4k(blocks, a)
    assert bf.stream_status() == 0
    max_abs, rel, finite = orc.gemm_errors(c.float().cpu().numpy(),
                                           orc.gemm_ref(a_np, orc.dequant_q4k_f32(orc.gen_q4k(n, k, seed=5), k)))
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2


def test_sweep_dependency_wait_that_runs_out_reports_timeout_and_next_sweep_is_right():
    """The layer sweep's dependency wait (an op reading an earlier op's output
    waits for that op's stored-tile count): with BUSFILL_OPT_SWEEP_UNMET_DEP
    the dependent op waits for one tile more than exists, its activation
    producer gives up after the 1 s bound, and busfill_stream_status reports
    the timeout and clears the stream's error words and sweep counters; the
    next sweep on the same stream (counters back at zero) is right."""
    m = 8
    w0_np, w1_np = orc.gen_q4k(512, 512, seed=81), orc.gen_q4k(256, 512, seed=82)
    a_np = (orc.gen_activations(m, 512, seed=83).astype(np.float32) / 64).astype(np.float16)
    w0, w1, a = (torch.from_numpy(x).to(DEV) for x in (w0_np, w1_np, a_np))
    h = torch.empty((m, 512), dtype=torch.float16, device=DEV)
    y = torch.empty((m, 256), dtype=torch.float16, device=DEV)
    ops = [{"w": w0, "a": a, "out": h}, {"w": w1, "a": h, "out": y, "dep": 0}]
    lib = bf.load_library()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        bf.gemm_q4k_sweep(ops, stream=st)                    # makes the stream's workspace
        assert bf.stream_status(st) == 0
        assert lib.busfill_set_option(8, 1) == 0
        try:
            bf.gemm_q4k_sweep(ops, stream=st)                # the launch itself is fine
            status, bits = bf.stream_status_bits(st)
        finally:
            assert lib.busfill_set_option(8, 0) == 0
        assert status == TIMEOUT, status
        assert bits & ACT_PRODUCER_BIT, bits
        h.zero_()
        y.zero_()
        bf.gemm_q4k_sweep(ops, stream=st)
        assert bf.stream_status(st) == 0
    h_np = h.cpu().numpy()
    max_abs, rel, finite = orc.gemm_errors(h_np.astype(np.float32), orc.gemm_ref(a_np, orc.dequant_q4k_f32(w0_np, 512)))
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2
    want = orc.gemm_ref(h_np, orc.dequant_q4k_f32(w1_np, 512))
    got = y.float().cpu().numpy()
    assert np.all(np.isfinite(got))
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-3
