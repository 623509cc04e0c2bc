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
