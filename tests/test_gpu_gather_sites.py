"""Chained gathered GEMMs whose launch shape changes from call to call.

A consuming gathered GEMM counts the calls of its call site on the device
(busfill_gather.wait_gen) to know which epoch of its producer's tile counter
to wait for. The count must hold whatever grid each call has: M <= 16 and
M > 16 run different batch tiles, and the K split (cluster size) changes the
number of CTAs. Here one producer site A and one consumer site B, in a group
of one rank (every peer store and counter is this GPU's own), are called with
M and the forced K split changing every call, eagerly and replayed from a
CUDA graph; every consumer output is checked against the oracle, so a wrong
epoch shows as a timeout status or as activations of another call.
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
K0, N1, N2 = 1280, 1024, 512           # A: [M, K0] x [N1, K0]^T; B: [M, N1] x [N2, N1]^T
SCHEDULE = [(8, 1), (32, 3), (17, 0), (32, 2), (8, 4), (1, 0), (24, 1)]   # (M, forced K split)


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _gather(out, flag_ptr, n, wait=None, wait_gen=None, wait_tiles=0):
    g = tp.Gather()
    g.npeers, g.col_off, g.ldc = 1, 0, n
    g.out[0] = out.data_ptr()
    g.flag[0] = flag_ptr
    if wait is not None:
        g.wait, g.wait_gen, g.nwait = wait, wait_gen, 1
        g.wait_tiles[0] = wait_tiles
    return g


class Chain:
    def __init__(self):
        self.wa_np = orc.gen_q4k(N1, K0, seed=71)
        self.wb_np = orc.gen_q4k(N2, N1, seed=72)
        self.wa, self.wb = cu(self.wa_np), cu(self.wb_np)
        self.words = torch.zeros(64, dtype=torch.int32, device=DEV)    # flag A, flag B, wait_gen[2] of B
        base = self.words.data_ptr()
        self.flag_a, self.flag_b, self.gen_b = base, base + 64, base + 128
        self.out_a = torch.zeros((32, N1), dtype=torch.float16, device=DEV)
        self.lib = bf.load_library()

    def call(self, x, out_b, ksplit, stream):
        m = x.shape[0]
        bf.set_ksplit(ksplit)
        try:
            ga = _gather(self.out_a, self.flag_a, N1)
            st = self.lib.busfill_gemm_q4k_gather(ctypes.c_void_p(self.wa.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                                  m, N1, K0, ctypes.byref(ga), ctypes.c_void_p(stream.cuda_stream))
            assert st == 0
            gb = _gather(out_b, self.flag_b, N2, wait=self.flag_a, wait_gen=self.gen_b, wait_tiles=N1 // 128)
            st = self.lib.busfill_gemm_q4k_gather(ctypes.c_void_p(self.wb.data_ptr()),
                                                  ctypes.c_void_p(self.out_a.data_ptr()), m, N2, N1,
                                                  ctypes.byref(gb), ctypes.c_void_p(stream.cuda_stream))
            assert st == 0
        finally:
            bf.set_ksplit(0)

    def check(self, x_np, out_b):
        a_ref = orc.gemm_ref(x_np, orc.dequant_q4k_f32(self.wa_np, K0)).astype(np.float16)
        b_ref = orc.gemm_ref(a_ref, orc.dequant_q4k_f32(self.wb_np, N1))
        max_abs, rel, finite = orc.gemm_errors(out_b.float().cpu().numpy(), b_ref)
        assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2, (max_abs, rel)


def inputs(seed0):
    # activations scaled by 1/4096 (exact in fp16) so that the chained product
    # of two config-2 weights stays near the magnitudes the absolute gate is for
    xs = [(orc.gen_activations(m, K0, seed=seed0 + i).astype(np.float32) / 4096).astype(np.float16)
          for i, (m, _) in enumerate(SCHEDULE)]
    outs = [torch.zeros((m, N2), dtype=torch.float16, device=DEV) for m, _ in SCHEDULE]
    return xs, [cu(x) for x in xs], outs


def test_changing_grids_at_one_site_eager():
    ch = Chain()
    st = torch.cuda.Stream()
    xs, xd, outs = inputs(100)
    for rnd in range(2):
        for (m, ks), x, o in zip(SCHEDULE, xd, outs):
            ch.call(x, o, ks, st)
        assert bf.stream_status(st) == 0
        for x_np, o in zip(xs, outs):
            ch.check(x_np, o)


def test_changing_grids_at_one_site_graph_replay():
    ch = Chain()
    st = torch.cuda.Stream()
    xs, xd, outs = inputs(200)
    with torch.cuda.stream(st):
        for (m, ks), x, o in zip(SCHEDULE, xd, outs):      # eager first (the library's per-stream words)
            ch.call(x, o, ks, st)
    assert bf.stream_status(st) == 0
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for (m, ks), x, o in zip(SCHEDULE, xd, outs):
            ch.call(x, o, ks, st)
    for o in outs:
        o.zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        with torch.cuda.stream(st):
            g.replay()
        assert bf.stream_status(st) == 0
    for x_np, o in zip(xs, outs):
        ch.check(x_np, o)
    del g
