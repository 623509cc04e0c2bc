"""GPU parity of the Q5_K path (busfill_gemm_q5k, busfill_dequant_q5k) through
the C ABI, against the oracle (gguf-py 0.19.0 Q5_K semantics, pinned by
tests/golden/q5k_gguf.npz).

Dequant: bit-exact fp16_rn(w32). GEMM: rel-L2 <= 1e-3 against an fp32 matmul
of the dequantized weights (the reference gate), every element within 0.6 plus
one fp16 ulp of the output (see check), and rel-L2 <= 5e-4 against float64
(the fp16 operand carries two roundings as for Q4_K).
"""
import os

import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402

DEV = "cuda:0"


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def test_dequant_q5k_bit_exact_gguf_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "q5k_gguf.npz"))
    for case in ("a", "b"):
        blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
        out = bf.dequant_q5k(cu(blocks), k)
        assert bf.stream_status() == 0
        with np.errstate(over="ignore"):
            want = w32.astype(np.float16)
        assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16)), case


def test_dequant_q5k_bit_exact_config_distribution():
    blocks = orc.gen_q5k(640, 5120, seed=5)
    out = bf.dequant_q5k(cu(blocks), 5120)
    assert bf.stream_status() == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), orc.dequant_q5k(blocks, 5120).view(np.uint16))


def check(c, a, w32):
    """Q5_K's values reach 31 (Q4 formats: 15), so outputs are about twice as
    large and one fp16 ulp of the output alone can exceed the reference's
    absolute bound: each element may miss by 0.6 plus one ulp (2^-10 |ref|),
    with the reference's rel-L2 <= 1e-3 unchanged."""
    got = c.float().cpu().numpy()
    ref = orc.gemm_ref(a, w32)
    max_abs, rel, finite = orc.gemm_errors(got, ref)
    assert finite and rel <= orc.GATE_REL_L2, (max_abs, rel)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= orc.GATE_MAX_ABS + 2.0 ** -10 * np.abs(ref)), max_abs
    exact = a.astype(np.float64) @ w32.astype(np.float64).T
    _, rel_t, _ = orc.gemm_errors(got, exact)
    assert rel_t <= 5e-4, rel_t


@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (8, 640, 1024), (17, 200, 2048), (32, 1280, 5120), (33, 384, 768),
                                   (5, 3840, 5120), (2, 512, 16384), (48, 1024, 512), (64, 2048, 1024)])
def test_gemm_q5k_decode(m, n, k):
    blocks = orc.gen_q5k(n, k, seed=m + n + k)
    a = orc.gen_activations(m, k, seed=m * 3 + k)
    c = bf.gemm_q5k(cu(blocks), cu(a))
    assert bf.stream_status() == 0
    check(c, a, orc.dequant_q5k_f32(blocks, k))


@pytest.mark.parametrize("bt", [128, 256, "pair"])
@pytest.mark.parametrize("m,n,k", [(128, 512, 512), (300, 640, 2048), (64, 256, 1024)])
def test_gemm_q5k_prefill(m, n, k, bt):
    bf.set_prefill_min_m(1)
    if bt == "pair":
        bf.set_prefill_pair(1)
    else:
        bf.set_prefill_pair(2)
        bf.set_prefill_batch_tile(bt)
    try:
        blocks = orc.gen_q5k(n, k, seed=m + 2 * n + k)
        a = orc.gen_activations(m, k, seed=m + k)
        c = bf.gemm_q5k(cu(blocks), cu(a))
        assert bf.stream_status() == 0
    finally:
        bf.set_prefill_min_m(0)
        bf.set_prefill_batch_tile(0)
        bf.set_prefill_pair(0)
    check(c, a, orc.dequant_q5k_f32(blocks, k))


@pytest.mark.parametrize("csize", [1, 3, 8])
def test_gemm_q5k_forced_ksplit(csize):
    bf.set_ksplit(csize)
    try:
        blocks = orc.gen_q5k(3072, 2048, seed=csize)
        a = orc.gen_activations(5, 2048, seed=csize + 1)
        c = bf.gemm_q5k(cu(blocks), cu(a))
        assert bf.stream_status() == 0
    finally:
        bf.set_ksplit(0)
    check(c, a, orc.dequant_q5k_f32(blocks, 2048))
