"""GPU parity of the Q6_K path (busfill_repack_q6k, busfill_dequant_q6k,
busfill_gemm_q6k) through the C ABI, against the oracle (gguf-py 0.19.0 Q6_K
semantics, pinned by tests/golden/q6k_gguf.npz).

Repack: bit-exact against the oracle's restatement. Dequant: bit-exact
fp16_rn(w32). GEMM: rel-L2 <= 1e-3 against an fp32 matmul of the dequantized
weights (the reference gate), every element within 0.6 plus one fp16 ulp of
the output, and rel-L2 <= 7e-4 against float64 (the fp16 operand carries two
roundings, of d*sc and of the product, each up to 2^-11 relative).
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


def device_layout(blocks, k):
    body, d = bf.repack_q6k(cu(blocks), k)
    assert bf.stream_status() == 0
    return body, d


def test_repack_q6k_matches_oracle(golden_dir):
    g = np.load(os.path.join(golden_dir, "q6k_gguf.npz"))
    cases = [(g["a_blocks"], int(g["a_k"])), (g["b_blocks"], int(g["b_k"])), (orc.gen_q6k(1000, 5120, seed=4), 5120)]
    for blocks, k in cases:
        body, d = device_layout(blocks, k)
        want_body, want_d = orc.repack_q6k(blocks, k)
        assert np.array_equal(body.cpu().numpy(), want_body)
        assert np.array_equal(d.cpu().numpy().view(np.uint16), want_d.view(np.uint16))


def test_dequant_q6k_bit_exact_gguf_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "q6k_gguf.npz"))
    for case in ("a", "b"):
        blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
        body, d = device_layout(blocks, k)
        out = bf.dequant_q6k(body, d, k)
        assert bf.stream_status() == 0
        with np.errstate(over="ignore"):
            want = w32.astype(np.float16)
        assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16)), case


def test_dequant_q6k_bit_exact_generator_distribution():
    blocks = orc.gen_q6k(640, 5120, seed=5)
    body, d = device_layout(blocks, 5120)
    out = bf.dequant_q6k(body, d, 5120)
    assert bf.stream_status() == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), orc.dequant_q6k(blocks, 5120).view(np.uint16))


def check(c, a, w32):
    got = c.float().cpu().numpy()
    ref = orc.gemm_ref(a, w32)
    max_abs, rel, finite = orc.gemm_errors(got, ref)
    assert finite and rel <= orc.GATE_REL_L2, (max_abs, rel)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= orc.GATE_MAX_ABS + 2.0 ** -10 * np.abs(ref)), max_abs
    exact = a.astype(np.float64) @ w32.astype(np.float64).T
    _, rel_t, _ = orc.gemm_errors(got, exact)
    assert rel_t <= 7e-4, rel_t


@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (8, 640, 1024), (17, 200, 2048), (32, 1280, 5120), (33, 384, 768),
                                   (5, 3840, 5120), (2, 512, 16384), (48, 1024, 512), (64, 2048, 1024)])
def test_gemm_q6k_decode(m, n, k):
    blocks = orc.gen_q6k(n, k, seed=m + n + k)
    a = orc.gen_activations(m, k, seed=m * 3 + k)
    body, d = device_layout(blocks, k)
    c = bf.gemm_q6k(body, d, cu(a))
    assert bf.stream_status() == 0
    check(c, a, orc.dequant_q6k_f32(blocks, k))


@pytest.mark.parametrize("bt", [128, 256, "pair"])
@pytest.mark.parametrize("m,n,k", [(128, 512, 512), (300, 640, 2048), (64, 200, 1024)])
def test_gemm_q6k_prefill(m, n, k, bt):
    bf.set_prefill_min_m(1)
    if bt == "pair":
        bf.set_prefill_pair(1)
    else:
        bf.set_prefill_pair(2)
        bf.set_prefill_batch_tile(bt)
    try:
        blocks = orc.gen_q6k(n, k, seed=m + 2 * n + k)
        a = orc.gen_activations(m, k, seed=m + k)
        body, d = device_layout(blocks, k)
        c = bf.gemm_q6k(body, d, cu(a))
        assert bf.stream_status() == 0
    finally:
        bf.set_prefill_min_m(0)
        bf.set_prefill_batch_tile(0)
        bf.set_prefill_pair(0)
    check(c, a, orc.dequant_q6k_f32(blocks, k))


@pytest.mark.parametrize("csize", [1, 3, 8])
def test_gemm_q6k_forced_ksplit(csize):
    bf.set_ksplit(csize)
    try:
        blocks = orc.gen_q6k(3072, 2048, seed=csize)
        a = orc.gen_activations(5, 2048, seed=csize + 1)
        body, d = device_layout(blocks, 2048)
        c = bf.gemm_q6k(body, d, cu(a))
        assert bf.stream_status() == 0
    finally:
        bf.set_ksplit(0)
    check(c, a, orc.dequant_q6k_f32(blocks, 2048))
