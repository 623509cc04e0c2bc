"""The GEMM kernels' fp16 weight operand, read back bit-exactly on B200.

With one-hot activations (row m of A is the unit vector e_k) the product is
C[m, n] = W'[n, k] exactly: every other term is 0 * w = 0 and the fp32 sum of
one fp16 value rounds back to itself. So the fp16 operand the kernel built
in tensor memory comes back through the public GEMM entry points, and is
compared bit for bit (zeros of either sign equal) with:

* Q4_0 (split planes and llama.cpp blocks): the reference's dequant
  fp16_rn((q - 8) d) (kernels/busfill_v0.cu:74-81), i.e. the oracle;
* Q4_K and Q5_K: the documented chain hfma2(q, ds, -dm) with
  ds = fp16_rn(fp32(d) sc), dm = fp16_rn(fp32(dmin) m): one fused fp16
  rounding of q ds - dm, modelled below in float64;
* Q6_K: hmul2(q - 32, ds) with ds = fp16_rn(fp32(d) sc).

For the K formats the same tests also count how often the chain differs
from the oracle's single rounding fp16_rn(w32), and bound by how much.
Both kernels (decode, and prefill forced onto the small batch) are checked.
"""
import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402

DEV = "cuda:0"
N, K = 384, 512


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def canon(w16):
    """fp16 bits with -0 mapped to +0."""
    b = np.asarray(w16, dtype=np.float16).view(np.uint16).copy()
    b[b == 0x8000] = 0
    return b


def operand_via_onehot(gemm, n, k, prefill):
    """[n, k] fp16 operand: 32 one-hot activation rows per call."""
    out = np.empty((n, k), dtype=np.float16)
    bf.set_prefill_min_m(1 if prefill else 10 ** 6)
    try:
        for g in range(0, k, 32):
            m = min(32, k - g)
            a = np.zeros((m, k), dtype=np.float16)
            a[np.arange(m), g + np.arange(m)] = 1.0
            c = gemm(cu(a))
            assert bf.stream_status() == 0
            out[:, g:g + m] = c.cpu().numpy().T
    finally:
        bf.set_prefill_min_m(0)
    return out


def rn16(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16)


def k_chain(d16, dmin16, sc, m, q):
    """hfma2(q, fp16_rn(fp32(d) sc), -fp16_rn(fp32(dmin) m)), one rounding."""
    n, s = d16.shape
    ds = (d16.astype(np.float32)[:, :, None] * sc.astype(np.float32)).astype(np.float16)
    ndm = (-(dmin16.astype(np.float32)[:, :, None] * m.astype(np.float32))).astype(np.float16)
    qf = q.reshape(n, s, 8, 32).astype(np.float64)
    w = rn16(qf * ds.astype(np.float64)[..., None] + ndm.astype(np.float64)[..., None])
    return w.reshape(n, s * 256)


def q6k_chain(blocks, k):
    d16, sc, q = orc.split_q6k_blocks(blocks, k)
    n, s = d16.shape
    ds = (d16.astype(np.float32)[:, :, None] * sc.astype(np.float32)).astype(np.float16)
    qm = (q.astype(np.int32) - 32).reshape(n, s, 16, 16).astype(np.float64)
    return rn16(qm * ds.astype(np.float64)[..., None]).reshape(n, k)


def check_chain_vs_oracle(chain, w32, max_frac):
    """The chain's fp16 operand against the oracle's fp16_rn(w32) (two
    roundings against one): the share of weights whose fp16 differs (about
    29 % for Q4_K / Q5_K, 20 % for Q6_K on these generators) and the relative
    L2 error against the exact weights (about 3e-4; the absolute per-weight
    bound of the chain is checked on the CPU in test_abi_cpu)."""
    want = w32.astype(np.float16)
    diff = canon(chain) != canon(want)
    assert diff.mean() <= max_frac, diff.mean()
    w = w32.astype(np.float64)
    rel = np.linalg.norm(chain.astype(np.float64) - w) / np.linalg.norm(w)
    assert rel <= 5e-4, rel
    return float(diff.mean())


@pytest.mark.parametrize("prefill", [False, True])
def test_q4_0_operand_is_reference_dequant(prefill):
    wq, ws = orc.gen_q4_0(N, K, seed=31)
    got = operand_via_onehot(lambda a: bf.gemm_q4_0(cu(wq), cu(ws), a), N, K, prefill)
    assert np.array_equal(canon(got), canon(orc.dequant_q4_0_planes(wq, ws)))
    blocks = orc.q4_0_planes_to_ggml_blocks(wq, ws)
    got_g = operand_via_onehot(lambda a: bf.gemm_q4_0_ggml(cu(blocks), a), N, K, prefill)
    assert np.array_equal(canon(got_g), canon(orc.dequant_q4_0_ggml(blocks, K)))


@pytest.mark.parametrize("prefill", [False, True])
def test_q4k_operand_is_the_documented_chain(prefill):
    blocks = orc.gen_q4k(N, K, seed=32)
    got = operand_via_onehot(lambda a: bf.gemm_q4k(cu(blocks), a), N, K, prefill)
    chain = k_chain(*orc.split_q4k_blocks(blocks, K))
    assert np.array_equal(canon(got), canon(chain))
    check_chain_vs_oracle(chain, orc.dequant_q4k_f32(blocks, K), max_frac=0.35)


@pytest.mark.parametrize("prefill", [False, True])
def test_q5k_operand_is_the_documented_chain(prefill):
    blocks = orc.gen_q5k(N, K, seed=33)
    got = operand_via_onehot(lambda a: bf.gemm_q5k(cu(blocks), a), N, K, prefill)
    chain = k_chain(*orc.split_q5k_blocks(blocks, K))
    assert np.array_equal(canon(got), canon(chain))
    check_chain_vs_oracle(chain, orc.dequant_q5k_f32(blocks, K), max_frac=0.35)


@pytest.mark.parametrize("prefill", [False, True])
def test_q6k_operand_is_the_documented_chain(prefill):
    blocks = orc.gen_q6k(N, K, seed=34)
    body, dplane = bf.repack_q6k(cu(blocks), K)
    got = operand_via_onehot(lambda a: bf.gemm_q6k(body, dplane, a), N, K, prefill)
    chain = q6k_chain(blocks, K)
    assert np.array_equal(canon(got), canon(chain))
    check_chain_vs_oracle(chain, orc.dequant_q6k_f32(blocks, K), max_frac=0.25)


@pytest.fixture
def exact_kquant():
    bf.set_exact_kquant(True)
    try:
        yield
    finally:
        bf.set_exact_kquant(False)


@pytest.mark.parametrize("prefill", [False, True])
def test_exact_option_operand_is_the_oracle(exact_kquant, prefill):
    """BUSFILL_OPT_EXACT_KQUANT: the Q4_K / Q5_K operand is the oracle's
    fp16_rn(w32) bit for bit (the bits of busfill_dequant_q4k / _q5k)."""
    b4 = orc.gen_q4k(N, K, seed=35)
    got4 = operand_via_onehot(lambda a: bf.gemm_q4k(cu(b4), a), N, K, prefill)
    assert np.array_equal(canon(got4), canon(orc.dequant_q4k(b4, K)))
    b5 = orc.gen_q5k(N, K, seed=36)
    got5 = operand_via_onehot(lambda a: bf.gemm_q5k(cu(b5), a), N, K, prefill)
    assert np.array_equal(canon(got5), canon(orc.dequant_q5k(b5, K)))


@pytest.mark.parametrize("name", ["q4k_gguf.npz", "q5k_gguf.npz"])
def test_exact_option_operand_on_golden_blocks(exact_kquant, golden_dir, name):
    """Every byte random (all 6-bit scale / min patterns, fp16 exponents over
    a wide range, negative dmin): still the gguf-py 0.19.0 fp16 bits."""
    import os
    g = np.load(os.path.join(golden_dir, name))
    blocks, w32, k = g["b_blocks"], g["b_w32"], int(g["b_k"])
    gemm = bf.gemm_q4k if name.startswith("q4k") else bf.gemm_q5k
    got = operand_via_onehot(lambda a: gemm(cu(blocks), a), blocks.shape[0], k, False)
    assert np.array_equal(canon(got), canon(w32.astype(np.float16)))


def test_exact_option_gemm_is_fp32_accumulation_of_oracle_weights(exact_kquant):
    """With the exact operand the only differences from an fp32 matmul of the
    oracle's fp16 weights are the accumulation order and the output rounding."""
    m, n, k = 32, 1280, 5120
    blocks = orc.gen_q4k(n, k, seed=37)
    a = orc.gen_activations(m, k, seed=38)
    c = bf.gemm_q4k(cu(blocks), cu(a)).float().cpu().numpy()
    assert bf.stream_status() == 0
    ref = a.astype(np.float64) @ orc.dequant_q4k(blocks, k).astype(np.float64).T
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(c - ref) <= ulp + 1e-3)
