"""The GEMM kernels' fp16 weight operand, read back bit-exactly on B200.

With one-hot activations (row m of A is the unit vector e_k) the product is
C[m, n] = W'[n, k] exactly: every other term is 0 * w = 0 and the fp32 sum of
one fp16 value rounds back to itself. So the fp16 operand the kernel built
in tensor memory comes back through the public GEMM entry points, and is
compared bit for bit (zeros of either sign equal) with the CPU dequant:

* Q4_0 (split planes and llama.cpp blocks): the reference's dequant
  fp16_rn((q - 8) d) (kernels/busfill_v0.cu:74-81), i.e. the oracle;
* Q4_K and Q5_K: fp16_rn(w32), w32 = fp32(d sc) q - fp32(dmin m), the
  llama.cpp / gguf-py order the oracle follows;
* Q6_K: fp16_rn(fp32(d sc) (q - 32)).

Every Q4_K entry point is covered (plain, no-allocation, gathered in a group
of one, the fused SwiGLU pair), on the decode kernel and on the prefill
kernel forced onto the small batch, and every K format on the golden blocks
whose bytes are all random (all scale / min patterns, wide fp16 exponents).
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402
from busfill_b200 import tp  # noqa: E402

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
    """[n, k] fp16 operand: 32 one-hot activation rows per call; prefill: 0 =
    the decode kernel, else the prefill kernel with that batch tile on one
    CTA, or "pair": on CTA pairs."""
    out = np.empty((n, k), dtype=np.float16)
    bf.set_prefill_min_m(1 if prefill else 10 ** 6)
    bf.set_prefill_pair(1 if prefill == "pair" else 2)
    bf.set_prefill_batch_tile(prefill if prefill in (128, 256) else 0)
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
        bf.set_prefill_batch_tile(0)
        bf.set_prefill_pair(0)
    return out


def assert_bits_equal(got, want):
    diff = canon(got) != canon(want)
    assert not diff.any(), f"{int(diff.sum())} of {diff.size} operand values differ from the oracle"


@pytest.mark.parametrize("prefill", [0, 128, 256, "pair"], ids=["decode", "prefill128", "prefill256", "pair"])
def test_q4_0_operand_is_reference_dequant(prefill):
    wq, ws = orc.gen_q4_0(N, K, seed=31)
    got = operand_via_onehot(lambda a: bf.gemm_q4_0(cu(wq), cu(ws), a), N, K, prefill)
    assert_bits_equal(got, orc.dequant_q4_0_planes(wq, ws))
    blocks = orc.q4_0_planes_to_ggml_blocks(wq, ws)
    got_g = operand_via_onehot(lambda a: bf.gemm_q4_0_ggml(cu(blocks), a), N, K, prefill)
    assert_bits_equal(got_g, orc.dequant_q4_0_ggml(blocks, K))


def gather_one_rank(blocks, n, k):
    """busfill_gemm_q4k_gather in a group of one (every peer store and tile
    counter is this GPU's own), called through the C ABI."""
    flags = torch.zeros(8, dtype=torch.int32, device=DEV)

    def gemm(a):
        out = torch.empty((a.shape[0], n), dtype=torch.float16, device=DEV)
        g = tp.Gather()
        g.npeers, g.col_off, g.ldc = 1, 0, n
        g.out[0] = out.data_ptr()
        g.flag[0] = flags.data_ptr()
        st = bf.load_library().busfill_gemm_q4k_gather(
            ctypes.c_void_p(blocks.data_ptr()), ctypes.c_void_p(a.data_ptr()), a.shape[0], n, k, ctypes.byref(g),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == 0
        return out
    return gemm


@pytest.mark.parametrize("prefill", [0, 128, 256, "pair"], ids=["decode", "prefill128", "prefill256", "pair"])
@pytest.mark.parametrize("entry", ["gemm", "noalloc", "gather"])
def test_q4k_operand_is_the_oracle(prefill, entry):
    if entry == "gather" and prefill:
        pytest.skip("the gathered GEMM always runs the decode kernel")
    blocks = orc.gen_q4k(N, K, seed=32)
    wb = cu(blocks)
    if entry == "gemm":
        gemm = lambda a: bf.gemm_q4k(wb, a)                                            # noqa: E731
    elif entry == "noalloc":
        gemm = lambda a: bf.gemm_q4k_noalloc(                                          # noqa: E731
            wb, a, torch.empty((a.shape[0], N), dtype=torch.float16, device=DEV))
    else:
        gemm = gather_one_rank(wb, N, K)
    got = operand_via_onehot(gemm, N, K, prefill)
    assert_bits_equal(got, orc.dequant_q4k(blocks, K))


def constant_q4k(n, k, value_q=8, sc=8):
    """block_q4_K rows whose every weight is d*sc*q = 1.0 * sc * q exactly."""
    s = k // 256
    d16 = np.ones((n, s), dtype=np.float16)
    dmin16 = np.zeros((n, s), dtype=np.float16)
    scs = np.full((n, s, 8), sc, dtype=np.uint8)
    ms = np.zeros((n, s, 8), dtype=np.uint8)
    q = np.full((n, s * 256), value_q, dtype=np.uint8)
    return orc.make_q4k_blocks(d16, dmin16, scs, ms, q)


@pytest.mark.parametrize("prefill", [0, 128, 256, "pair"], ids=["decode", "prefill128", "prefill256", "pair"])
def test_swiglu_up_operand_is_the_oracle(prefill):
    """Gate weights all 64.0: silu(64) is 64 exactly in fp32 (exp(-64) is
    below half an ulp of 1), so with one-hot rows h = fp16(64 * W_up'[n, k])
    = 64 * W_up'[n, k] exactly and the up operand comes back bit for bit."""
    gate = cu(constant_q4k(N, K))
    assert np.all(orc.dequant_q4k_f32(constant_q4k(4, K), K) == 64.0)
    up_np = orc.gen_q4k(N, K, seed=41)
    up = cu(up_np)
    got = operand_via_onehot(lambda a: bf.gemm_q4k_swiglu(gate, up, a), N, K, prefill)
    got = (got.astype(np.float32) / 64.0).astype(np.float16)
    assert_bits_equal(got, orc.dequant_q4k(up_np, K))


def test_swiglu_gate_operand_through_silu():
    """Up weights all 1.0 (sc = 1, q = 1): h = fp16(silu(W_gate'[n, k])). silu
    runs on the device through an exp approximation, so the output is
    compared with fp16(silu) of the oracle's operand in float64: they may
    differ only where that approximation moves a value across an fp16
    rounding boundary (rare), whereas an operand one fp16 ulp off in a
    quarter of the weights would move a large share of the outputs."""
    gate_np = orc.gen_q4k(N, K, seed=42)
    gate = cu(gate_np)
    up = cu(constant_q4k(N, K, value_q=1, sc=1))
    got = operand_via_onehot(lambda a: bf.gemm_q4k_swiglu(gate, up, a), N, K, False)
    g = orc.dequant_q4k(gate_np, K).astype(np.float64)
    want = (g / (1.0 + np.exp(-g))).astype(np.float16)
    diff = canon(got) != canon(want)
    assert diff.mean() <= 0.005, diff.mean()
    assert np.all(np.abs(got.astype(np.float64) - want.astype(np.float64)) <=
                  np.spacing(np.abs(want)).astype(np.float64) + 1e-12)


@pytest.mark.parametrize("prefill", [0, 128, 256, "pair"], ids=["decode", "prefill128", "prefill256", "pair"])
def test_q5k_operand_is_the_oracle(prefill):
    blocks = orc.gen_q5k(N, K, seed=33)
    got = operand_via_onehot(lambda a: bf.gemm_q5k(cu(blocks), a), N, K, prefill)
    assert_bits_equal(got, orc.dequant_q5k(blocks, K))


@pytest.mark.parametrize("prefill", [0, 128, 256, "pair"], ids=["decode", "prefill128", "prefill256", "pair"])
def test_q6k_operand_is_the_oracle(prefill):
    blocks = orc.gen_q6k(N, K, seed=34)
    body, dplane = bf.repack_q6k(cu(blocks), K)
    got = operand_via_onehot(lambda a: bf.gemm_q6k(body, dplane, a), N, K, prefill)
    assert_bits_equal(got, orc.dequant_q6k(blocks, K))


@pytest.mark.parametrize("prefill", [0, 128, 256, "pair"], ids=["decode", "prefill128", "prefill256", "pair"])
@pytest.mark.parametrize("name", ["q4k_gguf.npz", "q5k_gguf.npz", "q6k_gguf.npz"])
def test_operand_on_golden_blocks(golden_dir, name, prefill):
    """Every byte random (all 6-bit scale / min patterns, fp16 exponents over
    a wide range, negative dmin, negative Q6_K scales): still the gguf-py
    0.19.0 fp16 bits."""
    g = np.load(os.path.join(golden_dir, name))
    blocks, w32, k = g["b_blocks"], g["b_w32"], int(g["b_k"])
    n = blocks.shape[0]
    if name.startswith("q6k"):
        body, dplane = bf.repack_q6k(cu(blocks), k)
        gemm = lambda a: bf.gemm_q6k(body, dplane, a)                                  # noqa: E731
    else:
        fn = bf.gemm_q4k if name.startswith("q4k") else bf.gemm_q5k
        wb = cu(blocks)
        gemm = lambda a: fn(wb, a)                                                     # noqa: E731
    got = operand_via_onehot(gemm, n, k, prefill)
    assert_bits_equal(got, w32.astype(np.float16))


def test_gemm_is_fp32_accumulation_of_oracle_weights():
    """With the exact operand the only differences from a float64 matmul of
    the oracle's fp16 weights are the fp32 accumulation order and the output
    rounding (within one fp16 ulp plus 1e-3 at config-2 scale)."""
    m, n, k = 32, 1280, 5120
    blocks = orc.gen_q4k(n, k, seed=37)
    a = orc.gen_activations(m, k, seed=38)
    c = bf.gemm_q4k(cu(blocks), cu(a)).float().cpu().numpy()
    assert bf.stream_status() == 0
    ref = a.astype(np.float64) @ orc.dequant_q4k(blocks, k).astype(np.float64).T
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(c - ref) <= ulp + 1e-3)


def test_exact_option_is_accepted_and_changes_nothing():
    """BUSFILL_OPT_EXACT_KQUANT is kept for callers that set it: every K-quant
    operand is already the oracle's, so both values give the same bits."""
    blocks = cu(orc.gen_q4k(256, 1024, seed=39))
    a = cu(orc.gen_activations(8, 1024, seed=40))
    c0 = bf.gemm_q4k(blocks, a)
    bf.set_exact_kquant(True)
    try:
        c1 = bf.gemm_q4k(blocks, a)
    finally:
        bf.set_exact_kquant(False)
    assert bf.stream_status() == 0
    assert torch.equal(c0, c1)
