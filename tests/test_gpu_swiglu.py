"""GPU parity of the fused SwiGLU pair busfill_gemm_q4k_swiglu, through the C ABI:
h = silu(A deq(Wg)^T) * (A deq(Wu)^T), fp32 products, one fp16 rounding (two
on the CTA-pair path of M >= 256, where the up projection is rounded to fp16
before the product).

Checked against the oracle's float64 SwiGLU on the fp32-dequantized weights:
rel-L2 <= 1e-3 and max abs err <= 2e-3 of the largest |h| (the kernel's fp16
weight operands carry two roundings, ~3e-4 relative, and h is rounded once to
fp16). The activations are scaled by 1/64 so that h stays well inside fp16
with BASELINE's (unnormalised) synthetic weight distribution.
"""
import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402

DEV = "cuda:0"


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def run_and_check(m, n, k, seed):
    wg = orc.gen_q4k(n, k, seed=seed)
    wu = orc.gen_q4k(n, k, seed=seed + 1)
    a = (orc.gen_activations(m, k, seed=seed + 2).astype(np.float32) / 64).astype(np.float16)
    h = bf.gemm_q4k_swiglu(cu(wg), cu(wu), cu(a))
    assert bf.stream_status() == 0
    want = orc.swiglu_ref(a, orc.dequant_q4k_f32(wg, k), orc.dequant_q4k_f32(wu, k))
    got = h.float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 1e-3, rel
    assert np.max(np.abs(got - want)) <= 2e-3 * np.max(np.abs(want)), np.max(np.abs(got - want))
    return h, wg, wu, a


@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (8, 640, 1024), (17, 200, 2048), (32, 1280, 5120), (33, 384, 768)])
def test_swiglu_decode(m, n, k):
    run_and_check(m, n, k, seed=m + n + k)


@pytest.mark.parametrize("csize", [1, 3, 8])
def test_swiglu_decode_forced_ksplit(csize):
    """Several tile pairs per cluster (the reduction buffer reused between the
    gate and up segments and across pairs)."""
    bf.set_ksplit(csize)
    try:
        run_and_check(5, 7680, 2048, seed=csize)
    finally:
        bf.set_ksplit(0)


@pytest.mark.parametrize("pair", [0, 1, 2], ids=["auto", "pairs", "fused"])
@pytest.mark.parametrize("m,n,k", [(64, 512, 1024), (300, 640, 2048), (129, 200, 512), (520, 1000, 1536)])
def test_swiglu_prefill_forced(m, n, k, pair):
    """The prefill kernels: one fused launch of whole (gate, up) tile pairs,
    or (BUSFILL_OPT_PREFILL_PAIR, by default from M = 256) two CTA-pair GEMMs,
    the up projection into h and then the gate with h = silu(gate) * h."""
    bf.set_prefill_min_m(1)
    bf.set_prefill_pair(pair)
    try:
        run_and_check(m, n, k, seed=m * 3 + k)
    finally:
        bf.set_prefill_min_m(0)
        bf.set_prefill_pair(0)


@pytest.mark.parametrize("m", [48, 100, 200])
def test_swiglu_default_dispatch_mid_batch(m):
    """Default dispatch between the decode launches (M <= 32), one fused
    prefill launch (32 < M <= 128) and two CTA-pair GEMMs (M > 128)."""
    run_and_check(m, 8192, 512, seed=m + 11)


def test_swiglu_config3_shape():
    """The 27B layer set's gate/up pair (N = 17408, K = 5120) at M = 32."""
    run_and_check(32, 17408, 5120, seed=7)


def test_swiglu_equals_unfused_products():
    """Same bits as silu(fp32 gate) * fp32 up computed from the two plain
    GEMMs' fp32 outputs (busfill_q4 surface is Q4_0-only, so compare with a
    tolerance against the fp16 outputs of the plain Q4_K GEMMs instead)."""
    m, n, k = 16, 512, 2048
    h, wg, wu, a = run_and_check(m, n, k, seed=99)
    g = bf.gemm_q4k(cu(wg), cu(a)).float()
    u = bf.gemm_q4k(cu(wu), cu(a)).float()
    ref = torch.nn.functional.silu(g) * u
    assert torch.allclose(h.float(), ref, rtol=2e-3, atol=2e-3 * ref.abs().max().item())
