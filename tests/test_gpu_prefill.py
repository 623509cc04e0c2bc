"""GPU parity of the large-batch (prefill) kernel, through the C ABI.

Large batches (by default M > 64 for the plain GEMMs, whose prefill kernel
spreads the work over all SMs stream-K style; M >= 128 with at least 64 work
items of 256 weight rows x 128 batch rows where whole items are dealt out)
run one pass over the weights for all rows; the decode kernel covers the rest. These tests force the prefill kernel
(BUSFILL_OPT_PREFILL_MIN_M) onto small, ragged and multi-item shapes, with
every work-item shape (BUSFILL_OPT_PREFILL_BATCH_TILE 128 and 256 on one
CTA, BUSFILL_OPT_PREFILL_PAIR on CTA pairs), and run
the BASELINE config-4 shapes at full size through the default dispatch,
checked on sampled rows and columns against the oracle.
Gates as in test_gpu_parity: max abs err <= 0.6 and rel-L2 <= 1e-3 against
an fp32 matmul of the dequantized weights, plus a tighter fp64 check.
"""
import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402

DEV = "cuda:0"
TIGHT_REL_L2 = 5e-4


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def check(c_dev, a, w_ref, w_exact):
    c = c_dev.float().cpu().numpy()
    cref = orc.gemm_ref(a, w_ref)
    max_abs, rel, finite = orc.gemm_errors(c, cref)
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2, (max_abs, rel)
    exact = a.astype(np.float64) @ w_exact.astype(np.float64).T
    _, rel_t, _ = orc.gemm_errors(c, exact)
    assert rel_t <= TIGHT_REL_L2, rel_t


@pytest.fixture(params=[128, 256, "pair"], ids=["bt128", "bt256", "pair"])
def prefill_always(request):
    """The prefill kernel for every M: one CTA per work item of 128 batch rows
    (two weight tiles) or 256 (one weight tile, MMA N = 256), or CTA pairs
    (256 x 256 items, one cta_group::2 MMA over two SMs)."""
    bf.set_prefill_min_m(1)
    if request.param == "pair":
        bf.set_prefill_pair(1)
    else:
        bf.set_prefill_pair(2)
        bf.set_prefill_batch_tile(request.param)
    try:
        yield request.param
    finally:
        bf.set_prefill_min_m(0)
        bf.set_prefill_batch_tile(0)
        bf.set_prefill_pair(0)


PREFILL_SHAPES = [
    (128, 512, 512), (130, 384, 768), (256, 1280, 1024), (300, 640, 2048), (257, 200, 256), (512, 2304, 1536),
    (260, 100, 512),   # N % 8 != 0: the epilogue's scalar stores
]


@pytest.mark.parametrize("m,n,k", PREFILL_SHAPES)
def test_prefill_q4k(prefill_always, m, n, k):
    blocks = orc.gen_q4k(n, k, seed=m + 3 * n + k)
    a = orc.gen_activations(m, k, seed=m * 7 + k)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    assert bf.stream_status() == 0
    w32 = orc.dequant_q4k_f32(blocks, k)
    check(c, a, w32, w32)


@pytest.mark.parametrize("m,n,k", PREFILL_SHAPES)
def test_prefill_q4_0_planes_and_ggml(prefill_always, m, n, k):
    """Both Q4_0 layouts give the same fp16 operands, so the same bits."""
    wq, ws = orc.gen_q4_0(n, k, seed=m + 5 * n + k)
    blocks = orc.q4_0_planes_to_ggml_blocks(wq, ws)
    a = orc.gen_activations(m, k, seed=m * 11 + k)
    c = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
    cg = bf.gemm_q4_0_ggml(cu(blocks), cu(a))
    assert bf.stream_status() == 0
    assert torch.equal(c.view(torch.int16), cg.view(torch.int16))
    check(c, a, orc.dequant_q4_0_planes_f32(wq, ws), orc.dequant_q4_0_planes(wq, ws))


@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (17, 200, 512), (33, 1024, 2048), (64, 256, 5120)])
def test_prefill_forced_on_small_batches(prefill_always, m, n, k):
    blocks = orc.gen_q4k(n, k, seed=m + n)
    wq, ws = orc.gen_q4_0(n, k, seed=m + 2 * n)
    a = orc.gen_activations(m, k, seed=m + k)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    c0 = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
    assert bf.stream_status() == 0
    w32 = orc.dequant_q4k_f32(blocks, k)
    check(c, a, w32, w32)
    check(c0, a, orc.dequant_q4_0_planes_f32(wq, ws), orc.dequant_q4_0_planes(wq, ws))


def test_prefill_matches_decode_kernel(prefill_always):
    """Same GEMM through both kernels: they accumulate in different orders, so
    compare within a few fp16 ulps of the output."""
    m, n, k = 96, 640, 3072
    blocks = orc.gen_q4k(n, k, seed=5)
    a = cu(orc.gen_activations(m, k, seed=6))
    cp = bf.gemm_q4k(cu(blocks), a).float()
    bf.set_prefill_min_m(10 ** 6)
    cd = bf.gemm_q4k(cu(blocks), a).float()
    assert bf.stream_status() == 0
    assert torch.allclose(cp, cd, rtol=2e-3, atol=2e-3)


def test_prefill_fp32_reference_surface(prefill_always):
    """busfill_q4 (fp32 output, the reference's argument order) on the prefill path."""
    m, n, k = 40, 256, 512
    wq, ws = orc.gen_q4_0(n, k, seed=41)
    a = orc.gen_activations(m, k, seed=42)
    c = torch.empty((m, n), dtype=torch.float32, device=DEV)
    bf.busfill_q4(cu(a), cu(wq), cu(ws), c, m, k, n)
    assert bf.stream_status() == 0
    check(c, a, orc.dequant_q4_0_planes_f32(wq, ws), orc.dequant_q4_0_planes(wq, ws))


@pytest.mark.parametrize("m,n,k", [(2048, 5120, 17408), (2048, 17408, 5120), (512, 5120, 17408)])
def test_prefill_config4_sampled(m, n, k):
    """BASELINE config 4 at full size: the whole output is computed, and a
    sample of 64 rows x 512 columns is checked against the oracle."""
    blocks = orc.gen_q4k(n, k, seed=m + n + k)
    a = orc.gen_activations(m, k, seed=m + k)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    assert bf.stream_status() == 0
    rng = np.random.default_rng(m + n)
    rows = np.sort(rng.choice(m, 64, replace=False))
    cols = np.sort(rng.choice(n, 512, replace=False))
    w32 = orc.dequant_q4k_f32(blocks[cols], k)
    check(c[rows][:, cols], a[rows], w32, w32)
    assert torch.isfinite(c.float()).all()


@pytest.mark.parametrize("m,n,k", [(128, 5120, 17408), (128, 17408, 5120), (64, 1024, 17408)])
def test_prefill_stream_k_split_items_sampled(prefill_always, m, n, k):
    """Few work items over many units: with stream-K every item of N = 5120,
    K = 17408 is split between about seven CTAs and summed by the fix-up
    kernel; the output is checked on sampled columns against the oracle."""
    blocks = orc.gen_q4k(n, k, seed=3 * m + n + k)
    a = orc.gen_activations(m, k, seed=m + 2 * k)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    assert bf.stream_status() == 0
    rng = np.random.default_rng(n + k)
    cols = np.sort(rng.choice(n, 512, replace=False))
    w32 = orc.dequant_q4k_f32(blocks[cols], k)
    check(c[:, cols], a, w32, w32)
    assert torch.isfinite(c.float()).all()


def test_prefill_stream_k_is_deterministic(prefill_always):
    """The split points depend only on the shape and the SM count, and split
    items are summed in CTA order: two runs give the same bits."""
    m, n, k = 96, 2048, 17408
    blocks = cu(orc.gen_q4k(n, k, seed=8))
    a = cu(orc.gen_activations(m, k, seed=9))
    c1 = bf.gemm_q4k(blocks, a).clone()
    c2 = bf.gemm_q4k(blocks, a)
    assert bf.stream_status() == 0
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))


def test_prefill_without_workspace_round_robin(prefill_always):
    """The no-allocation entry point has no partial-tile workspace: whole
    items go round-robin over the CTAs (the path without stream-K)."""
    m, n, k = 200, 1280, 2048
    blocks = orc.gen_q4k(n, k, seed=21)
    a = orc.gen_activations(m, k, seed=22)
    out = torch.empty((m, n), dtype=torch.float16, device=DEV)
    bf.gemm_q4k_noalloc(cu(blocks), cu(a), out)
    assert bf.stream_status() == 0
    w32 = orc.dequant_q4k_f32(blocks, k)
    check(out, a, w32, w32)
