"""The planar Q4_K entry points and the ggml mul_mat call site on B200.

* busfill_repack_q4k_planar rebuilds block_q4_K rows byte for byte from the
  planes (qs, d, dmin, scales12);
* busfill_gemm_q4k_planar returns busfill_gemm_q4k's bits on the same weight
  (decode and prefill kernels) and meets the gates against the oracle;
* busfill_mul_mat (ggml_mul_mat semantics: src0 [K, N] blocks, src1 [K, M]
  fp16, dst [N, M]) returns the matching busfill_gemm_* bits per batch slice,
  with src0 broadcast over src1's batch dimension.
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


def planes(blocks, n, k):
    """block_q4_K rows -> (qs [n, k/2], d [n, s], dmin [n, s], scales12 [n, s*12])."""
    s = k // 256
    b = blocks.reshape(n, s, 144)
    qs = np.ascontiguousarray(b[:, :, 16:144]).reshape(n, s * 128)
    d = np.ascontiguousarray(b[:, :, 0:2]).view(np.float16).reshape(n, s)
    dmin = np.ascontiguousarray(b[:, :, 2:4]).view(np.float16).reshape(n, s)
    sc = np.ascontiguousarray(b[:, :, 4:16]).reshape(n, s * 12)
    return qs, d, dmin, sc


@pytest.mark.parametrize("n,k", [(256, 1024), (384, 5120)])
def test_planar_repack_rebuilds_the_blocks(n, k):
    blocks = orc.gen_q4k(n, k, seed=81)
    got = bf.repack_q4k_planar(*[cu(x) for x in planes(blocks, n, k)])
    assert np.array_equal(got.cpu().numpy(), blocks)


@pytest.mark.parametrize("m", [8, 32, 130])
def test_planar_gemm_is_the_block_gemm(m):
    n, k = 640, 2048
    blocks = orc.gen_q4k(n, k, seed=82)
    a = orc.gen_activations(m, k, seed=83)
    got = bf.gemm_q4k_planar(*[cu(x) for x in planes(blocks, n, k)], cu(a))
    want = bf.gemm_q4k(cu(blocks), cu(a))
    assert bf.stream_status() == 0
    assert torch.equal(got, want)
    max_abs, rel, finite = orc.gemm_errors(got.float().cpu().numpy(), orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k)))
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2


def _weights(ggml_type, n, k, seed):
    if ggml_type == bf.TYPE_Q4_K:
        w = orc.gen_q4k(n, k, seed=seed)
        return w, lambda wt, a: bf.gemm_q4k(wt, a), orc.dequant_q4k_f32(w, k)
    if ggml_type == bf.TYPE_Q5_K:
        w = orc.gen_q5k(n, k, seed=seed)
        return w, lambda wt, a: bf.gemm_q5k(wt, a), orc.dequant_q5k_f32(w, k)
    wq, ws = orc.gen_q4_0(n, k, seed=seed)
    w = orc.q4_0_planes_to_ggml_blocks(wq, ws)
    return w, lambda wt, a: bf.gemm_q4_0_ggml(wt, a), orc.dequant_q4_0_ggml(w, k).astype(np.float32)


@pytest.mark.parametrize("ggml_type", [bf.TYPE_Q4_0, bf.TYPE_Q4_K, bf.TYPE_Q5_K])
def test_mul_mat_2d(ggml_type):
    n, k, m = 384, 1536, 24
    w, gemm, wf = _weights(ggml_type, n, k, 84)
    a = orc.gen_activations(m, k, seed=85)
    wt, at = cu(w), cu(a)
    out = torch.empty((m, n), dtype=torch.float16, device=DEV)
    bf.mul_mat(bf.tensor_desc(wt, ggml_type, [k, n]), bf.tensor_desc(at, bf.TYPE_F16, [k, m]),
               bf.tensor_desc(out, bf.TYPE_F16, [n, m]))
    want = gemm(wt, at)
    assert bf.stream_status() == 0
    assert torch.equal(out, want)
    max_abs, rel, finite = orc.gemm_errors(out.float().cpu().numpy(), orc.gemm_ref(a, wf))
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2


def test_mul_mat_broadcasts_the_weight_over_batches():
    n, k, m, nb = 256, 1024, 8, 3
    w, gemm, _ = _weights(bf.TYPE_Q4_K, n, k, 86)
    a = np.stack([orc.gen_activations(m, k, seed=87 + i) for i in range(nb)])
    wt, at = cu(w), cu(a)
    out = torch.empty((nb, m, n), dtype=torch.float16, device=DEV)
    bf.mul_mat(bf.tensor_desc(wt, bf.TYPE_Q4_K, [k, n, 1]), bf.tensor_desc(at, bf.TYPE_F16, [k, m, nb]),
               bf.tensor_desc(out, bf.TYPE_F16, [n, m, nb]))
    assert bf.stream_status() == 0
    for i in range(nb):
        assert torch.equal(out[i], gemm(wt, at[i].contiguous()))
