"""Pin the CPU oracle against golden vectors (no GPU needed).

* Q4_0 quantizer / dequant / gate product vs the reference's own
  ``quantize_q4q`` (kernels/q4k_batched.py:65-79,100), fixture q4_0_reference.npz.
* Q4_K dequant vs gguf-py 0.19.0 ``Q4_K.dequantize_blocks``, fixture q4k_gguf.npz.
* llama.cpp AoS Q4_0 dequant vs gguf-py ``Q4_0.dequantize_blocks``, q4_0_gguf.npz.
* Q5_K dequant vs gguf-py ``Q5_K.dequantize_blocks``, q5k_gguf.npz.
* Q6_K dequant vs gguf-py ``Q6_K.dequantize_blocks``, q6k_gguf.npz, and the
  device layout of busfill_repack_q6k (208-byte block bodies + a d plane).
* Exhaustive checks of the 6-bit scale/min packing.
"""
import os

import numpy as np
import pytest

from oracle import q4_oracle as orc


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_quantize_q4q_matches_reference(golden_dir, case):
    g = _load(golden_dir, "q4_0_reference.npz")
    wq, ws, ref = orc.quantize_q4q(g[f"{case}_wf"])
    assert np.array_equal(wq, g[f"{case}_wq"])
    assert np.array_equal(ws.view(np.uint16), g[f"{case}_ws"].view(np.uint16))
    assert np.array_equal(ref.view(np.uint32), g[f"{case}_ref"].view(np.uint32))


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_dequant_q4_0_matches_reference(golden_dir, case):
    g = _load(golden_dir, "q4_0_reference.npz")
    wq, ws, ref = g[f"{case}_wq"], g[f"{case}_ws"], g[f"{case}_ref"]
    # fp32 dequant is the reference gate's `ref` exactly
    assert np.array_equal(orc.dequant_q4_0_planes_f32(wq, ws).view(np.uint32), ref.view(np.uint32))
    # fp16 operand = RN16 of that exact product (kernels/busfill_v0.cu:74-81)
    w16 = orc.dequant_q4_0_planes(wq, ws)
    assert np.array_equal(w16.view(np.uint16), ref.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_gemm_ref_matches_reference_gate_product(golden_dir, case):
    g = _load(golden_dir, "q4_0_reference.npz")
    c = orc.gemm_ref(g[f"{case}_a"], orc.dequant_q4_0_planes_f32(g[f"{case}_wq"], g[f"{case}_ws"]))
    # torch and numpy fp32 GEMMs may sum in different orders: tiny tolerance
    np.testing.assert_allclose(c, g[f"{case}_c"], rtol=1e-5, atol=1e-5)


def test_pack_unpack_q4_0_planes_roundtrip():
    rng = np.random.default_rng(0)
    wq = rng.integers(0, 256, size=(7, 48), dtype=np.uint8)
    assert np.array_equal(orc.pack_q4_0_planes(orc.unpack_q4_0_planes(wq)), wq)


@pytest.mark.parametrize("case", ["a", "b"])
def test_dequant_q4k_matches_gguf(golden_dir, case):
    g = _load(golden_dir, "q4k_gguf.npz")
    blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
    mine = orc.dequant_q4k_f32(blocks, k)
    assert np.array_equal(mine.view(np.uint32), w32.view(np.uint32))
    assert np.array_equal(orc.dequant_q4k(blocks, k).view(np.uint16), w32.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("case", ["a", "b"])
def test_q5k_dequant_matches_gguf_golden(golden_dir, case):
    """Q5_K dequant vs gguf-py 0.19.0 ``Q5_K.dequantize_blocks`` (q5k_gguf.npz)."""
    g = _load(golden_dir, "q5k_gguf.npz")
    blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
    assert np.array_equal(orc.dequant_q5k_f32(blocks, k).view(np.uint32), w32.view(np.uint32))
    with np.errstate(over="ignore"):
        want16 = w32.astype(np.float16)
    assert np.array_equal(orc.dequant_q5k(blocks, k).view(np.uint16), want16.view(np.uint16))


def test_q5k_block_split_make_roundtrip(golden_dir):
    g = _load(golden_dir, "q5k_gguf.npz")
    blocks, k = g["b_blocks"], int(g["b_k"])
    assert np.array_equal(orc.make_q5k_blocks(*orc.split_q5k_blocks(blocks, k)), blocks)
    # the generator's values come back out of the blocks
    w = orc.gen_q5k(8, 512, seed=3)
    d, dmin, sc, m, q = orc.split_q5k_blocks(w, 512)
    assert q.max() <= 31 and q.min() >= 0 and sc.max() < 64 and m.max() < 64


@pytest.mark.parametrize("case", ["a", "b"])
def test_q6k_dequant_matches_gguf_golden(golden_dir, case):
    """Q6_K dequant vs gguf-py 0.19.0 ``Q6_K.dequantize_blocks`` (q6k_gguf.npz)."""
    g = _load(golden_dir, "q6k_gguf.npz")
    blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
    assert np.array_equal(orc.dequant_q6k_f32(blocks, k).view(np.uint32), w32.view(np.uint32))
    with np.errstate(over="ignore"):
        want16 = w32.astype(np.float16)
    assert np.array_equal(orc.dequant_q6k(blocks, k).view(np.uint16), want16.view(np.uint16))


def test_q6k_block_split_make_repack_roundtrip(golden_dir):
    g = _load(golden_dir, "q6k_gguf.npz")
    blocks, k = g["b_blocks"], int(g["b_k"])
    assert np.array_equal(orc.make_q6k_blocks(*orc.split_q6k_blocks(blocks, k)), blocks)
    qb, d = orc.repack_q6k(blocks, k)
    n, s = blocks.shape[0], k // 256
    assert qb.shape == (n, s * 208) and d.shape == (s, n) and d.dtype == np.float16
    assert (s * 208) % 16 == 0
    assert np.array_equal(orc.unpack_q6k(qb, d, k), blocks)
    # the generator's values come back out of the blocks
    w = orc.gen_q6k(8, 512, seed=3)
    d16, sc, q = orc.split_q6k_blocks(w, 512)
    assert q.min() >= 0 and q.max() <= 63 and sc.min() >= -128 and sc.max() <= 127


def test_q6k_element_placement():
    """One non-zero 6-bit value at a time lands at its own element index."""
    n, k = 1, 256
    d = np.full((n, 1), 1.0, dtype=np.float16)
    sc = np.arange(1, 17, dtype=np.int8).reshape(n, 1, 16)
    for e in (0, 17, 31, 32, 63, 64, 100, 127, 128, 161, 200, 255):
        q = np.full((n, k), 32, dtype=np.uint8)
        q[0, e] = 32 + 29
        w = orc.dequant_q6k_f32(orc.make_q6k_blocks(d, sc, q), k)
        want = np.zeros((n, k), dtype=np.float32)
        want[0, e] = 29.0 * (e // 16 + 1)
        assert np.array_equal(w, want), e


def test_q4k_block_split_make_roundtrip(golden_dir):
    g = _load(golden_dir, "q4k_gguf.npz")
    blocks, k = g["b_blocks"], int(g["b_k"])
    d, dmin, sc, m, q = orc.split_q4k_blocks(blocks, k)
    assert np.array_equal(orc.make_q4k_blocks(d, dmin, sc, m, q), blocks)


def test_dequant_q4_0_ggml_matches_gguf(golden_dir):
    g = _load(golden_dir, "q4_0_gguf.npz")
    blocks, w32, k = g["blocks"], g["w32"], int(g["k"])
    mine = orc.dequant_q4_0_ggml(blocks, k)
    assert np.array_equal(mine.view(np.uint16), w32.astype(np.float16).view(np.uint16))


def test_q4_0_planes_to_ggml_blocks_consistent():
    wq, ws = orc.gen_q4_0(8, 256, seed=5)
    blocks = orc.q4_0_planes_to_ggml_blocks(wq, ws)
    assert blocks.shape == (8, 256 // 32 * 18)
    assert np.array_equal(orc.dequant_q4_0_ggml(blocks, 256).view(np.uint16),
                          orc.dequant_q4_0_planes(wq, ws).view(np.uint16))


def _get_scale_min_k4_scalar(j, q):
    """Scalar restatement of the 6-bit unpack for sub-block j (llama.cpp
    get_scale_min_k4 as published in gguf-py 0.19.0 Q4_K.get_scale_min)."""
    if j < 4:
        return q[j] & 63, q[j + 4] & 63
    return (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4), (q[j + 4] >> 4) | ((q[j - 0] >> 6) << 4)


@pytest.mark.parametrize("j", range(8))
def test_unpack_q4k_scales_exhaustive_per_subblock(j):
    # Every (sc_j, m_j) depends on at most two bytes for sc and two for m; walk
    # all 65536 values of each byte pair while the other bytes hold random data.
    rng = np.random.default_rng(j)
    base = rng.integers(0, 256, size=12, dtype=np.uint8)
    if j < 4:
        pairs = [(j, j + 4)]
    else:
        pairs = [(j + 4, j - 4), (j + 4, j)]
    for b0, b1 in pairs:
        s = np.tile(base, (65536, 1))
        grid = np.arange(65536)
        s[:, b0] = grid & 0xFF
        s[:, b1] = grid >> 8
        sc, m = orc.unpack_q4k_scales(s)
        want_sc = np.array([_get_scale_min_k4_scalar(j, row)[0] for row in s[::257]], dtype=np.uint8)
        want_m = np.array([_get_scale_min_k4_scalar(j, row)[1] for row in s[::257]], dtype=np.uint8)
        assert np.array_equal(sc[::257, j], want_sc)
        assert np.array_equal(m[::257, j], want_m)
        # vectorised scalar restatement over the full grid
        full_sc = np.where(j < 4, s[:, j % 12] & 63, 0)
        if j >= 4:
            full_sc = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
            full_m = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        else:
            full_m = s[:, j + 4] & 63
        assert np.array_equal(sc[:, j], full_sc)
        assert np.array_equal(m[:, j], full_m)


def test_pack_unpack_q4k_scales_roundtrip_all_values():
    # all 64 values in every one of the 16 (sc, m) slots
    v = np.arange(64, dtype=np.uint8)
    for slot in range(8):
        sc = np.zeros((64, 8), dtype=np.uint8)
        m = np.zeros((64, 8), dtype=np.uint8)
        sc[:, slot] = v
        m[:, slot] = v[::-1]
        s2, m2 = orc.unpack_q4k_scales(orc.pack_q4k_scales(sc, m))
        assert np.array_equal(s2, sc) and np.array_equal(m2, m)


def test_generators_follow_config_distributions():
    wq, ws = orc.gen_q4_0(64, 512, seed=1)
    assert wq.shape == (64, 256) and ws.shape == (64, 16) and ws.dtype == np.float16
    assert float(ws.min()) >= 0.000999 and float(ws.max()) <= 0.0201
    blocks = orc.gen_q4k(32, 512, seed=2)
    assert blocks.shape == (32, 2 * 144)
    d, dmin, sc, m, q = orc.split_q4k_blocks(blocks, 512)
    assert float(d.min()) >= 0.000999 and float(d.max()) <= 0.01001
    assert float(dmin.min()) >= 0.0 and float(dmin.max()) <= 0.005
    assert sc.max() <= 63 and m.max() <= 63 and q.max() <= 15
    a = orc.gen_activations(8, 512, seed=3)
    assert a.dtype == np.float16 and abs(float(a.astype(np.float32).std()) - 1.0) < 0.1


def test_gate_rejects_nan_and_large_error():
    cref = np.ones((2, 4), dtype=np.float32)
    assert orc.gate_ok(cref.copy(), cref)
    bad = cref.copy()
    bad[0, 0] = np.nan
    assert not orc.gate_ok(bad, cref)
    far = cref.copy()
    far[1, 1] += 0.7
    assert not orc.gate_ok(far, cref)


def test_algorithmic_bytes_match_hand_computed_figures():
    # 4.5-bit weights + fp16 A + fp16 C at K=N=5120
    assert orc.algorithmic_bytes(1, 5120, 5120) == 14_766_080
    assert orc.algorithmic_bytes(8, 5120, 5120) == 14_909_440
    assert orc.algorithmic_bytes(32, 5120, 5120) == 15_400_960
    assert orc.algorithmic_bytes(32, 17408, 5120) == 51_576_832
