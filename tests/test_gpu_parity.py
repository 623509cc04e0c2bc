"""GPU parity tests: every call goes through the C ABI (libbusfill.so) on a
B200 and is checked against the CPU oracle (oracle/q4_oracle.py).

Gates (kernels/q4k_batched.py:97-104):
* dequant: bit-exact fp16 against the oracle;
* GEMM: all outputs finite, max abs err <= 0.6 and rel-L2 <= 1e-3 against an
  fp32 matmul of the dequantized weights. We also hold a much tighter
  tolerance against an fp64 product of the exact weights (below), since the
  kernels accumulate exact products in fp32.
"""
import os

import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import busfill_b200 as bf  # noqa: E402

DEV = "cuda:0"
# Beyond the reference gate: the kernel output is one fp16 rounding of an
# fp32-accumulated sum of exact products, so against fp64 it must agree to a
# few fp16 ulps of the output magnitude.
TIGHT_REL_L2 = 2e-3 * 0.25


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def assert_gates(c_dev, cref, tight_ref=None):
    c = c_dev.float().cpu().numpy()
    max_abs, rel, finite = orc.gemm_errors(c, cref)
    assert finite, "non-finite output"
    assert max_abs <= orc.GATE_MAX_ABS, f"max abs err {max_abs}"
    assert rel <= orc.GATE_REL_L2, f"rel-L2 {rel}"
    if tight_ref is not None:
        _, rel_t, _ = orc.gemm_errors(c, tight_ref)
        assert rel_t <= TIGHT_REL_L2, f"rel-L2 vs fp64 exact {rel_t}"
    return max_abs, rel


def check_status():
    assert bf.stream_status() == 0


# ---------------------------------------------------------------------------
# tcgen05 layout probe
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("nb", [16, 32, 64])
def test_probe_umma_layout(nb):
    rng = np.random.default_rng(nb)
    a = rng.integers(-4, 5, size=(128, 64)).astype(np.float16)
    b = rng.integers(-4, 5, size=(nb, 64)).astype(np.float16)
    d = bf.probe_umma(cu(a), cu(b), nb)
    check_status()
    want = a.astype(np.float64) @ b.astype(np.float64).T   # small integers: exact in fp32
    got = d.cpu().numpy()
    assert np.array_equal(got, want.astype(np.float32)), np.argwhere(got != want)[:8]


# ---------------------------------------------------------------------------
# dequant: bit-exact
# ---------------------------------------------------------------------------
def test_dequant_q4_0_bit_exact_config0():
    wq, ws = orc.gen_q4_0(512, 5120, seed=10)
    out = bf.dequant_q4_0(cu(wq), cu(ws))
    check_status()
    want = orc.dequant_q4_0_planes(wq, ws)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_dequant_q4_0_bit_exact_all_scale_patterns():
    # every finite fp16 scale (subnormals and negatives included), random nibbles
    rng = np.random.default_rng(11)
    bits = np.arange(0x10000, dtype=np.uint32)
    bits = bits[(bits & 0x7C00) != 0x7C00].astype(np.uint16)        # drop inf/nan
    n = bits.size // 8
    ws = bits[: n * 8].view(np.float16).reshape(n, 8)
    wq = rng.integers(0, 256, size=(n, 128), dtype=np.uint8)
    out = bf.dequant_q4_0(cu(wq), cu(ws))
    check_status()
    with np.errstate(over="ignore"):
        want = orc.dequant_q4_0_planes(wq, ws)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_dequant_q4_0_matches_reference_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "q4_0_reference.npz"))
    for case in "abc":
        out = bf.dequant_q4_0(cu(g[f"{case}_wq"]), cu(g[f"{case}_ws"]))
        want = g[f"{case}_ref"].astype(np.float16)
        assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16)), case
    check_status()


def test_dequant_q4k_bit_exact_gguf_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "q4k_gguf.npz"))
    for case in "ab":
        k = int(g[f"{case}_k"])
        out = bf.dequant_q4k(cu(g[f"{case}_blocks"]), k)
        with np.errstate(over="ignore"):
            want = g[f"{case}_w32"].astype(np.float16)
        assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16)), case
    check_status()


def test_dequant_q4k_bit_exact_config2():
    blocks = orc.gen_q4k(1024, 5120, seed=12)
    out = bf.dequant_q4k(cu(blocks), 5120)
    check_status()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), orc.dequant_q4k(blocks, 5120).view(np.uint16))


def test_dequant_q4_0_ggml_bit_exact_gguf_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "q4_0_gguf.npz"))
    k = int(g["k"])
    out = bf.dequant_q4_0_ggml(cu(g["blocks"]), k)
    check_status()
    with np.errstate(over="ignore"):
        want = g["w32"].astype(np.float16)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


# ---------------------------------------------------------------------------
# GEMM parity
# ---------------------------------------------------------------------------
SHAPES = [
    (1, 128, 256), (3, 256, 512), (8, 640, 1024), (16, 384, 768), (17, 200, 512), (32, 1024, 2048),
    (33, 256, 512), (48, 130, 256), (64, 512, 1536), (65, 256, 512), (130, 384, 768),
    (1, 128, 16384),   # one tile, K split over a cluster of 8
    (8, 256, 8192),
    (5, 3840, 5120),   # 30 tiles: clusters of 3-4, ~5-7 units per CTA
    (2, 1024, 40960),  # 8 tiles x 160 units: 20 units per CTA, deep operand-slot reuse
    (40, 1024, 512), (64, 2560, 1024), (57, 520, 256),   # N > K, 33-64 rows: one 64-row decode launch
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_q4k_parity(m, n, k):
    blocks = orc.gen_q4k(n, k, seed=m * 7 + n + k)
    a = orc.gen_activations(m, k, seed=m + 3 * k)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    check_status()
    w32 = orc.dequant_q4k_f32(blocks, k)
    cref = orc.gemm_ref(a, w32)
    exact = a.astype(np.float64) @ w32.astype(np.float64).T
    assert_gates(c, cref, exact)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_q4_0_parity(m, n, k):
    wq, ws = orc.gen_q4_0(n, k, seed=m * 5 + n + k)
    a = orc.gen_activations(m, k, seed=m + 5 * k)
    c = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
    check_status()
    w16 = orc.dequant_q4_0_planes(wq, ws)   # the kernel's operand, bit-exact
    cref = orc.gemm_ref(a, orc.dequant_q4_0_planes_f32(wq, ws))
    exact = a.astype(np.float64) @ w16.astype(np.float64).T
    assert_gates(c, cref, exact)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_q4_0_ggml_parity(m, n, k):
    """llama.cpp block_q4_0 rows: the same weights as the split planes, so the
    fp16 operands are identical and so is the whole accumulation order: the
    output must equal the split-plane GEMM's bit for bit, and pass the gates."""
    wq, ws = orc.gen_q4_0(n, k, seed=m * 3 + n + k)
    blocks = orc.q4_0_planes_to_ggml_blocks(wq, ws)
    a = orc.gen_activations(m, k, seed=m + 11 * k)
    c = bf.gemm_q4_0_ggml(cu(blocks), cu(a))
    c_planes = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
    check_status()
    assert torch.equal(c.view(torch.int16), c_planes.view(torch.int16))
    w16 = orc.dequant_q4_0_ggml(blocks, k)
    cref = orc.gemm_ref(a, orc.dequant_q4_0_planes_f32(wq, ws))
    assert_gates(c, cref, a.astype(np.float64) @ w16.astype(np.float64).T)


def test_gemm_q4_0_ggml_gguf_golden(golden_dir):
    """GEMM over the gguf-py block_q4_0 fixture (16 rows x 256), tiled to 128 rows."""
    g = np.load(os.path.join(golden_dir, "q4_0_gguf.npz"))
    k = int(g["k"])
    blocks = np.tile(g["blocks"], (8, 1))
    w32 = np.tile(g["w32"], (8, 1))
    a = orc.gen_activations(9, k, seed=99)
    c = bf.gemm_q4_0_ggml(cu(blocks), cu(a))
    check_status()
    # The fixture's scales are arbitrary fp16 values (weights up to ~126), so
    # outputs reach ~1e3 and the absolute gate does not apply; the result must
    # still be the fp16 rounding of an fp32 sum of the exact fp16 products.
    exact = a.astype(np.float64) @ w32.astype(np.float16).astype(np.float64).T
    got = c.float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - exact) <= 2.0 ** -10 * np.abs(exact) + 1e-2)


# (cluster size, M, N, K): forced K splits, including schedules where every
# cluster takes several tiles in turn (the reduction buffer is reused)
KSPLIT_CASES = [
    (1, 32, 384, 512),
    (2, 8, 640, 1024),
    (3, 32, 7680, 768),    # 60 tiles over <= 49 clusters: two tiles per cluster
    (4, 17, 1280, 1280),   # 5 units over 4 ranks: uneven split
    (5, 3, 2560, 5120),
    (8, 5, 3072, 2048),    # 24 tiles over <= 18 clusters
    (8, 1, 128, 2048),     # one unit per rank
    (2, 64, 2048, 1024),   # 64-row batch tile, split over a cluster of 2
    (2, 48, 5120, 512),    # 64-row batch tile, 40 tiles, two tiles per cluster for some
]


@pytest.mark.parametrize("csize,m,n,k", KSPLIT_CASES)
def test_gemm_forced_ksplit(csize, m, n, k):
    blocks = orc.gen_q4k(n, k, seed=csize * 11 + m)
    wq, ws = orc.gen_q4_0(n, k, seed=csize * 13 + m)
    a = orc.gen_activations(m, k, seed=csize + 7 * m)
    bf.set_ksplit(csize)
    try:
        c = bf.gemm_q4k(cu(blocks), cu(a))
        c0 = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
        check_status()
    finally:
        bf.set_ksplit(0)
    w32 = orc.dequant_q4k_f32(blocks, k)
    assert_gates(c, orc.gemm_ref(a, w32), a.astype(np.float64) @ w32.astype(np.float64).T)
    w16 = orc.dequant_q4_0_planes(wq, ws)
    assert_gates(c0, orc.gemm_ref(a, orc.dequant_q4_0_planes_f32(wq, ws)),
                 a.astype(np.float64) @ w16.astype(np.float64).T)


@pytest.mark.parametrize("m", [1, 8, 32])
def test_gemm_headline_shapes(m):
    k = n = 5120
    blocks = orc.gen_q4k(n, k, seed=2)
    a = orc.gen_activations(m, k, seed=3)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    wq, ws = orc.gen_q4_0(n, k, seed=4)
    c0 = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
    check_status()
    assert_gates(c, orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k)))
    assert_gates(c0, orc.gemm_ref(a, orc.dequant_q4_0_planes_f32(wq, ws)))


def test_gemm_q4k_config2_wide():
    m, n, k = 32, 17408, 5120
    blocks = orc.gen_q4k(n, k, seed=21)
    a = orc.gen_activations(m, k, seed=22)
    c = bf.gemm_q4k(cu(blocks), cu(a))
    check_status()
    assert_gates(c, orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k)))


def test_reference_golden_gate(golden_dir):
    # the reference's own quantizer output and gate product (kernels/q4k_batched.py:97-104)
    g = np.load(os.path.join(golden_dir, "q4_0_reference.npz"))
    for case in "ab":
        wq, ws, a, cref = g[f"{case}_wq"], g[f"{case}_ws"], g[f"{case}_a"], g[f"{case}_c"]
        k = a.shape[1]
        if k % 256:
            continue
        c = bf.gemm_q4_0(cu(wq), cu(ws), cu(a))
        assert_gates(c, cref)
    check_status()


def test_busfill_q4_compat_fp32_all_rows():
    # the reference computes only rows < 32 (kernels/busfill_v1a.cu:55-56); we compute all
    bsz, n, k = 40, 256, 1024
    wq, ws = orc.gen_q4_0(n, k, seed=31)
    a = orc.gen_activations(bsz, k, seed=32)
    c = torch.full((bsz, n), float("nan"), dtype=torch.float32, device=DEV)
    bf.busfill_q4(cu(a), cu(wq), cu(ws), c, bsz, k, n)
    check_status()
    cref = orc.gemm_ref(a, orc.dequant_q4_0_planes_f32(wq, ws))
    max_abs, rel, finite = orc.gemm_errors(c.cpu().numpy(), cref)
    assert finite and max_abs <= 0.6 and rel <= 1e-3
    # fp32 output keeps more than fp16 would
    exact = a.astype(np.float64) @ orc.dequant_q4_0_planes(wq, ws).astype(np.float64).T
    assert orc.gemm_errors(c.cpu().numpy(), exact)[1] < 1e-5


def test_no_writes_outside_output():
    m, n, k = 5, 200, 512
    blocks = orc.gen_q4k(n, k, seed=41)
    a = orc.gen_activations(m, k, seed=42)
    big = torch.full((m + 2, n), -7.0, dtype=torch.float16, device=DEV)
    out = big[1:1 + m]
    assert out.is_contiguous()
    bf.gemm_q4k(cu(blocks), cu(a), out=out)
    check_status()
    assert torch.all(big[0] == -7.0) and torch.all(big[m + 1] == -7.0)
    assert_gates(out, orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k)))


@pytest.mark.parametrize("m,n,k,shift", [(20, 130, 512, 0), (32, 256, 1024, 1), (9, 640, 2048, 0)])
def test_decode_output_store_paths(m, n, k, shift):
    """The decode epilogue writes 8 consecutive outputs per 16-byte store when
    N % 8 == 0 and C is 16-byte aligned, one output per store otherwise
    (N = 130; C one element past an aligned address); every case against the
    oracle, nothing written outside C."""
    bf.set_prefill_min_m(10 ** 6)
    try:
        blocks = orc.gen_q4k(n, k, seed=m + n)
        a = orc.gen_activations(m, k, seed=m + k)
        big = torch.full((m * n + shift + 8,), -7.0, dtype=torch.float16, device=DEV)
        out = big[shift:shift + m * n].view(m, n)
        bf.gemm_q4k(cu(blocks), cu(a), out=out)
        check_status()
    finally:
        bf.set_prefill_min_m(0)
    assert torch.all(big[:shift] == -7.0) and torch.all(big[shift + m * n:] == -7.0)
    assert_gates(out, orc.gemm_ref(a, orc.dequant_q4k_f32(blocks, k)))


def test_deterministic_bitwise():
    m, n, k = 32, 640, 5120     # split-K tiles: fix-up order must be fixed
    blocks = cu(orc.gen_q4k(n, k, seed=51))
    a = cu(orc.gen_activations(m, k, seed=52))
    c1 = bf.gemm_q4k(blocks, a)
    c2 = bf.gemm_q4k(blocks, a)
    check_status()
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))


def test_back_to_back_pdl_and_graph_replay():
    # a chain of dependent GEMMs (output of one feeds the next) in a CUDA graph
    k = n = 1024
    layers = [cu(orc.gen_q4k(n, k, seed=60 + i)) for i in range(4)]
    x0 = cu(orc.gen_activations(8, k, seed=61))

    def chain(x):
        for w in layers:
            x = bf.gemm_q4k(w, x) * 0.05
        return x

    eager = chain(x0)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain(x0)   # warm-up on the capture stream (allocates its workspace)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = chain(x0)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), eager.view(torch.int16))
    assert bf.stream_status(s) == 0
    check_status()


def test_pdl_off_matches_pdl_on():
    m, n, k = 16, 512, 2048
    blocks = cu(orc.gen_q4k(n, k, seed=71))
    a = cu(orc.gen_activations(m, k, seed=72))
    c_on = bf.gemm_q4k(blocks, a)
    bf.set_pdl(False)
    try:
        c_off = bf.gemm_q4k(blocks, a)
    finally:
        bf.set_pdl(True)
    check_status()
    assert torch.equal(c_on.view(torch.int16), c_off.view(torch.int16))


def test_argument_errors():
    lib = bf.load_library()
    blocks = cu(orc.gen_q4k(128, 512, seed=81))
    a = cu(orc.gen_activations(4, 512, seed=82))
    c = torch.empty((4, 128), dtype=torch.float16, device=DEV)
    s = bf._stream(None)
    p = bf._ptr
    assert lib.busfill_gemm_q4k(p(blocks), p(a), p(c), 4, 128, 300, s) == -2      # K % 256
    assert lib.busfill_gemm_q4k(p(blocks), p(a), p(c), 0, 128, 512, s) == -2      # M < 1
    mis = torch.empty(4 * 512 + 8, dtype=torch.float16, device=DEV)[1:1 + 4 * 512]
    import ctypes
    assert lib.busfill_gemm_q4k(p(blocks), ctypes.c_void_p(mis.data_ptr()), p(c), 4, 128, 512, s) == -3
    with pytest.raises(ValueError):
        bf.gemm_q4k(blocks, a[:, :256].contiguous())      # K disagrees with the block rows
    with pytest.raises(bf.BusfillError) as ei:
        bf.busfill_q4(a, cu(np.zeros((128, 150), np.uint8)), cu(np.zeros((128, 9), np.float16)),
                      torch.empty((4, 128), dtype=torch.float32, device=DEV), 4, 300, 128)
    assert ei.value.status == -2
    check_status()
