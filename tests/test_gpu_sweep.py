"""GPU parity of the layer sweep busfill_gemm_q4k_sweep (several Q4_K GEMMs
in one launch, ops split stream-K over all SMs), through the C ABI.

Every op is checked against the oracle on the input the GPU actually read (for
a dependent op, the earlier op's fp16 output as stored): plain GEMMs with the
north_star gates (max abs err <= 0.6, rel-L2 <= 1e-3) where the outputs have
the headline's magnitude, else rel-L2 <= 1e-3 and max abs err <= 2e-3 of the
largest |C| (chained layers with unnormalised synthetic weights grow by ~1e2
per GEMM; the first input is scaled down so that every output stays in fp16).
A split tile's partials are added in CTA order, so repeated calls are bitwise
equal; against the one-GEMM entry points the sums differ only in fp32 order.
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


def host(t):
    return t.cpu().numpy()


def check_rel(got, want, where, rel_gate=1e-3, abs_frac=2e-3):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.all(np.isfinite(got)), where
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    err = np.max(np.abs(got - want))
    assert rel <= rel_gate, (where, rel)
    assert err <= abs_frac * np.max(np.abs(want)) + 1e-6, (where, err, np.max(np.abs(want)))


def layer(m, seed, o=(512, 768), qkv=(604, 512), ffn=1024, down=512, scale=16384.0):
    """A decoder layer's four ops at small sizes: O (input `attn`), QKV (input
    `x`, independent), gate/up SwiGLU on O's output, down on the SwiGLU
    output. QKV's N = 604 is not a multiple of 8 (the scalar store path)."""
    rng = seed
    w = {
        "o": orc.gen_q4k(o[0], o[1], seed=rng + 1),
        "qkv": orc.gen_q4k(qkv[0], qkv[1], seed=rng + 2),
        "gate": orc.gen_q4k(ffn, o[0], seed=rng + 3),
        "up": orc.gen_q4k(ffn, o[0], seed=rng + 4),
        "down": orc.gen_q4k(down, ffn, seed=rng + 5),
    }
    attn = (orc.gen_activations(m, o[1], seed=rng + 6).astype(np.float32) / scale).astype(np.float16)
    x = (orc.gen_activations(m, qkv[1], seed=rng + 7).astype(np.float32) / 64).astype(np.float16)
    d = {k: cu(v) for k, v in w.items()}
    a_attn, a_x = cu(attn), cu(x)
    out = {
        "o": torch.empty((m, o[0]), dtype=torch.float16, device=DEV),
        "qkv": torch.empty((m, qkv[0]), dtype=torch.float16, device=DEV),
        "h": torch.empty((m, ffn), dtype=torch.float16, device=DEV),
        "down": torch.empty((m, down), dtype=torch.float16, device=DEV),
    }
    ops = [
        {"w": d["o"], "a": a_attn, "out": out["o"]},
        {"w": d["qkv"], "a": a_x, "out": out["qkv"]},
        {"w": d["gate"], "w_up": d["up"], "a": out["o"], "out": out["h"], "dep": 0},
        {"w": d["down"], "a": out["h"], "out": out["down"], "dep": 2},
    ]
    return w, d, attn, x, out, ops


def check_layer(w, attn, x, out):
    k_o, k_qkv = attn.shape[1], x.shape[1]
    o = host(out["o"])
    check_rel(o, orc.gemm_ref(attn, orc.dequant_q4k_f32(w["o"], k_o)), "o")
    c = orc.gemm_ref(x, orc.dequant_q4k_f32(w["qkv"], k_qkv))
    max_abs, rel, finite = orc.gemm_errors(host(out["qkv"]).astype(np.float32), c)
    assert finite and max_abs <= 0.6 and rel <= 1e-3, ("qkv", max_abs, rel)
    h = host(out["h"])
    k_h = o.shape[1]
    check_rel(h, orc.swiglu_ref(o, orc.dequant_q4k_f32(w["gate"], k_h), orc.dequant_q4k_f32(w["up"], k_h)), "swiglu")
    check_rel(host(out["down"]), orc.gemm_ref(h, orc.dequant_q4k_f32(w["down"], h.shape[1])), "down")


@pytest.mark.parametrize("m", [1, 8, 16, 17, 32])
def test_sweep_layer(m):
    w, d, attn, x, out, ops = layer(m, seed=100 + m)
    bf.gemm_q4k_sweep(ops)
    assert bf.stream_status() == 0
    check_layer(w, attn, x, out)


def test_sweep_deterministic_and_repeatable():
    """Back-to-back calls on one stream (the counters return to zero at the end
    of every launch) give bitwise equal outputs."""
    w, d, attn, x, out, ops = layer(32, seed=7)
    bf.gemm_q4k_sweep(ops)
    first = {k: v.clone() for k, v in out.items()}
    for _ in range(3):
        for v in out.values():
            v.zero_()
        bf.gemm_q4k_sweep(ops)
    assert bf.stream_status() == 0
    for k in out:
        assert torch.equal(out[k], first[k]), k
    check_layer(w, attn, x, out)


def test_sweep_matches_one_gemm_entry_points():
    """The same GEMMs through busfill_gemm_q4k / busfill_gemm_q4k_swiglu
    differ only in the order of fp32 additions."""
    w, d, attn, x, out, ops = layer(32, seed=11)
    bf.gemm_q4k_sweep(ops)
    o = bf.gemm_q4k(d["o"], ops[0]["a"])
    qkv = bf.gemm_q4k(d["qkv"], ops[1]["a"])
    h = bf.gemm_q4k_swiglu(d["gate"], d["up"], out["o"])
    dn = bf.gemm_q4k(d["down"], out["h"])
    assert bf.stream_status() == 0
    for name, ref in (("o", o), ("qkv", qkv), ("h", h), ("down", dn)):
        check_rel(host(out[name]).astype(np.float64), host(ref).astype(np.float64), name, rel_gate=2e-3,
                  abs_frac=4e-3)


def test_sweep_ops_smaller_than_grid():
    """Ops of fewer units than CTAs (most CTAs have no share of them) next to a
    larger one; one op of a single unit."""
    m = 5
    w1 = orc.gen_q4k(128, 256, seed=1)       # 1 unit
    w2 = orc.gen_q4k(2048, 1024, seed=2)     # 64 units
    w3 = orc.gen_q4k(384, 2048, seed=3)      # 24 units
    a1 = (orc.gen_activations(m, 256, seed=4).astype(np.float32) / 64).astype(np.float16)
    a2 = (orc.gen_activations(m, 1024, seed=5).astype(np.float32) / 64).astype(np.float16)
    a3 = (orc.gen_activations(m, 2048, seed=6).astype(np.float32) / 64).astype(np.float16)
    outs = [torch.empty((m, n), dtype=torch.float16, device=DEV) for n in (128, 2048, 384)]
    ops = [{"w": cu(w1), "a": cu(a1), "out": outs[0]}, {"w": cu(w2), "a": cu(a2), "out": outs[1]},
           {"w": cu(w3), "a": cu(a3), "out": outs[2]}]
    bf.gemm_q4k_sweep(ops)
    assert bf.stream_status() == 0
    for (wq, a, k), o in zip(((w1, a1, 256), (w2, a2, 1024), (w3, a3, 2048)), outs):
        max_abs, rel, finite = orc.gemm_errors(host(o).astype(np.float32), orc.gemm_ref(a, orc.dequant_q4k_f32(wq, k)))
        assert finite and max_abs <= 0.6 and rel <= 1e-3, (k, max_abs, rel)


def test_sweep_single_op_many_splits():
    """One op whose tiles are split between many CTAs each: 10 tiles of 32
    units (K = 8192) over 148 CTAs, 2-3 units a CTA, ~15 contributors a tile."""
    m, n, k = 32, 1280, 8192
    wq = orc.gen_q4k(n, k, seed=21)
    a = (orc.gen_activations(m, k, seed=22).astype(np.float32) / 64).astype(np.float16)
    out = torch.empty((m, n), dtype=torch.float16, device=DEV)
    bf.gemm_q4k_sweep([{"w": cu(wq), "a": cu(a), "out": out}])
    assert bf.stream_status() == 0
    max_abs, rel, finite = orc.gemm_errors(host(out).astype(np.float32), orc.gemm_ref(a, orc.dequant_q4k_f32(wq, k)))
    assert finite and max_abs <= 0.6 and rel <= 1e-3, (max_abs, rel)


def test_sweep_graph_replay():
    """Captured once (after a first eager call made the stream's workspace)
    and replayed: each replay equals the eager result."""
    w, d, attn, x, out, ops = layer(16, seed=31)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        bf.gemm_q4k_sweep(ops, stream=st)
        st.synchronize()
        first = {k: v.clone() for k, v in out.items()}
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            bf.gemm_q4k_sweep(ops, stream=st)
        for _ in range(3):
            for v in out.values():
                v.zero_()
            g.replay()
        st.synchronize()
        assert bf.stream_status(st) == 0
    for k in out:
        assert torch.equal(out[k], first[k]), k
    del g


def test_sweep_full_size_layer():
    """BASELINE config 3's layer at M = 32 (QKV 5120 -> 10240, O 8192 -> 5120,
    gate/up 5120 -> 2 x 17408, down 17408 -> 5120) against the one-GEMM entry
    points on the same inputs."""
    m = 32
    gen = torch.Generator(device=DEV)
    gen.manual_seed(5)

    def q4k(n, k):
        return cu(orc.gen_q4k(n, k, seed=n + 3 * k))

    wo, wqkv, wg, wu, wd = q4k(5120, 8192), q4k(10240, 5120), q4k(17408, 5120), q4k(17408, 5120), q4k(5120, 17408)
    attn = (torch.randn((m, 8192), device=DEV, generator=gen) / 2 ** 20).half()   # keeps every output inside fp16
    x = (torch.randn((m, 5120), device=DEV, generator=gen) / 64).half()
    o = torch.empty((m, 5120), dtype=torch.float16, device=DEV)
    qkv = torch.empty((m, 10240), dtype=torch.float16, device=DEV)
    h = torch.empty((m, 17408), dtype=torch.float16, device=DEV)
    dn = torch.empty((m, 5120), dtype=torch.float16, device=DEV)
    bf.gemm_q4k_sweep([{"w": wo, "a": attn, "out": o}, {"w": wqkv, "a": x, "out": qkv},
                       {"w": wg, "w_up": wu, "a": o, "out": h, "dep": 0}, {"w": wd, "a": h, "out": dn, "dep": 2}])
    assert bf.stream_status() == 0
    ref_o = bf.gemm_q4k(wo, attn)
    ref_qkv = bf.gemm_q4k(wqkv, x)
    ref_h = bf.gemm_q4k_swiglu(wg, wu, o)
    ref_d = bf.gemm_q4k(wd, h)
    assert bf.stream_status() == 0
    for name, got, ref in (("o", o, ref_o), ("qkv", qkv, ref_qkv), ("h", h, ref_h), ("down", dn, ref_d)):
        check_rel(host(got), host(ref), name, rel_gate=2e-3, abs_frac=4e-3)


def test_sweep_whole_tile_ops():
    """Ops whose tile count nearly fills the grid take whole tiles per CTA (no
    split tiles): 140 tiles, 280 tiles (two per CTA) and a SwiGLU pair of 148
    tiles on a 148-SM B200, next to a split op."""
    m = 8
    specs = [(140 * 128, 512, False), (280 * 128, 256, False), (148 * 128, 256, True), (1280, 1024, False)]
    ops, ref = [], []
    for i, (n, k, sw) in enumerate(specs):
        wq = orc.gen_q4k(n, k, seed=40 + i)
        a = (orc.gen_activations(m, k, seed=50 + i).astype(np.float32) / 64).astype(np.float16)
        out = torch.empty((m, n), dtype=torch.float16, device=DEV)
        op = {"w": cu(wq), "a": cu(a), "out": out}
        if sw:
            wu = orc.gen_q4k(n, k, seed=60 + i)
            op["w_up"] = cu(wu)
            ref.append(("swiglu", orc.swiglu_ref(a, orc.dequant_q4k_f32(wq, k), orc.dequant_q4k_f32(wu, k))))
        else:
            ref.append(("gemm", orc.gemm_ref(a, orc.dequant_q4k_f32(wq, k))))
        ops.append(op)
    bf.gemm_q4k_sweep(ops)
    assert bf.stream_status() == 0
    for op, (kind, want) in zip(ops, ref):
        got = host(op["out"]).astype(np.float32)
        if kind == "swiglu":
            check_rel(got, want, "swiglu")
        else:
            max_abs, rel, finite = orc.gemm_errors(got, want)
            assert finite and max_abs <= 0.6 and rel <= 1e-3, (max_abs, rel)


def test_sweep_two_layers_eight_ops():
    """Two layers in one launch (BUSFILL_SWEEP_MAX_OPS = 8), interleaved so
    that no op directly follows the op it reads: O1, O2, QKV1, gate/up1 (after
    O1), gate/up2 (after O2), down1, down2, QKV2."""
    w1, d1, attn1, x1, out1, ops1 = layer(16, seed=71)
    w2, d2, attn2, x2, out2, ops2 = layer(16, seed=72)
    o1, o2, q1, g1, g2, dn1, dn2, q2 = ops1[0], ops2[0], ops1[1], dict(ops1[2]), dict(ops2[2]), dict(ops1[3]), \
        dict(ops2[3]), ops2[1]
    g1["dep"], g2["dep"], dn1["dep"], dn2["dep"] = 0, 1, 3, 4
    bf.gemm_q4k_sweep([o1, o2, q1, g1, g2, dn1, dn2, q2])
    assert bf.stream_status() == 0
    check_layer(w1, attn1, x1, out1)
    check_layer(w2, attn2, x2, out2)
