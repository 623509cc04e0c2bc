"""Generate the golden fixtures that pin the CPU oracle.

Run in a container that has the reference checkout and gguf-py installed:

    python tests/golden/make_golden.py --reference /path/to/bus-fill

Fixtures written next to this script (small .npz files, committed):

* ``q4_0_reference.npz`` -- the reference's own quantizer
  ``quantize_q4q`` (kernels/q4k_batched.py:65-79) run on seeded fp32 weights,
  plus the reference gate's product ``A.float() @ ref.T``
  (kernels/q4k_batched.py:100).
* ``q4k_gguf.npz`` -- gguf-py 0.19.0 ``Q4_K.dequantize_blocks`` (the published
  llama.cpp ``block_q4_K`` dequant in numpy) on seeded random blocks. The
  reference has no Q4_K code, so this third-party implementation is the anchor.
* ``q5k_gguf.npz`` -- gguf-py 0.19.0 ``Q5_K.dequantize_blocks`` on seeded
  random ``block_q5_K`` rows (a BASELINE "next" format; no reference code).
* ``q6k_gguf.npz`` -- gguf-py 0.19.0 ``Q6_K.dequantize_blocks`` on seeded
  random ``block_q6_K`` rows (the other "next" k-quant format).
* ``q4_0_gguf.npz`` -- gguf-py 0.19.0 ``Q4_0.dequantize_blocks`` on seeded
  random llama.cpp ``block_q4_0`` rows (the AoS Q4_0 layout).

Nothing here runs at test time; the tests only read the .npz files.
"""
from __future__ import annotations

import argparse
import importlib.util
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference_quantizer(ref_root: str):
    path = os.path.join(ref_root, "kernels", "q4k_batched.py")
    spec = importlib.util.spec_from_file_location("busfill_reference_q4k_batched", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.quantize_q4q


def make_q4_0_reference(ref_root: str):
    import torch

    quantize_q4q = _load_reference_quantizer(ref_root)
    out = {}
    cases = [("a", 64, 256, 0.02, 0), ("b", 32, 512, 0.4, 1), ("c", 8, 64, 1.0, 2)]
    for name, n, k, scale, seed in cases:
        g = torch.Generator().manual_seed(1000 + seed)
        wf = torch.randn(n, k, generator=g) * scale
        if name == "c":
            wf[0].zero_()                          # amax clamp path (1e-6)
            wf[1, :32] = torch.linspace(-1, 1, 32)  # exact-tie rounding inputs
        bytes_, srep, ref = quantize_q4q(wf, "cpu")
        a = torch.randn(4, k, generator=g).to(torch.float16)
        c = a.float() @ ref.T
        out[f"{name}_wf"] = wf.numpy().astype(np.float32)
        out[f"{name}_wq"] = bytes_.numpy().astype(np.uint8)
        out[f"{name}_ws"] = srep[:, ::16].contiguous().numpy().astype(np.float16)
        out[f"{name}_ref"] = ref.numpy().astype(np.float32)
        out[f"{name}_a"] = a.numpy()
        out[f"{name}_c"] = c.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4_0_reference.npz"), **out)


def _random_f16(rng, shape, lo_exp, hi_exp, signed):
    """fp16 values with exponents spread over [lo_exp, hi_exp] (all normal)."""
    mant = rng.integers(0, 1024, size=shape)
    exp = rng.integers(lo_exp + 15, hi_exp + 15 + 1, size=shape)
    sign = rng.integers(0, 2, size=shape) if signed else np.zeros(shape, dtype=np.int64)
    bits = (sign << 15) | (exp << 10) | mant
    return bits.astype(np.uint16).view(np.float16)


def make_q4k_gguf():
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    rng = np.random.default_rng(2024)
    out = {}
    # case a: config-2 distributions; case b: every byte random (all 6-bit
    # scale/min bit patterns, broad fp16 exponents, negative dmin allowed)
    n, k = 16, 512
    s = k // 256
    d = rng.uniform(0.001, 0.01, size=(n, s)).astype(np.float16)
    dmin = rng.uniform(0.0, 0.005, size=(n, s)).astype(np.float16)
    scales = rng.integers(0, 256, size=(n, s, 12), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(n, s, 128), dtype=np.uint8)
    blocks_a = np.concatenate([d.reshape(n, s, 1).view(np.uint8), dmin.reshape(n, s, 1).view(np.uint8),
                               scales, qs], axis=2).reshape(n, s * 144)
    n2, k2 = 24, 768
    s2 = k2 // 256
    d2 = _random_f16(rng, (n2, s2), -10, 2, signed=False)
    dmin2 = _random_f16(rng, (n2, s2), -12, 0, signed=True)
    scales2 = rng.integers(0, 256, size=(n2, s2, 12), dtype=np.uint8)
    qs2 = rng.integers(0, 256, size=(n2, s2, 128), dtype=np.uint8)
    blocks_b = np.concatenate([d2.reshape(n2, s2, 1).view(np.uint8), dmin2.reshape(n2, s2, 1).view(np.uint8),
                               scales2, qs2], axis=2).reshape(n2, s2 * 144)
    for name, blocks, kk in (("a", blocks_a, k), ("b", blocks_b, k2)):
        w32 = dequantize(blocks, GGMLQuantizationType.Q4_K)
        assert w32.shape == (blocks.shape[0], kk) and w32.dtype == np.float32
        out[f"{name}_blocks"] = blocks
        out[f"{name}_w32"] = w32
        out[f"{name}_k"] = np.array(kk)
    np.savez_compressed(os.path.join(HERE, "q4k_gguf.npz"), **out)


def make_q5k_gguf():
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    rng = np.random.default_rng(2025)
    out = {}
    # case a: config-2-like distributions; case b: every byte random
    for name, n, k, wide in (("a", 16, 512, False), ("b", 24, 768, True)):
        s = k // 256
        if wide:
            d = _random_f16(rng, (n, s), -10, 2, signed=False)
            dmin = _random_f16(rng, (n, s), -12, 0, signed=True)
        else:
            d = rng.uniform(0.001, 0.01, size=(n, s)).astype(np.float16)
            dmin = rng.uniform(0.0, 0.005, size=(n, s)).astype(np.float16)
        rest = rng.integers(0, 256, size=(n, s, 12 + 32 + 128), dtype=np.uint8)
        blocks = np.concatenate([d.reshape(n, s, 1).view(np.uint8), dmin.reshape(n, s, 1).view(np.uint8), rest],
                                axis=2).reshape(n, s * 176)
        w32 = dequantize(blocks, GGMLQuantizationType.Q5_K)
        assert w32.shape == (n, k) and w32.dtype == np.float32
        out[f"{name}_blocks"] = blocks
        out[f"{name}_w32"] = w32
        out[f"{name}_k"] = np.array(k)
    np.savez_compressed(os.path.join(HERE, "q5k_gguf.npz"), **out)


def make_q6k_gguf():
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    rng = np.random.default_rng(2026)
    out = {}
    # case a: the generator's distributions; case b: every byte random except
    # d, whose exponents are spread over the normal fp16 range (either sign)
    for name, n, k, wide in (("a", 16, 512, False), ("b", 24, 768, True)):
        s = k // 256
        if wide:
            d = _random_f16(rng, (n, s), -14, 3, signed=True)
        else:
            d = rng.uniform(0.0001, 0.0005, size=(n, s)).astype(np.float16)
        body = rng.integers(0, 256, size=(n, s, 208), dtype=np.uint8)
        blocks = np.concatenate([body, d.reshape(n, s, 1).view(np.uint8)], axis=2).reshape(n, s * 210)
        w32 = dequantize(blocks, GGMLQuantizationType.Q6_K)
        assert w32.shape == (n, k) and w32.dtype == np.float32
        out[f"{name}_blocks"] = blocks
        out[f"{name}_w32"] = w32
        out[f"{name}_k"] = np.array(k)
    np.savez_compressed(os.path.join(HERE, "q6k_gguf.npz"), **out)


def make_q4_0_gguf():
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    rng = np.random.default_rng(77)
    n, k = 16, 256
    nb = k // 32
    d = _random_f16(rng, (n, nb), -10, 3, signed=True)
    qs = rng.integers(0, 256, size=(n, nb, 16), dtype=np.uint8)
    blocks = np.concatenate([d.reshape(n, nb, 1).view(np.uint8), qs], axis=2).reshape(n, nb * 18)
    w32 = dequantize(blocks, GGMLQuantizationType.Q4_0)
    np.savez_compressed(os.path.join(HERE, "q4_0_gguf.npz"), blocks=blocks, w32=w32, k=np.array(k))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="bus-fill checkout (read-only)")
    args = ap.parse_args()
    make_q4_0_reference(args.reference)
    make_q4k_gguf()
    make_q5k_gguf()
    make_q6k_gguf()
    make_q4_0_gguf()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
