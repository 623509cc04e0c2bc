"""CPU oracle for the batched dequant-fused 4-bit-weight GEMM.

TEST INFRASTRUCTURE ONLY. This module is the checker, never the thing that is
measured or shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``) may import it.
The product path (``busfill_b200`` and ``libbusfill.so``) never touches it.

What it restates (numpy, byte/integer arithmetic plus IEEE fp16/fp32 rounding):

* Q4_0 "split planes" -- the reference's weight layout
  (kernels/busfill_v1a.cu:43-45, kernels/q4k_batched.py:9-11):
  ``Wq[N, K/2]`` u8, byte j of 32-value block b of a row holds element
  ``32b+2j`` in its low nibble and ``32b+2j+1`` in its high nibble
  (kernels/busfill_v1a.cu:126-130, kernels/q4k_batched.py:72-73);
  ``Ws[N, K/32]`` fp16, one scale ``d`` per block.
* Q4_0 dequant semantics -- kernels/busfill_v0.cu:74-81:
  ``w = fp16_rn(float(nib - 8) * float(d))`` (the fp32 product is exact, so
  this is one round-to-nearest-even to fp16).
* The reference quantizer ``quantize_q4q`` -- kernels/q4k_batched.py:65-79.
* The GEMM gate -- kernels/q4k_batched.py:97-104: ``C`` vs
  ``A.float() @ ref.T`` in fp32, max abs err <= 0.6; plus rel-L2 <= 1e-3 and
  "every output finite".
* Q4_K: NOT IN THE REFERENCE (the name appears only at
  kernels/q4k_batched.py:7-8 and RESULTS.md:86-88). The format is llama.cpp's
  ``block_q4_K`` (256-value super-block, 144 bytes: fp16 d, fp16 dmin,
  12 bytes of packed 6-bit sub-block scales/mins, 128 nibble bytes), as
  published in gguf-py 0.19.0 (``gguf/quants.py``, ``Q4_K.get_scale_min`` and
  ``Q4_K.dequantize_blocks``), a third-party dependency that the reference
  does not vendor. Its dequant is ``w32 = fp32(d)*sc * q - fp32(dmin)*m`` in
  fp32; the fp16 operand is ``fp16_rn(w32)``.

Parity pins (tests/test_oracle.py):
* Q4_0 -- pinned against golden vectors produced by running the reference's own
  ``quantize_q4q`` (tests/golden/make_golden.py, fixture ``q4_0_reference.npz``).
* Q4_K -- pinned against golden vectors produced by gguf-py 0.19.0's
  ``Q4_K.dequantize_blocks`` (fixture ``q4k_gguf.npz``); the reference itself
  has no Q4_K code, so this is the only available anchor.
* Q5_K and Q6_K (llama.cpp ``block_q5_K`` / ``block_q6_K``, the formats that
  Q4_K_M models mix in) -- pinned the same way against gguf-py 0.19.0
  (``q5k_gguf.npz``, ``q6k_gguf.npz``).
"""
from __future__ import annotations

import numpy as np

QK4_0 = 32          # values per Q4_0 block
QK_K = 256          # values per Q4_K super-block
Q4K_BLOCK_BYTES = 144
Q5K_BLOCK_BYTES = 176
Q6K_BLOCK_BYTES = 210
Q6K_PACKED_BYTES = 208   # a block_q6_K without its trailing fp16 d
Q4K_SCALE_BYTES = 12


# --------------------------------------------------------------------------
# Q4_0 split planes (reference layout)
# --------------------------------------------------------------------------
def quantize_q4q(wf: np.ndarray):
    """fp32 [N, K] -> (Wq [N, K/2] u8, Ws [N, K/32] fp16, ref [N, K] fp32).

    Restates kernels/q4k_batched.py:65-79: per 32-block ``scale = max(amax,
    1e-6) / 8`` in fp32, ``q = clamp(round_half_even(w/scale + 8), 0, 15)``,
    even element -> low nibble, odd -> high nibble, ``Ws = fp16(scale)`` and
    ``ref = (q - 8) * float(Ws)``. (The reference returns the scales replicated
    16x for its Triton kernel, kernels/q4k_batched.py:76-78; the planes here
    are the kernel ABI of kernels/busfill_v1a.cu:43-45.)
    """
    wf = np.ascontiguousarray(wf, dtype=np.float32)
    n, k = wf.shape
    assert k % QK4_0 == 0
    w = wf.reshape(n, k // QK4_0, QK4_0)
    amax = np.maximum(np.abs(w).max(axis=2), np.float32(1e-6))
    scale = (amax / np.float32(8.0)).astype(np.float32)
    q = np.clip(np.round(w / scale[:, :, None] + np.float32(8.0)), 0, 15).astype(np.uint8)
    lo = q[:, :, 0::2]
    hi = q[:, :, 1::2]
    wq = (lo | (hi << 4)).reshape(n, k // 2)
    s16 = scale.astype(np.float16)
    ref = ((q.astype(np.float32) - np.float32(8.0)) * s16.astype(np.float32)[:, :, None]).reshape(n, k)
    return wq, s16, ref


def unpack_q4_0_planes(wq: np.ndarray) -> np.ndarray:
    """Wq [N, K/2] u8 -> nibbles [N, K] u8 in element order (busfill_v1a.cu:126-130)."""
    n, kh = wq.shape
    out = np.empty((n, kh * 2), dtype=np.uint8)
    out[:, 0::2] = wq & 0x0F
    out[:, 1::2] = wq >> 4
    return out


def pack_q4_0_planes(nib: np.ndarray) -> np.ndarray:
    """Inverse of :func:`unpack_q4_0_planes`."""
    nib = np.asarray(nib, dtype=np.uint8)
    return (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)


def dequant_q4_0_planes_f32(wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Q4_0 dequant kept in fp32: ``(q - 8) * float(d)``, exact.

    This is the reference gate's weight matrix ``ref``
    (kernels/q4k_batched.py:75, kernels/busfill_v1a.cu:131-132).
    """
    nib = unpack_q4_0_planes(wq).astype(np.float32) - np.float32(8.0)
    n, k = nib.shape
    d = np.asarray(ws, dtype=np.float16).astype(np.float32).reshape(n, k // QK4_0, 1)
    return (nib.reshape(n, k // QK4_0, QK4_0) * d).reshape(n, k)


def dequant_q4_0_planes(wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Bit-exact Q4_0 dequant -> fp16 [N, K].

    kernels/busfill_v0.cu:74-81: ``__float2half((float)(nib - 8) * sc)`` with
    ``sc = __half2float(Ws)``. The fp32 product of a 4-bit integer and an fp16
    value is exact, so the result is one RN-even rounding to fp16.
    """
    nib = unpack_q4_0_planes(wq).astype(np.float32) - np.float32(8.0)
    n, k = nib.shape
    d = np.asarray(ws, dtype=np.float16).astype(np.float32).reshape(n, k // QK4_0, 1)
    return (nib.reshape(n, k // QK4_0, QK4_0) * d).reshape(n, k).astype(np.float16)


# --------------------------------------------------------------------------
# Q4_0 llama.cpp AoS blocks (18 bytes: fp16 d, 16 nibble bytes; byte j holds
# element j in its low nibble and element j+16 in its high nibble)
# --------------------------------------------------------------------------
def q4_0_planes_to_ggml_blocks(wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Re-pack reference split planes as llama.cpp ``block_q4_0`` rows [N, K/32*18] u8."""
    nib = unpack_q4_0_planes(wq)
    n, k = nib.shape
    nb = k // QK4_0
    nib = nib.reshape(n, nb, QK4_0)
    qs = (nib[:, :, :16] | (nib[:, :, 16:] << 4)).astype(np.uint8)
    d = np.asarray(ws, dtype=np.float16).reshape(n, nb, 1).view(np.uint8)
    return np.concatenate([d, qs], axis=2).reshape(n, nb * 18)


def dequant_q4_0_ggml(blocks: np.ndarray, k: int) -> np.ndarray:
    """llama.cpp ``block_q4_0`` rows -> fp16 [N, K] (same RN16((q-8)*d) rule)."""
    n = blocks.shape[0]
    nb = k // QK4_0
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(n, nb, 18)
    d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)  # [n, nb, 1]
    qs = b[:, :, 2:18]
    nib = np.concatenate([qs & 0x0F, qs >> 4], axis=2).astype(np.float32) - np.float32(8.0)
    return (nib * d).reshape(n, k).astype(np.float16)


# --------------------------------------------------------------------------
# Q4_K (llama.cpp block_q4_K, 144 bytes per 256 values)
# --------------------------------------------------------------------------
def unpack_q4k_scales(s12: np.ndarray):
    """12 packed bytes -> (sc[8], m[8]) 6-bit values.

    Format as published in gguf-py 0.19.0 ``Q4_K.get_scale_min``: for j < 4,
    ``sc = s[j] & 63, m = s[j+4] & 63``; for j >= 4,
    ``sc = (s[j+4] & 15) | ((s[j-4] >> 6) << 4)`` and
    ``m = (s[j+4] >> 4) | ((s[j] >> 6) << 4)``.
    Works on any leading shape ``[..., 12]``.
    """
    s = np.asarray(s12, dtype=np.uint8)
    sc = np.empty(s.shape[:-1] + (8,), dtype=np.uint8)
    m = np.empty_like(sc)
    sc[..., 0:4] = s[..., 0:4] & 63
    m[..., 0:4] = s[..., 4:8] & 63
    sc[..., 4:8] = (s[..., 8:12] & 15) | ((s[..., 0:4] >> 6) << 4)
    m[..., 4:8] = (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 6) << 4)
    return sc, m


def pack_q4k_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """Inverse of :func:`unpack_q4k_scales` for 6-bit inputs ``[..., 8]``."""
    sc = np.asarray(sc, dtype=np.uint8)
    m = np.asarray(m, dtype=np.uint8)
    assert int(sc.max(initial=0)) < 64 and int(m.max(initial=0)) < 64
    s = np.zeros(sc.shape[:-1] + (12,), dtype=np.uint8)
    s[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = (m[..., 0:4] & 63) | ((m[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 15) | ((m[..., 4:8] & 15) << 4)
    return s


def make_q4k_blocks(d16, dmin16, sc, m, q) -> np.ndarray:
    """Assemble ``block_q4_K`` rows.

    d16, dmin16: fp16 [N, S]; sc, m: u8 [N, S, 8] (6-bit); q: u8 [N, S*256]
    nibbles in element order. Returns u8 [N, S*144]. Within a super-block the
    128 ``qs`` bytes form four 32-byte chunks; byte l of chunk c holds element
    64c+l (sub-block 2c) in its low nibble and 64c+32+l (sub-block 2c+1) in its
    high nibble.
    """
    d16 = np.asarray(d16, dtype=np.float16)
    n, s = d16.shape
    q = np.asarray(q, dtype=np.uint8).reshape(n, s, 4, 2, 32)
    qs = (q[:, :, :, 0, :] | (q[:, :, :, 1, :] << 4)).reshape(n, s, 128)
    hdr_d = d16.reshape(n, s, 1).view(np.uint8)
    hdr_m = np.asarray(dmin16, dtype=np.float16).reshape(n, s, 1).view(np.uint8)
    scales = pack_q4k_scales(sc, m)
    return np.concatenate([hdr_d, hdr_m, scales, qs], axis=2).reshape(n, s * Q4K_BLOCK_BYTES)


def split_q4k_blocks(blocks: np.ndarray, k: int):
    """``block_q4_K`` rows -> (d16 [N,S], dmin16 [N,S], sc [N,S,8], m [N,S,8], q [N,K])."""
    n = blocks.shape[0]
    s = k // QK_K
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(n, s, Q4K_BLOCK_BYTES)
    d16 = b[:, :, 0:2].copy().view(np.float16).reshape(n, s)
    dmin16 = b[:, :, 2:4].copy().view(np.float16).reshape(n, s)
    sc, m = unpack_q4k_scales(b[:, :, 4:16])
    qs = b[:, :, 16:144].reshape(n, s, 4, 1, 32)
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=3).reshape(n, s * QK_K)
    return d16, dmin16, sc, m, q


def dequant_q4k_f32(blocks: np.ndarray, k: int) -> np.ndarray:
    """Q4_K dequant in fp32 (gguf-py 0.19.0 ``Q4_K.dequantize_blocks`` order).

    ``d1 = fp32(d) * sc`` and ``m1 = fp32(dmin) * m`` are exact in fp32
    (11-bit by 6-bit significands); ``d1 * q`` is exact too, so
    ``w32 = d1 * q - m1`` carries exactly one fp32 rounding whether or not the
    multiply and subtract are fused.
    """
    d16, dmin16, sc, m, q = split_q4k_blocks(blocks, k)
    n, s = d16.shape
    d1 = (d16.astype(np.float32)[:, :, None] * sc.astype(np.float32))   # [n, s, 8]
    m1 = (dmin16.astype(np.float32)[:, :, None] * m.astype(np.float32))
    qf = q.reshape(n, s, 8, 32).astype(np.float32)
    w32 = d1[:, :, :, None] * qf - m1[:, :, :, None]
    return w32.reshape(n, k).astype(np.float32)


def dequant_q4k(blocks: np.ndarray, k: int) -> np.ndarray:
    """Bit-exact Q4_K fp16 operand: ``fp16_rn(w32)``."""
    return dequant_q4k_f32(blocks, k).astype(np.float16)


# --------------------------------------------------------------------------
# Q5_K (llama.cpp block_q5_K, 176 bytes per 256 values)
# --------------------------------------------------------------------------
def make_q5k_blocks(d16, dmin16, sc, m, q) -> np.ndarray:
    """Assemble ``block_q5_K`` rows: fp16 d, fp16 dmin, the 12 scale/min
    bytes of Q4_K, 32 bytes ``qh`` and 128 bytes ``qs``.

    q: u8 [N, S*256] 5-bit values in element order. Element e of a
    super-block (sub-block G = e // 32, l = e % 32) keeps its low 4 bits in
    ``qs[32*(G//2) + l]`` (low nibble for even G, high nibble for odd G) and
    its fifth bit as bit G of ``qh[l]`` (gguf-py 0.19.0 ``Q5_K``).
    """
    d16 = np.asarray(d16, dtype=np.float16)
    n, s = d16.shape
    q = np.asarray(q, dtype=np.uint8).reshape(n, s, 8, 32)
    lo = q & 0x0F
    qs = (lo[:, :, 0::2, :] | (lo[:, :, 1::2, :] << 4)).reshape(n, s, 128)
    hi = (q >> 4) & 1                                     # [n, s, 8, 32]
    qh = np.zeros((n, s, 32), dtype=np.uint8)
    for g in range(8):
        qh |= (hi[:, :, g, :] << g).astype(np.uint8)
    hdr_d = d16.reshape(n, s, 1).view(np.uint8)
    hdr_m = np.asarray(dmin16, dtype=np.float16).reshape(n, s, 1).view(np.uint8)
    return np.concatenate([hdr_d, hdr_m, pack_q4k_scales(sc, m), qh, qs], axis=2).reshape(n, s * Q5K_BLOCK_BYTES)


def split_q5k_blocks(blocks: np.ndarray, k: int):
    """``block_q5_K`` rows -> (d16 [N,S], dmin16 [N,S], sc [N,S,8], m [N,S,8], q [N,K] in 0..31)."""
    n = blocks.shape[0]
    s = k // QK_K
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(n, s, Q5K_BLOCK_BYTES)
    d16 = b[:, :, 0:2].copy().view(np.float16).reshape(n, s)
    dmin16 = b[:, :, 2:4].copy().view(np.float16).reshape(n, s)
    sc, m = unpack_q4k_scales(b[:, :, 4:16])
    qh = b[:, :, 16:48]
    qs = b[:, :, 48:176].reshape(n, s, 4, 1, 32)
    lo = np.concatenate([qs & 0x0F, qs >> 4], axis=3).reshape(n, s, 8, 32)
    hi = np.stack([(qh >> g) & 1 for g in range(8)], axis=2)   # [n, s, 8, 32]
    q = (lo | (hi << 4)).reshape(n, s * QK_K)
    return d16, dmin16, sc, m, q


def dequant_q5k_f32(blocks: np.ndarray, k: int) -> np.ndarray:
    """Q5_K dequant in fp32 (gguf-py 0.19.0 ``Q5_K.dequantize_blocks`` order):
    ``fp32(d) * sc * q - fp32(dmin) * m``, one fp32 rounding (as Q4_K)."""
    d16, dmin16, sc, m, q = split_q5k_blocks(blocks, k)
    n, s = d16.shape
    d1 = (d16.astype(np.float32)[:, :, None] * sc.astype(np.float32))
    m1 = (dmin16.astype(np.float32)[:, :, None] * m.astype(np.float32))
    qf = q.reshape(n, s, 8, 32).astype(np.float32)
    return (d1[:, :, :, None] * qf - m1[:, :, :, None]).reshape(n, k).astype(np.float32)


def dequant_q5k(blocks: np.ndarray, k: int) -> np.ndarray:
    """Bit-exact Q5_K fp16 operand: ``fp16_rn(w32)``."""
    return dequant_q5k_f32(blocks, k).astype(np.float16)


# --------------------------------------------------------------------------
# Q6_K (llama.cpp block_q6_K, 210 bytes per 256 values)
# --------------------------------------------------------------------------
def make_q6k_blocks(d16, sc, q) -> np.ndarray:
    """Assemble ``block_q6_K`` rows: 128 bytes ``ql``, 64 bytes ``qh``, 16
    int8 sub-block scales, fp16 d (gguf-py 0.19.0 ``Q6_K`` layout).

    q: u8 [N, S*256] 6-bit values in element order. Element e of a block
    (half h = e // 128, group j = (e % 128) // 32, l = e % 32) keeps its low 4
    bits in ``ql[64h + 32(j % 2) + l]`` (low nibble for j < 2, high nibble for
    j >= 2) and its top 2 bits in bits 2j, 2j+1 of ``qh[32h + l]``; scale
    ``sc[e // 16]`` (int8) multiplies it.
    """
    d16 = np.asarray(d16, dtype=np.float16)
    n, s = d16.shape
    q = np.asarray(q, dtype=np.uint8).reshape(n, s, 2, 4, 32)
    lo = q & 0x0F
    ql = np.concatenate([lo[:, :, :, 0] | (lo[:, :, :, 2] << 4), lo[:, :, :, 1] | (lo[:, :, :, 3] << 4)],
                        axis=3).reshape(n, s, 128)
    hi = (q >> 4) & 3
    qh = (hi[:, :, :, 0] | (hi[:, :, :, 1] << 2) | (hi[:, :, :, 2] << 4) | (hi[:, :, :, 3] << 6)).reshape(n, s, 64)
    scb = np.asarray(sc, dtype=np.int8).reshape(n, s, 16).view(np.uint8)
    hdr_d = d16.reshape(n, s, 1).view(np.uint8)
    return np.concatenate([ql, qh.astype(np.uint8), scb, hdr_d], axis=2).reshape(n, s * Q6K_BLOCK_BYTES)


def split_q6k_blocks(blocks: np.ndarray, k: int):
    """``block_q6_K`` rows -> (d16 [N,S], sc int8 [N,S,16], q [N,K] in 0..63)."""
    n = blocks.shape[0]
    s = k // QK_K
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(n, s, Q6K_BLOCK_BYTES)
    ql = b[:, :, 0:128].reshape(n, s, 2, 2, 32)          # [h][j % 2][l]
    qh = b[:, :, 128:192].reshape(n, s, 2, 32)           # [h][l]
    sc = b[:, :, 192:208].copy().view(np.int8)
    d16 = b[:, :, 208:210].copy().view(np.float16).reshape(n, s)
    lo = np.stack([ql[:, :, :, 0] & 0x0F, ql[:, :, :, 1] & 0x0F, ql[:, :, :, 0] >> 4, ql[:, :, :, 1] >> 4], axis=2)
    hi = np.stack([(qh >> (2 * j)) & 3 for j in range(4)], axis=2)   # [n, s, 4(j), 2(h), 32]
    q = (lo | (hi << 4)).transpose(0, 1, 3, 2, 4).reshape(n, s * QK_K)
    return d16, sc, q


def dequant_q6k_f32(blocks: np.ndarray, k: int) -> np.ndarray:
    """Q6_K dequant in fp32 (gguf-py 0.19.0 ``Q6_K.dequantize_blocks`` order):
    ``(fp32(d) * sc) * (q - 32)``; ``d * sc`` is exact (19 bits), the product
    rounds once."""
    d16, sc, q = split_q6k_blocks(blocks, k)
    n, s = d16.shape
    ds = d16.astype(np.float32)[:, :, None] * sc.astype(np.float32)          # [n, s, 16]
    qf = (q.astype(np.int16) - 32).astype(np.float32).reshape(n, s, 16, 16)
    return (ds[:, :, :, None] * qf).reshape(n, k).astype(np.float32)


def dequant_q6k(blocks: np.ndarray, k: int) -> np.ndarray:
    """Bit-exact Q6_K fp16 operand: ``fp16_rn(w32)``."""
    return dequant_q6k_f32(blocks, k).astype(np.float16)


def repack_q6k(blocks: np.ndarray, k: int):
    """The device layout ``busfill_repack_q6k`` writes: every block's first
    208 bytes (``ql``, ``qh``, scales) as rows u8 [N, S*208], and the blocks'
    fp16 d as a plane [S, N] (block-major), so that both have row strides of
    whole 16-byte multiples (the tensor-memory-access copy rule; 210-byte
    rows have none unless K is a multiple of 2048)."""
    n = blocks.shape[0]
    s = k // QK_K
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(n, s, Q6K_BLOCK_BYTES)
    qb = b[:, :, :Q6K_PACKED_BYTES].reshape(n, s * Q6K_PACKED_BYTES).copy()
    d = b[:, :, Q6K_PACKED_BYTES:].copy().view(np.float16).reshape(n, s).T.copy()
    return qb, d


def unpack_q6k(qb: np.ndarray, d: np.ndarray, k: int) -> np.ndarray:
    """Inverse of repack_q6k: ``block_q6_K`` rows u8 [N, S*210]."""
    n = qb.shape[0]
    s = k // QK_K
    body = np.ascontiguousarray(qb, dtype=np.uint8).reshape(n, s, Q6K_PACKED_BYTES)
    hdr = np.ascontiguousarray(np.asarray(d, dtype=np.float16).T).reshape(n, s, 1).view(np.uint8)
    return np.concatenate([body, hdr], axis=2).reshape(n, s * Q6K_BLOCK_BYTES)


# --------------------------------------------------------------------------
# Seeded synthetic generators (no public dataset)
# --------------------------------------------------------------------------
def gen_activations(m: int, k: int, seed: int) -> np.ndarray:
    """fp16 N(0,1) activations [M, K]."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)


def gen_q4_0(n: int, k: int, seed: int, dlo: float = 0.001, dhi: float = 0.02):
    """Config 0/1 weights: d ~ U(0.001, 0.02) fp16, nibbles uniform [0, 15].

    Returns (Wq [N, K/2] u8, Ws [N, K/32] fp16).
    """
    rng = np.random.default_rng(seed)
    ws = rng.uniform(dlo, dhi, size=(n, k // QK4_0)).astype(np.float16)
    wq = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    return wq, ws


def gen_q4k(n: int, k: int, seed: int):
    """Config 2-4 weights: d ~ U(0.001, 0.01), dmin ~ U(0, 0.005) (fp16),
    6-bit scales and mins uniform [0, 63], nibbles uniform [0, 15].

    Returns ``block_q4_K`` rows u8 [N, K/256*144].
    """
    assert k % QK_K == 0
    rng = np.random.default_rng(seed)
    s = k // QK_K
    d16 = rng.uniform(0.001, 0.01, size=(n, s)).astype(np.float16)
    dmin16 = rng.uniform(0.0, 0.005, size=(n, s)).astype(np.float16)
    sc = rng.integers(0, 64, size=(n, s, 8), dtype=np.uint8)
    m = rng.integers(0, 64, size=(n, s, 8), dtype=np.uint8)
    q = rng.integers(0, 16, size=(n, k), dtype=np.uint8)
    return make_q4k_blocks(d16, dmin16, sc, m, q)


def gen_q5k(n: int, k: int, seed: int):
    """Q5_K weights with the config-2 scale distributions (d ~ U(0.001, 0.01),
    dmin ~ U(0, 0.005), 6-bit scales and mins uniform) and 5-bit values
    uniform [0, 31]. Returns ``block_q5_K`` rows u8 [N, K/256*176]."""
    assert k % QK_K == 0
    rng = np.random.default_rng(seed)
    s = k // QK_K
    d16 = rng.uniform(0.001, 0.01, size=(n, s)).astype(np.float16)
    dmin16 = rng.uniform(0.0, 0.005, size=(n, s)).astype(np.float16)
    sc = rng.integers(0, 64, size=(n, s, 8), dtype=np.uint8)
    m = rng.integers(0, 64, size=(n, s, 8), dtype=np.uint8)
    q = rng.integers(0, 32, size=(n, k), dtype=np.uint8)
    return make_q5k_blocks(d16, dmin16, sc, m, q)


def gen_q6k(n: int, k: int, seed: int):
    """Q6_K weights: d ~ U(0.0001, 0.0005) fp16, int8 sub-block scales
    uniform [-128, 127], 6-bit values uniform [0, 63] (weights of the same
    order as config 2's). Returns ``block_q6_K`` rows u8 [N, K/256*210]."""
    assert k % QK_K == 0
    rng = np.random.default_rng(seed)
    s = k // QK_K
    d16 = rng.uniform(0.0001, 0.0005, size=(n, s)).astype(np.float16)
    sc = rng.integers(-128, 128, size=(n, s, 16)).astype(np.int8)
    q = rng.integers(0, 64, size=(n, k), dtype=np.uint8)
    return make_q6k_blocks(d16, sc, q)


# --------------------------------------------------------------------------
# GEMM reference and gates
# --------------------------------------------------------------------------
def gemm_ref(a16: np.ndarray, w: np.ndarray) -> np.ndarray:
    """fp32 matmul of fp16 activations with dequantized weights:
    ``A.float() @ W.float().T`` (kernels/q4k_batched.py:100). The reference
    gate passes its fp32 dequantized matrix (``ref``); fp16 operands work too."""
    return np.asarray(a16, np.float32) @ np.asarray(w, np.float32).T


GATE_MAX_ABS = 0.6      # kernels/q4k_batched.py:102
GATE_REL_L2 = 1e-3


def swiglu_ref(a16: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray) -> np.ndarray:
    """silu(A Wg^T) * (A Wu^T) in float64 on the given (dequantized) weights:
    the fused gate/up epilogue of a gated feed-forward layer, silu(x) =
    x / (1 + exp(-x))."""
    a = np.asarray(a16, dtype=np.float16).astype(np.float64)
    g = a @ np.asarray(w_gate, dtype=np.float64).T
    u = a @ np.asarray(w_up, dtype=np.float64).T
    return g / (1.0 + np.exp(-g)) * u


def gemm_errors(c, cref):
    """(max_abs_err, rel_l2, all_finite) of a GEMM output against the reference."""
    c = np.asarray(c, dtype=np.float64)
    cref = np.asarray(cref, dtype=np.float64)
    finite = bool(np.isfinite(c).all())
    if c.size == 0:
        return 0.0, 0.0, finite
    diff = c - cref
    max_abs = float(np.abs(diff).max()) if finite else float("inf")
    denom = float(np.linalg.norm(cref))
    rel = float(np.linalg.norm(diff) / denom) if denom > 0 else float(np.linalg.norm(diff))
    return max_abs, rel, finite


def gate_ok(c, cref) -> bool:
    """The GEMM gate: finite, max abs err <= 0.6 and rel-L2 <= 1e-3."""
    max_abs, rel, finite = gemm_errors(c, cref)
    return finite and max_abs <= GATE_MAX_ABS and rel <= GATE_REL_L2


def algorithmic_bytes(m: int, n: int, k: int) -> int:
    """Bytes a Q4 GEMM must move: 4.5-bit weights + fp16 A + fp16 C."""
    return n * k * 18 // 32 + 2 * m * k + 2 * m * n
