"""CPU-side checks of the C ABI and of the kernels' host/bit-level logic.

No GPU: the library is loaded and its exports and status strings checked; the
dequant instruction chains of busfill_b200/csrc/formats.cuh are emulated
bit for bit in numpy and compared with the oracle (the K formats' exact
chains against the gguf-py golden vectors too); the cluster K split
and tile assignment are checked to cover every unit exactly once.
"""
import ctypes
import os

import numpy as np
import pytest

import busfill_b200 as bf
from oracle import q4_oracle as orc


def test_library_loads_and_exports_every_header_function():
    names = bf.header_functions()
    assert len(names) >= 10
    lib = bf.load_library()
    for n in names:
        assert hasattr(lib, n), n
    raw = ctypes.CDLL(bf.library_path())
    for n in names:
        getattr(raw, n)  # raises AttributeError if not exported


def test_status_strings_and_version():
    lib = bf.load_library()
    assert bf.version() >= 100
    for code, name in bf.STATUS.items():
        s = lib.busfill_status_string(code)
        assert isinstance(s, bytes) and len(s) > 0
    assert lib.busfill_status_string(12345) == b"unknown status"


def test_set_option_rejects_unknown():
    lib = bf.load_library()
    assert lib.busfill_set_option(99, 1) == -1
    assert lib.busfill_set_option(1, 1) == 0
    assert lib.busfill_set_option(4, 2) == -1          # the exact option is 0 or 1
    assert lib.busfill_set_option(4, 1) == 0 and lib.busfill_set_option(4, 0) == 0


def test_null_pointer_rejected_before_any_device_work():
    lib = bf.load_library()
    # argument validation happens before the device is touched
    assert lib.busfill_gemm_q4k(None, None, None, 8, 128, 256, None) == -1
    assert lib.busfill_gemm_q4_0(None, None, None, None, 8, 128, 256, None) == -1
    assert lib.busfill_gemm_q4_0_ggml(None, None, None, 8, 128, 256, None) == -1
    assert lib.busfill_gemm_q4k_swiglu(None, None, None, None, 8, 128, 256, None) == -1
    assert lib.busfill_gemm_q5k(None, None, None, 8, 128, 256, None) == -1
    assert lib.busfill_dequant_q5k(None, None, 4, 256, None) == -1
    assert lib.busfill_gemm_q6k(None, None, None, None, 8, 128, 256, None) == -1
    assert lib.busfill_repack_q6k(None, None, None, 4, 256, None) == -1
    assert lib.busfill_dequant_q6k(None, None, None, 4, 256, None) == -1
    assert lib.busfill_dequant_q4k(None, None, 4, 256, None) == -1
    assert lib.busfill_probe_umma(None, None, None, 16, None) == -1


# ---------------------------------------------------------------------------
# bit-level emulation of the device dequant chains
# ---------------------------------------------------------------------------
def prmt(a, b, sel):
    a = np.asarray(a, dtype=np.uint64)
    b = np.asarray(b, dtype=np.uint64)
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = np.zeros_like(a)
    for i in range(4):
        idx = (sel >> (4 * i)) & 0x7
        out |= src[idx] << (8 * i)
    return out.astype(np.uint32)


def lop3_and_or(a, b, c):
    return ((np.asarray(a, np.uint32) & np.uint32(b)) | np.uint32(c)).astype(np.uint32)


def h2(u):
    """uint32 -> (lo, hi) float16 halves."""
    u = np.asarray(u, dtype=np.uint32)
    return (u & 0xFFFF).astype(np.uint16).view(np.float16), (u >> 16).astype(np.uint16).view(np.float16)


def rn16(x64):
    return np.asarray(x64, dtype=np.float64).astype(np.float16)


def hfma(x, y, z):
    return rn16(np.float64(x) * np.float64(y) + np.float64(z))


@pytest.mark.filterwarnings("ignore:overflow encountered")
def test_q4_0_block_chain_matches_reference_dequant_for_all_fp16_scales():
    # kernel: t = prmt(w, w>>4, ((4+x)<<8)|x); v = lop3(t & 0x000F000F | 0x64006400);
    #         out = hmul2(hsub2(v, 1032), d)  ==  fp16_rn((q-8)*d)  (busfill_v0.cu:74-81)
    d_bits = np.arange(0, 0x7C00, dtype=np.uint32)          # every finite non-negative fp16
    d_bits = np.concatenate([d_bits, d_bits | 0x8000])       # and negative
    d = d_bits.astype(np.uint16).view(np.float16)
    for byte in range(256):
        w = np.full(d.shape, byte * 0x01010101, dtype=np.uint32)
        for x in range(4):
            t = prmt(w, w >> np.uint32(4), ((4 + x) << 8) | x)
            v = lop3_and_or(t, 0x000F000F, 0x64006400)
            lo, hi = h2(v)
            assert np.all(lo.astype(np.float64) == 1024 + (byte & 15))
            assert np.all(hi.astype(np.float64) == 1024 + (byte >> 4))
        q_lo, q_hi = byte & 15, byte >> 4
        got_lo = rn16((np.float16(1024 + q_lo) - np.float16(1032)).astype(np.float64) * d.astype(np.float64))
        want_lo = (np.float32(q_lo - 8) * d.astype(np.float32)).astype(np.float16)
        assert np.array_equal(got_lo.view(np.uint16), want_lo.view(np.uint16))
        got_hi = rn16((np.float16(1024 + q_hi) - np.float16(1032)).astype(np.float64) * d.astype(np.float64))
        want_hi = (np.float32(q_hi - 8) * d.astype(np.float32)).astype(np.float16)
        assert np.array_equal(got_hi.view(np.uint16), want_hi.view(np.uint16))


def test_q4_0_block_chain_column_order_is_natural():
    rng = np.random.default_rng(0)
    blk = rng.integers(0, 256, size=16, dtype=np.uint8)
    words = blk.view(np.uint32)
    cols = []
    for i in range(4):
        w = np.uint32(words[i])
        for x in range(4):
            t = prmt(w, w >> np.uint32(4), ((4 + x) << 8) | x)
            lo, hi = h2(lop3_and_or(t, 0x000F000F, 0x64006400))
            cols.append((float(lo) - 1024, float(hi) - 1024))
    nib = orc.unpack_q4_0_planes(blk.reshape(1, 16))[0]
    # column c holds elements (2c, 2c+1)
    assert [v for pair in cols for v in pair] == [float(v) for v in nib]


def test_q4k_nibble_bias_is_exact():
    # low nibble: (b & 0x0F) | 0x6400 == 1024 + q (mantissa step 1);
    # high nibble: (b & 0xF0) | 0x5400 == 64 + q (0x5400 = 64.0, mantissa step 1/16)
    for byte in range(256):
        lo = np.uint16((byte & 0x0F) | 0x6400).view(np.float16)
        hi = np.uint16((byte & 0xF0) | 0x5400).view(np.float16)
        assert float(lo) == 1024 + (byte & 15)
        assert float(hi) == 64 + (byte >> 4)
        assert float(np.float16(float(lo) - 1024)) == byte & 15   # hsub2 exact
        assert float(np.float16(float(hi) - 64)) == byte >> 4


def fma_f16_f32(a16, b16, c32):
    """fma.rn.f32.f16: fp16 a times fp16 b plus fp32 c, rounded once to fp32.
    The product is exact in float64 (at most 22 significant bits); the sum is
    checked to be exact in float64 too (TwoSum error 0), so rounding it to
    float32 once models the device instruction exactly."""
    p = np.asarray(a16, np.float16).astype(np.float64) * np.asarray(b16, np.float16).astype(np.float64)
    c = np.asarray(c32, np.float32).astype(np.float64)
    s = p + c
    bb = s - p
    err = (p - (s - bb)) + (c - bb)
    assert np.all(err == 0)
    return s.astype(np.float32)


def k_exact_operand(d16, dmin16, sc, m, q, bias):
    """Bit-level model of k_exact_pair (formats.cuh): the fp16 word bias + q
    (exact), hfma2(bias + q, sc, -bias*sc) = q*sc (checked exact), the mixed
    fma q*sc*d - m1 rounded once to fp32, then fp16_rn."""
    q = np.asarray(q, np.int64)
    sc = np.asarray(sc, np.int64)
    biased = (bias + q).astype(np.float16)
    assert np.all(biased.astype(np.int64) == bias + q)
    nbsc = (-bias * sc).astype(np.float16)
    assert np.all(nbsc.astype(np.int64) == -bias * sc)
    qs = hfma(biased, sc.astype(np.float16), nbsc)
    assert np.all(qs.astype(np.int64) == q * sc)
    nm1 = -(np.asarray(dmin16, np.float16).astype(np.float32) * np.asarray(m, np.float32))
    return fma_f16_f32(qs, d16, nm1).astype(np.float16)


def q4k_model(blocks, k):
    d16, dmin16, sc, m, q = orc.split_q4k_blocks(blocks, k)
    n, s = d16.shape
    qf = q.reshape(n, s, 8, 32)
    # sub-blocks 2c (low nibbles, bias 1024) and 2c+1 (high nibbles, bias 64)
    bias = np.where(np.arange(8) % 2 == 0, 1024, 64)[None, None, :, None]
    w = k_exact_operand(d16[:, :, None, None], dmin16[:, :, None, None], sc[:, :, :, None], m[:, :, :, None], qf,
                        bias)
    return w.reshape(n, k)


def canon16(w):
    b = np.asarray(w, np.float16).view(np.uint16).copy()
    b[b == 0x8000] = 0
    return b


def test_q4k_exact_chain_steps_are_exact_for_every_nibble_and_scale():
    # every (q, sc) of both nibble positions: bias + q and q*sc exact in fp16
    q = np.arange(16)[:, None]
    sc = np.arange(64)[None, :]
    for bias in (1024, 64):
        k_exact_operand(np.float16(1.0), np.float16(0.0), sc, np.zeros_like(sc), q, bias)
    # Q5_K: 5-bit values under the bias 1024
    k_exact_operand(np.float16(1.0), np.float16(0.0), sc, np.zeros_like(sc), np.arange(32)[:, None], 1024)


def test_q4k_exact_chain_is_the_oracle():
    blocks = orc.gen_q4k(64, 2048, seed=7)
    assert np.array_equal(canon16(q4k_model(blocks, 2048)), canon16(orc.dequant_q4k(blocks, 2048)))


def test_q4k_exact_chain_on_golden_random_blocks(golden_dir):
    g = np.load(os.path.join(golden_dir, "q4k_gguf.npz"))
    for case in ("a", "b"):
        blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
        assert np.array_equal(canon16(q4k_model(blocks, k)), canon16(w32.astype(np.float16)))


def test_q5k_exact_chain_on_golden_random_blocks(golden_dir):
    g = np.load(os.path.join(golden_dir, "q5k_gguf.npz"))
    for case in ("a", "b"):
        blocks, w32, k = g[f"{case}_blocks"], g[f"{case}_w32"], int(g[f"{case}_k"])
        d16, dmin16, sc, m, q = orc.split_q5k_blocks(blocks, k)
        n, s = d16.shape
        w = k_exact_operand(d16[:, :, None, None], dmin16[:, :, None, None], sc[:, :, :, None], m[:, :, :, None],
                            q.reshape(n, s, 8, 32), 1024)
        assert np.array_equal(canon16(w.reshape(n, k)), canon16(w32.astype(np.float16)))


def test_q6k_shape_and_alignment_checked_before_any_device_work():
    lib = bf.load_library()
    fake = 0x10000                     # never dereferenced: the checks come first
    # the d plane [K/256][N] fp16 needs a 16-byte row stride: N % 8 == 0
    assert lib.busfill_gemm_q6k(fake, fake, fake, fake, 4, 100, 256, None) == -2
    assert lib.busfill_gemm_q6k(fake, fake, fake, fake, 4, 128, 300, None) == -2
    assert lib.busfill_gemm_q6k(fake + 8, fake, fake, fake, 4, 128, 256, None) == -3
    assert lib.busfill_repack_q6k(fake + 1, fake, fake, 4, 256, None) == -3
    assert lib.busfill_repack_q6k(fake, fake, fake, 4, 100, None) == -2


def test_q5k_chunk_chain_values_and_order():
    """Bit-level model of dequant_q5k_chunk<cc> (formats.cuh): each byte made
    the 5-bit value, then set under the fp16 exponent byte 0x64 by a
    byte-permute; hsub2 by 1024 leaves the exact integer q."""
    blocks = orc.gen_q5k(4, 512, seed=12)
    _, _, _, _, q = orc.split_q5k_blocks(blocks, 512)
    b = blocks.reshape(4, 2, 176)
    for r in range(4):
        for blk in range(2):
            row = b[r, blk]
            hw = row[16:48].copy().view(np.uint32)
            for cc in range(4):
                w = row[48 + 32 * cc: 80 + 32 * cc].copy().view(np.uint32)
                lo, hi = [], []
                for i in range(8):
                    def fifth(bit):
                        x = int(hw[i])
                        return ((x << (4 - bit)) & 0xFFFFFFFF if bit <= 4 else x >> (bit - 4)) & 0x10101010
                    ql = (int(w[i]) & 0x0F0F0F0F) | fifth(2 * cc)
                    qh = ((int(w[i]) >> 4) & 0x0F0F0F0F) | fifth(2 * cc + 1)
                    for src, dst in ((ql, lo), (qh, hi)):
                        for sel in (0x4140, 0x4342):
                            for half in h2(prmt(src, 0x64, sel)):
                                dst.append(float(np.float16(np.float64(half) - 1024.0)))
                e0 = 256 * blk + 64 * cc
                assert lo + hi == [float(v) for v in q[r, e0: e0 + 64]]


def q6k_chunk_chain(body, d16, cc):
    """Bit-level model of dequant_q6k_chunk<cc % 2> (formats.cuh) on one
    208-byte block body: returns the chunk's 64 exact integers q - 32 (from
    the biased fp16 words) and its 64 fp16 operands, in column order. The
    mixed fma (1024 + q) d - 1056 d gives (q - 32) d exactly; the product
    with the group's int8 scale is exact in fp32 (checked); one rounding to
    fp16 follows."""
    h, odd = cc >> 1, cc & 1
    ql = body[64 * h: 64 * h + 64].copy().view(np.uint32)
    qh = body[128 + 32 * h: 128 + 32 * h + 32].copy().view(np.uint32)
    sc = body[192 + 4 * cc: 196 + 4 * cc].copy().view(np.int8)
    nd1056 = np.float32(-1056.0) * np.float32(d16)
    ints, vals = [], []
    for jj in range(2):
        s = 4 * odd + 2 * jj
        for i in range(8):
            w = int(qh[i])
            hq = ((w << (4 - s)) & 0xFFFFFFFF) if s <= 4 else (w >> (s - 4))
            q4 = ((int(ql[8 * jj + i]) >> (4 * odd)) & 0x0F0F0F0F) | (hq & 0x30303030)
            for sel in (0x4140, 0x4342):
                for half in h2(prmt(q4, 0x64, sel)):
                    t = fma_f16_f32(half, d16, nd1056)                 # (q - 32) d, exact
                    ints.append(float(half) - 1056.0)
                    assert float(t) == ints[-1] * float(d16)
                    scale = np.float32(sc[2 * jj + i // 4])
                    v = np.float32(t) * scale
                    assert float(v) == float(t) * float(scale)        # exact: <= 23 significant bits
                    vals.append(np.float16(v))
    return ints, np.array(vals, dtype=np.float16)


def test_q6k_chunk_chain_order_and_exactness():
    blocks = orc.gen_q6k(6, 512, seed=11)
    d16, sc, q = orc.split_q6k_blocks(blocks, 512)
    body, dplane = orc.repack_q6k(blocks, 512)
    want16 = orc.dequant_q6k(blocks, 512)
    for r in range(6):
        for b in range(2):
            blk = body[r, 208 * b: 208 * (b + 1)]
            for cc in range(4):
                ints, vals = q6k_chunk_chain(blk, dplane[b, r], cc)
                e0 = 256 * b + 64 * cc
                assert ints == [float(v) - 32 for v in q[r, e0: e0 + 64]]
                assert np.array_equal(canon16(vals), canon16(want16[r, e0: e0 + 64]))


def test_q6k_chunk_chain_on_golden_random_blocks(golden_dir):
    g = np.load(os.path.join(golden_dir, "q6k_gguf.npz"))
    blocks, w32, k = g["b_blocks"], g["b_w32"], int(g["b_k"])
    body, dplane = orc.repack_q6k(blocks, k)
    want16 = w32.astype(np.float16)
    for r in range(0, blocks.shape[0], 5):
        for b in range(k // 256):
            blk = body[r, 208 * b: 208 * (b + 1)]
            for cc in range(4):
                _, vals = q6k_chunk_chain(blk, dplane[b, r], cc)
                e0 = 256 * b + 64 * cc
                assert np.array_equal(canon16(vals), canon16(want16[r, e0: e0 + 64]))


def test_q4k_chunk_extraction_and_order():
    rng = np.random.default_rng(1)
    chunk = rng.integers(0, 256, size=32, dtype=np.uint8)
    words = chunk.view(np.uint32)
    lo_cols, hi_cols = [], []
    for i in range(8):
        w = np.uint32(words[i])
        t0 = prmt(w, w, 0x0100)
        t1 = prmt(w, w, 0x0302)
        for t in (t0, t1):
            a, b = h2(lop3_and_or(t, 0x000F000F, 0x64006400))
            lo_cols += [float(a) - 1024, float(b) - 1024]
            a, b = h2(lop3_and_or(t, 0x00F000F0, 0x54005400))
            hi_cols += [float(a) - 64, float(b) - 64]
    assert lo_cols == [float(v & 15) for v in chunk]      # sub-block 2c, elements 0..31
    assert hi_cols == [float(v >> 4) for v in chunk]      # sub-block 2c+1


def test_q4k_scale_words_match_oracle_unpack():
    rng = np.random.default_rng(2)
    s = rng.integers(0, 256, size=(4096, 12), dtype=np.uint8)
    y = s[:, 0:4].copy().view(np.uint32)[:, 0]
    z = s[:, 4:8].copy().view(np.uint32)[:, 0]
    w = s[:, 8:12].copy().view(np.uint32)[:, 0]
    sc_lo = y & 0x3F3F3F3F
    m_lo = z & 0x3F3F3F3F
    sc_hi = (w & 0x0F0F0F0F) | ((y >> 2) & 0x30303030)
    m_hi = ((w >> 4) & 0x0F0F0F0F) | ((z >> 2) & 0x30303030)
    sc, m = orc.unpack_q4k_scales(s)
    for j in range(8):
        word_sc = sc_lo if j < 4 else sc_hi
        word_m = m_lo if j < 4 else m_hi
        assert np.array_equal((word_sc >> (8 * (j % 4))) & 0xFF, sc[:, j])
        assert np.array_equal((word_m >> (8 * (j % 4))) & 0xFF, m[:, j])
    # the dequant warp of group grp reads bytes 2grp, 2grp+1 of the _lo words for
    # chunk grp and of the _hi words for chunk grp + 2 (sub-blocks 2cc, 2cc+1)
    for grp in range(2):
        for k2 in range(2):
            cc = grp + 2 * k2
            word_sc = sc_hi if k2 else sc_lo
            word_m = m_hi if k2 else m_lo
            sh = 16 * grp
            assert np.array_equal((word_sc >> sh) & 0xFF, sc[:, 2 * cc])
            assert np.array_equal((word_sc >> (sh + 8)) & 0xFF, sc[:, 2 * cc + 1])
            assert np.array_equal((word_m >> sh) & 0xFF, m[:, 2 * cc])
            assert np.array_equal((word_m >> (sh + 8)) & 0xFF, m[:, 2 * cc + 1])


# ---------------------------------------------------------------------------
# cluster K split and tile assignment (decode_gemm.cuh: ksplit_begin, unit_info)
# ---------------------------------------------------------------------------
def ksplit_begin(rank, S, c):
    return rank * S // c


def unit_info(i, length, sb0, g, nclusters):
    seg = i // length
    j = i - seg * length
    return g + seg * nclusters, sb0 + j, seg, j == 0, j == length - 1


@pytest.mark.parametrize("S", [1, 2, 3, 7, 20, 32, 64, 68, 160])
@pytest.mark.parametrize("T", [1, 3, 40, 136, 300])
def test_cluster_schedule_covers_every_unit_once(S, T):
    for c in range(1, min(8, S) + 1):
        for ncl in sorted({1, min(T, 148 // c), min(T, 7)}):
            seen = np.zeros((T, S), dtype=np.int64)
            for g in range(ncl):
                ntiles = (T - g + ncl - 1) // ncl
                for rank in range(c):
                    sb0 = ksplit_begin(rank, S, c)
                    length = ksplit_begin(rank + 1, S, c) - sb0
                    assert length >= 1  # no idle rank when c <= S
                    for i in range(ntiles * length):
                        tile, sb, seg, first, last = unit_info(i, length, sb0, g, ncl)
                        assert tile % ncl == g and seg == (tile - g) // ncl
                        assert first == (sb == sb0) and last == (sb == sb0 + length - 1)
                        seen[tile, sb] += 1
            assert (seen == 1).all()


def test_ksplit_option_values():
    lib = bf.load_library()
    for v in range(0, 9):
        assert lib.busfill_set_option(2, v) == 0
    assert lib.busfill_set_option(2, 9) == -1
    assert lib.busfill_set_option(2, -1) == -1
    assert lib.busfill_set_option(2, 0) == 0


def test_prefill_batch_tile_option_values():
    lib = bf.load_library()
    for v in (0, 128, 256):
        assert lib.busfill_set_option(5, v) == 0
    for v in (-1, 1, 64, 192, 512):
        assert lib.busfill_set_option(5, v) == -1
    assert lib.busfill_set_option(5, 0) == 0


def test_prefill_pair_option_values():
    lib = bf.load_library()
    for v in (0, 1, 2):
        assert lib.busfill_set_option(6, v) == 0
    for v in (-1, 3):
        assert lib.busfill_set_option(6, v) == -1
    assert lib.busfill_set_option(6, 0) == 0


def test_sweep_unmet_dep_option_values():
    lib = bf.load_library()
    for v in (0, 1, 0):
        assert lib.busfill_set_option(8, v) == 0
    for v in (-1, 2):
        assert lib.busfill_set_option(8, v) == -1


def test_sweep_ctas_option_values():
    lib = bf.load_library()
    for v in (0, 1, 120, 148, 4096):
        assert lib.busfill_set_option(7, v) == 0
    assert lib.busfill_set_option(7, -1) == -1
    assert lib.busfill_set_option(7, 4097) == -1
    assert lib.busfill_set_option(7, 0) == 0


def test_kernel_choice_by_shape():
    """Default dispatch of the plain GEMMs: the stream-K prefill kernel for
    M > 64, and for M > 32 when N <= K and K >= 12288; the decode kernel
    otherwise. The option forces a plain M threshold and 0 restores the
    default."""
    bf.load_library()
    assert not bf.uses_prefill(32, 5120, 5120)
    assert not bf.uses_prefill(64, 17408, 5120)   # many decode tiles: one 64-row launch wins
    assert not bf.uses_prefill(33, 5120, 5120) and not bf.uses_prefill(64, 5120, 8192)
    assert bf.uses_prefill(33, 5120, 17408) and bf.uses_prefill(64, 5120, 17408)   # long K: stream-K wins
    assert bf.uses_prefill(65, 17408, 5120)       # from three decode launches on
    assert bf.uses_prefill(128, 5120, 17408) and bf.uses_prefill(128, 17408, 5120)
    assert bf.uses_prefill(512, 5120, 5120) and bf.uses_prefill(2048, 5120, 17408)
    bf.set_prefill_min_m(1)
    try:
        assert bf.uses_prefill(1, 128, 256)
    finally:
        bf.set_prefill_min_m(0)
    assert not bf.uses_prefill(1, 128, 256)


# ---------------------------------------------------------------------------
# stream-K partition of the prefill kernel (prefill_gemm.cuh), restated
# ---------------------------------------------------------------------------
def _first_unit(t, c, g):
    return t * c // g


def _cta_of_unit(t, x, g):
    return ((x + 1) * g - 1) // t


@pytest.mark.parametrize("items,s,g", [(20, 68, 148), (80, 68, 148), (1088, 20, 148), (3, 2, 5), (1, 1, 1),
                                       (7, 3, 21), (68, 20, 148), (2, 20, 40), (5, 1, 5)])
def test_stream_k_partition_covers_every_unit_once(items, s, g):
    t = items * s
    g = min(g, t)
    covered = np.zeros(t, dtype=np.int32)
    slots = {}          # (cta, item) -> slot of a partial piece
    for c in range(g):
        g0, g1 = _first_unit(t, c, g), _first_unit(t, c + 1, g)
        assert g1 > g0                                    # every CTA has work
        covered[g0:g1] += 1
        for x in (g0, g1 - 1):
            assert _cta_of_unit(t, x, g) == c
        pieces = list(range(g0 // s, (g1 - 1) // s + 1))
        for j, it in enumerate(pieces):
            whole = it * s >= g0 and (it + 1) * s <= g1
            if not whole:
                assert j in (0, len(pieces) - 1)          # only the first or last piece is partial
                slots[(c, it)] = 2 * c + (0 if j == 0 else 1)
    assert np.all(covered == 1)
    # the fix-up: one owner block per split item, summing exactly its CTAs' slots
    owned = {}
    for cb in range(1, g):
        gb = _first_unit(t, cb, g)
        if gb % s == 0:
            continue
        it = gb // s
        c_lo = _cta_of_unit(t, it * s, g)
        if c_lo != cb - 1:
            continue
        c_hi = _cta_of_unit(t, (it + 1) * s - 1, g)
        assert it not in owned
        owned[it] = [2 * cc + (0 if it == _first_unit(t, cc, g) // s else 1) for cc in range(c_lo, c_hi + 1)]
        # the fix-up kernel's shortcut: every CTA after c_lo holds the item as its first piece
        assert owned[it][1:] == [2 * cc for cc in range(c_lo + 1, c_hi + 1)]
        assert all(0 <= sl < 2 * g for sl in owned[it])
    split_items = {it for (_, it) in slots}
    assert set(owned) == split_items
    for it, sl in owned.items():
        assert sorted(sl) == sorted(v for (c, i), v in slots.items() if i == it)


# ---------------------------------------------------------------------------
# planar Q4_K and the ggml mul_mat call site (host-side checks)
# ---------------------------------------------------------------------------
def test_ggml_type_numbering_matches_gguf():
    gguf = pytest.importorskip("gguf")
    t = gguf.GGMLQuantizationType
    assert (int(t.F32), int(t.F16), int(t.Q4_0), int(t.Q4_K), int(t.Q5_K), int(t.Q6_K)) == (0, 1, 2, 12, 13, 14)
    assert (bf.TYPE_F16, bf.TYPE_Q4_0, bf.TYPE_Q4_K, bf.TYPE_Q5_K) == (1, 2, 12, 13)


class _FakeDev:
    """Stand-in for a device tensor: only its (never dereferenced) address."""

    def __init__(self, ptr):
        self.ptr = ptr

    def data_ptr(self):
        return self.ptr


def test_mul_mat_checks_before_any_device_work():
    lib = bf.load_library()
    fake = 0x10000
    w = bf.tensor_desc(_FakeDev(fake), bf.TYPE_Q4_K, [512, 256])
    x = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [512, 8])
    y = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [256, 8])
    call = lambda a, b, c: lib.busfill_mul_mat(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None)  # noqa: E731
    assert lib.busfill_mul_mat(None, None, None, None) == -1
    q6 = bf.tensor_desc(_FakeDev(fake), bf.TYPE_Q4_K, [512, 256])
    q6.type = 14                                     # Q6_K rows need busfill_repack_q6k first
    assert call(q6, x, y) == -1
    x32 = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [512, 8])
    x32.type = 0                                     # fp32 activations are not taken
    assert call(w, x32, y) == -1
    bad_k = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [256, 8])
    assert call(w, bad_k, y) == -2                   # K mismatch
    bad_n = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [128, 8])
    assert call(w, x, bad_n) == -2                   # N mismatch
    strided = bf.tensor_desc(_FakeDev(fake), bf.TYPE_Q4_K, [512, 256])
    strided.nb[1] += 16                              # padded rows are not taken
    assert call(strided, x, y) == -2
    wb = bf.tensor_desc(_FakeDev(fake), bf.TYPE_Q4_K, [512, 256, 2])
    xb = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [512, 8, 3])
    yb = bf.tensor_desc(_FakeDev(fake), bf.TYPE_F16, [256, 8, 3])
    assert call(wb, xb, yb) == -2                    # 3 batches do not broadcast over 2


def test_planar_q4k_checks_before_any_device_work():
    lib = bf.load_library()
    fake = 0x10000
    assert lib.busfill_repack_q4k_planar(None, None, None, None, None, 4, 256, None) == -1
    assert lib.busfill_repack_q4k_planar(fake, fake, fake, fake, fake, 4, 300, None) == -2
    assert lib.busfill_repack_q4k_planar(fake + 8, fake, fake, fake, fake, 4, 256, None) == -3
    assert lib.busfill_repack_q4k_planar(fake, fake + 1, fake, fake, fake, 4, 256, None) == -3
    assert lib.busfill_repack_q4k_planar(fake, fake, fake, fake + 2, fake, 4, 256, None) == -3
    assert lib.busfill_gemm_q4k_planar(fake, fake, fake, fake, None, fake, 8, 4, 256, None) == -1
    assert lib.busfill_gemm_q4k_planar(fake, fake, fake, fake, fake, fake, 0, 4, 256, None) == -2


def test_gathered_call_of_a_rank_without_rows_is_a_no_op():
    """A rank that owns no rows of a weight (fewer 128-row tiles than ranks)
    still makes the gathered call; it launches nothing, whatever its weight
    pointers, and so needs no device."""
    from busfill_b200 import tp
    lib = bf.load_library()
    fake = 0x10000
    g = tp.Gather()
    g.npeers, g.col_off, g.ldc = 4, 0, 384
    for q in range(4):
        g.out[q] = fake
        g.flag[q] = fake
    assert lib.busfill_gemm_q4k_gather(None, fake, 8, 0, 1280, ctypes.byref(g), None) == 0
    assert lib.busfill_gemm_q4k_swiglu_gather(None, None, fake, 8, 0, 1280, ctypes.byref(g), None) == 0
    assert lib.busfill_gemm_q4k_gather(None, fake, 8, -1, 1280, ctypes.byref(g), None) == -2


def test_gemm_launch_count_by_shape():
    """busfill_gemm_launches mirrors the dispatch: one decode launch per 64
    batch rows; the prefill kernel, plus its fix-up when the stream-K ranges
    over 148 SMs split a work item."""
    assert bf.gemm_launches(32, 5120, 5120, 148) == 1
    assert bf.gemm_launches(8, 5120, 5120, 148) == 1
    assert bf.gemm_launches(64, 17408, 5120, 148) == 1          # N > K: one 64-row decode launch
    assert bf.gemm_launches(48, 5120, 5120, 148) == 1           # K < 12288: one 64-row decode launch
    # M = 128, N = K = 5120: 20 pairs x 1 batch tile x 20 units over 148 CTAs splits items
    assert bf.gemm_launches(128, 5120, 5120, 148) == 2
    # 40 items x 20 units = 800 units over 40 CTAs: every range boundary on an item edge
    assert bf.gemm_launches(256, 5120, 5120, 40) == 1
    assert bf.gemm_launches(256, 5120, 5120, 100) == 2
    # CTA pairs: 136 items of 256 x 256 on 68 of the 74 pairs, whole items, no fix-up
    assert bf.gemm_launches(512, 17408, 5120, 148) == 1
    # 40 items of 68 units on 74 pairs: stream-K, split items summed by the fix-up
    assert bf.gemm_launches(512, 5120, 17408, 148) == 2
    assert bf.load_library().busfill_gemm_launches(8, 5120, 300, 148) == -2


# ---------------------------------------------------------------------------
# layer sweep (busfill_gemm_q4k_sweep)
# ---------------------------------------------------------------------------
def _sweep_ops(specs):
    arr = (bf.SweepOp * max(1, len(specs)))()
    buf = ctypes.create_string_buffer(64)
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    for i, (n, k, dep, up) in enumerate(specs):
        arr[i].w, arr[i].a, arr[i].c = base, base, base
        arr[i].w_up = base if up else None
        arr[i].N, arr[i].K, arr[i].dep = n, k, dep
    return arr, buf


def test_sweep_checks_before_any_device_work():
    lib = bf.load_library()
    ops, keep = _sweep_ops([(256, 512, -1, False), (512, 256, 0, True)])
    assert lib.busfill_gemm_q4k_sweep(None, 1, 8, None) == -1
    assert lib.busfill_gemm_q4k_sweep(ops, 0, 8, None) == -2          # no ops
    assert lib.busfill_gemm_q4k_sweep(ops, 9, 8, None) == -2          # more than BUSFILL_SWEEP_MAX_OPS
    assert lib.busfill_gemm_q4k_sweep(ops, 2, 0, None) == -2          # M < 1
    assert lib.busfill_gemm_q4k_sweep(ops, 2, 33, None) == -2         # M > 32
    bad, keep2 = _sweep_ops([(256, 512, 0, False)])                   # depends on itself
    assert lib.busfill_gemm_q4k_sweep(bad, 1, 8, None) == -1
    bad, keep3 = _sweep_ops([(256, 512, -1, False), (256, 512, 1, False)])   # on a later op
    assert lib.busfill_gemm_q4k_sweep(bad, 2, 8, None) == -1
    bad, keep4 = _sweep_ops([(256, 500, -1, False)])                  # K % 256
    assert lib.busfill_gemm_q4k_sweep(bad, 1, 8, None) == -2
    bad, keep5 = _sweep_ops([(1024 * 128 + 1, 256, -1, False)])      # N beyond 1024 tiles
    assert lib.busfill_gemm_q4k_sweep(bad, 1, 8, None) == -2
    bad, keep6 = _sweep_ops([(256, 512, -1, False)])
    bad[0].a = bad[0].a + 2                                           # activations not 16-byte aligned
    assert lib.busfill_gemm_q4k_sweep(bad, 1, 8, None) == -3


def _sweep_schedule(ops, g):
    """The sweep kernel's split restated (sweep_gemm.cuh: range_begin, owner,
    slot_of): per op, CTA b takes units [U b / G, U (b + 1) / G); returns per
    op the units covered, the partial slots written and the tiles stored."""
    def rb(u, b):
        return u * b // g

    def owner(u_tot, u):
        return ((u + 1) * g - 1) // u_tot

    res = []
    for tiles, s, planes in ops:
        u_tot, q = tiles * s * planes, s * planes
        covered, slots, arrivals, stored = {}, {}, {}, []
        for b in range(g):
            rs, re = rb(u_tot, b), rb(u_tot, b + 1)
            u = rs
            while u < re:
                tile, w = divmod(u, q)
                pl, sb = divmod(w, s)
                ln = min(s - sb, re - u)
                for j in range(ln):
                    assert (tile, pl, sb + j) not in covered
                    covered[(tile, pl, sb + j)] = b
                whole = rs <= tile * q and (tile + 1) * q <= re
                if whole:
                    if pl == planes - 1:
                        stored.append(tile)
                else:
                    k = (0 if rs // q == tile else 2) + pl
                    assert (b, k) not in slots
                    slots[(b, k)] = (tile, pl)
                    if u + ln == min((tile + 1) * q, re):
                        arrivals.setdefault(tile, []).append(b)
                u += ln
        for tile, bs in arrivals.items():
            c_lo, c_hi = owner(u_tot, tile * q), owner(u_tot, tile * q + q - 1)
            assert bs == [c for c in range(c_lo, c_hi + 1) if rb(u_tot, c) < rb(u_tot, c + 1)]
            stored.append(tile)
            for pl in range(planes):
                lo, hi = tile * q + pl * s, tile * q + (pl + 1) * s
                n = 0
                for c in range(c_lo, c_hi + 1):
                    a0, a1 = rb(u_tot, c), rb(u_tot, c + 1)
                    if max(a0, lo) < min(a1, hi):
                        assert slots[(c, (0 if a0 // q == tile else 2) + pl)] == (tile, pl)
                        n += min(a1, hi) - max(a0, lo)
                assert n == s
        res.append((len(covered) == u_tot, sorted(stored) == list(range(tiles))))
    return res


@pytest.mark.parametrize("g", [1, 2, 7, 64, 148])
def test_sweep_schedule_covers_every_unit_and_stores_every_tile_once(g):
    # BASELINE config 3's layer (O, QKV, gate/up pair, down) and small ops
    # with fewer units than CTAs
    layer = [(40, 32, 1), (80, 20, 1), (136, 20, 2), (40, 68, 1)]
    small = [(1, 1, 1), (3, 2, 2), (16, 4, 1), (5, 3, 2)]
    for ops in (layer, small):
        gg = min(g, max(t * s * p for t, s, p in ops))
        assert all(a and b for a, b in _sweep_schedule(ops, gg))
