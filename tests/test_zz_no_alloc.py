"""busfill_gemm_q4k_noalloc: the Q4_K GEMM for callers that cannot let a
library allocate device memory -- a host whose own pool already holds nearly
all of the GPU's memory (an outside cudaMalloc would fail or fragment it), an
operator or plugin interface that hands a kernel only its inputs and outputs,
or a latency-bound loop where a cudaMalloc would stall the device. Its only
scratch, the error words, is a fixed 256-byte array compiled into the
library; large batches take whole work items, without the stream-K workspace.

The checks: the output is the plain entry point's bit for bit on the decode
kernel and within the oracle's gates on the whole-item prefill path, on two
calls in a row; a first call on a fresh stream makes no device allocation;
the static error word reads back clean through busfill_noalloc_status.

Collected last on purpose (file name), so that a run stopping at the first
failure has run every other test before this one.
"""
import numpy as np
import pytest

from oracle import q4_oracle as orc

torch = pytest.importorskip("torch")

import busfill_b200 as bf  # noqa: E402

DEV = "cuda:0"


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def test_noalloc_rejects_null_pointers_without_device():
    lib = bf.load_library()
    assert lib.busfill_gemm_q4k_noalloc(None, None, None, 8, 128, 256, None) == -1


def _inputs(m, n, k, seed):
    blocks_np = orc.gen_q4k(n, k, seed=seed)
    a_np = orc.gen_activations(m, k, seed=seed + 1)
    out = torch.full((m, n), float("nan"), dtype=torch.float16, device=DEV)
    return blocks_np, a_np, cu(blocks_np), cu(a_np), out


def _oracle_check(c, a_np, blocks_np, k, cols):
    """The gates on the output columns `cols` (weight rows), against an fp32
    matmul of the oracle's dequantized rows."""
    ref = orc.gemm_ref(a_np, orc.dequant_q4k_f32(blocks_np[cols], k))
    max_abs, rel, finite = orc.gemm_errors(c[:, cols], ref)
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2, (max_abs, rel)


@pytest.mark.gpu
def test_noalloc_matches_gemm_q4k_two_calls_in_a_row():
    # the headline shape (tiles split along K over a cluster), then right after
    # on the same stream a shape with more tiles and another batch size
    cases = [(32, 5120, 5120, 31), (17, 3840, 5120, 33)]
    stream = torch.cuda.current_stream()
    runs = [_inputs(m, n, k, seed) for m, n, k, seed in cases]
    for _, _, blocks, a, out in runs:
        bf.gemm_q4k_noalloc(blocks, a, out, stream=stream)
    assert bf.noalloc_status(stream) == (0, 0)
    for (m, n, k, _), (blocks_np, a_np, blocks, a, out) in zip(cases, runs):
        want = bf.gemm_q4k(blocks, a, stream=stream)
        assert bf.stream_status() == 0
        # same decode schedule as the plain entry point: the same bits
        assert torch.equal(out, want)
        _oracle_check(out.float().cpu().numpy(), a_np, blocks_np, k, np.arange(0, n, 7))


@pytest.mark.gpu
def test_noalloc_large_batch_takes_whole_items_two_calls_in_a_row():
    """M = 256 on the config-4 up projection: the prefill kernel with whole
    work items (the plain entry point splits items over all SMs through its
    stream-K workspace, so the sums differ in order: gates, not bits)."""
    m, n, k = 256, 17408, 5120
    blocks_np, a_np, blocks, a, out = _inputs(m, n, k, 51)
    out2 = torch.empty_like(out)
    bf.gemm_q4k_noalloc(blocks, a, out, stream=torch.cuda.current_stream())
    bf.gemm_q4k_noalloc(blocks, a, out2, stream=torch.cuda.current_stream())
    assert bf.noalloc_status() == (0, 0)
    assert torch.equal(out, out2)                       # deterministic
    c = out.float().cpu().numpy()
    rng = np.random.default_rng(5)
    cols = np.unique(np.concatenate([np.arange(0, 256), np.arange(n - 256, n), rng.integers(0, n, 512)]))
    _oracle_check(c, a_np, blocks_np, k, cols)
    want = bf.gemm_q4k(blocks, a)
    assert bf.stream_status() == 0
    max_abs, rel, finite = orc.gemm_errors(c, want.float().cpu().numpy())
    assert finite and max_abs <= orc.GATE_MAX_ABS and rel <= orc.GATE_REL_L2, (max_abs, rel)


@pytest.mark.gpu
def test_noalloc_allocates_nothing_on_a_fresh_stream():
    decode = _inputs(32, 5120, 5120, 61)
    prefill = _inputs(256, 17408, 5120, 63)
    for _, _, blocks, a, out in (decode, prefill):       # kernels loaded, device set-up done
        bf.gemm_q4k_noalloc(blocks, a, out)
    torch.cuda.synchronize()
    fresh = torch.cuda.Stream()
    torch.cuda.synchronize()
    count0 = bf.internal_allocations()
    free0 = torch.cuda.mem_get_info()[0]
    with torch.cuda.stream(fresh):
        for _, _, blocks, a, out in (decode, prefill):
            bf.gemm_q4k_noalloc(blocks, a, out, stream=fresh)
    assert bf.noalloc_status(fresh) == (0, 0)
    assert bf.internal_allocations() == count0
    assert torch.cuda.mem_get_info()[0] == free0
    # the counter does see allocations: the plain entry point's first call on
    # another fresh stream makes that stream's error words
    other = torch.cuda.Stream()
    bf.gemm_q4k(decode[2], decode[3], stream=other)
    assert bf.stream_status(other) == 0
    assert bf.internal_allocations() == count0 + 1
