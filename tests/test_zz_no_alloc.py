"""busfill_gemm_q4k_noalloc: the Q4_K GEMM whose device scratch (its error
words) is a static array in the library instead of a cudaMalloc'd buffer.

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


@pytest.mark.gpu
def test_noalloc_matches_gemm_q4k_two_calls_in_a_row():
    # first: the headline shape (row tiles split along K over a cluster);
    # second: a shape with more tiles and a different activation-row count,
    # run right after on the same stream
    cases = [(32, 5120, 5120, 31), (17, 3840, 5120, 32)]
    stream = torch.cuda.current_stream()
    inputs, outs = [], []
    for m, n, k, seed in cases:
        blocks = cu(orc.gen_q4k(n, k, seed=seed))
        a = cu(orc.gen_activations(m, k, seed=seed + 1))
        out = torch.full((m, n), float("nan"), dtype=torch.float16, device=DEV)
        inputs.append((blocks, a))
        outs.append(out)
    for (blocks, a), out in zip(inputs, outs):
        bf.gemm_q4k_noalloc(blocks, a, out, stream=stream)
    torch.cuda.synchronize()
    for (blocks, a), out in zip(inputs, outs):
        want = bf.gemm_q4k(blocks, a, stream=stream)
        torch.cuda.synchronize()
        assert bf.stream_status() == 0
        max_abs, rel, finite = orc.gemm_errors(out.float().cpu().numpy(), want.float().cpu().numpy())
        assert finite, "non-finite output"
        assert max_abs <= orc.GATE_MAX_ABS, f"max abs diff {max_abs}"
        assert rel <= orc.GATE_REL_L2, f"rel-L2 diff {rel}"
