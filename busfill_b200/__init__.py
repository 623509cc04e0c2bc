"""bus-fill on B200: Python host API over the C ABI in include/busfill.h.

The kernels live in ``busfill_b200/lib/libbusfill.so`` (built in-tree by
``python -m busfill_b200.build``). Every call here goes through that C ABI via
ctypes; there is no CPU or PyTorch fallback -- if the library is missing or the
device is not sm_100, calls raise :class:`BusfillError`.

Layouts (see include/busfill.h):
* Q4_0 split planes, the reference's kernel ABI (kernels/busfill_v1a.cu:43-45):
  ``wq`` uint8 [N, K/2], ``ws`` fp16 [N, K/32].
* Q4_K: llama.cpp ``block_q4_K`` rows, uint8 [N, K/256*144].
* activations fp16 [M, K]; outputs fp16 [M, N] (``busfill_q4``: fp32).
"""
from __future__ import annotations

import ctypes
import os
import re

__all__ = [
    "BusfillError", "load_library", "library_path", "header_functions",
    "gemm_q4_0", "gemm_q4k", "gemm_q4_0_ggml", "gemm_q4k_swiglu", "gemm_q4k_sweep", "SweepOp", "gemm_q4k_noalloc", "gemm_q5k", "gemm_q6k", "repack_q6k",
    "busfill_q4", "repack_q4k_planar", "gemm_q4k_planar", "Tensor", "tensor_desc", "mul_mat", "dequant_q4_0", "dequant_q4_0_ggml", "dequant_q4k", "dequant_q5k", "dequant_q6k",
    "stream_status", "stream_status_bits", "noalloc_status", "internal_allocations", "set_pdl", "set_ksplit", "set_prefill_min_m", "set_exact_kquant", "uses_prefill", "gemm_launches", "probe_umma", "version",
]

_PKG = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(_PKG)
_HEADER = os.path.join(_ROOT, "include", "busfill.h")
_LIB = None

STATUS = {
    0: "BUSFILL_OK", -1: "BUSFILL_ERR_INVALID_ARG", -2: "BUSFILL_ERR_SHAPE", -3: "BUSFILL_ERR_ALIGNMENT",
    -4: "BUSFILL_ERR_UNSUPPORTED_DEVICE", -5: "BUSFILL_ERR_LAUNCH", -6: "BUSFILL_ERR_ALLOC",
    -7: "BUSFILL_ERR_DEVICE_TIMEOUT", -8: "BUSFILL_ERR_CUDA",
}


class BusfillError(RuntimeError):
    """A busfill C-ABI call returned a non-zero status."""

    def __init__(self, status: int, where: str):
        self.status = status
        text = _LIB.busfill_status_string(status).decode() if _LIB is not None else ""
        super().__init__(f"{where}: {STATUS.get(status, status)} ({text})")


def library_path() -> str:
    return os.environ.get("BUSFILL_LIB", os.path.join(_PKG, "lib", "libbusfill.so"))


def header_functions(path: str = _HEADER):
    """Names of the functions include/busfill.h declares."""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"^\s*BUSFILL_API\s+(?:const\s+)?\w+\**\s+\**(busfill_\w+)\s*\(", src, flags=re.M)


_P = ctypes.c_void_p
_I = ctypes.c_int
_SIGS = {
    "busfill_gemm_q4_0": [_P, _P, _P, _P, _I, _I, _I, _P],
    "busfill_gemm_q4k": [_P, _P, _P, _I, _I, _I, _P],
    "busfill_gemm_q4_0_ggml": [_P, _P, _P, _I, _I, _I, _P],
    "busfill_gemm_q4k_swiglu": [_P, _P, _P, _P, _I, _I, _I, _P],
    "busfill_gemm_q4k_sweep": [_P, _I, _I, _P],
    "busfill_gemm_q5k": [_P, _P, _P, _I, _I, _I, _P],
    "busfill_dequant_q5k": [_P, _P, _I, _I, _P],
    "busfill_gemm_q6k": [_P, _P, _P, _P, _I, _I, _I, _P],
    "busfill_repack_q6k": [_P, _P, _P, _I, _I, _P],
    "busfill_dequant_q6k": [_P, _P, _P, _I, _I, _P],
    "busfill_gemm_q4k_noalloc": [_P, _P, _P, _I, _I, _I, _P],
    "busfill_repack_q4k_planar": [_P, _P, _P, _P, _P, _I, _I, _P],
    "busfill_gemm_q4k_planar": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "busfill_mul_mat": [_P, _P, _P, _P],
    "busfill_noalloc_status": [_P, ctypes.POINTER(ctypes.c_uint)],
    "busfill_internal_allocations": [],
    "busfill_q4": [_P, _P, _P, _P, _I, _I, _I, _P],
    "busfill_dequant_q4_0": [_P, _P, _P, _I, _I, _P],
    "busfill_dequant_q4_0_ggml": [_P, _P, _I, _I, _P],
    "busfill_dequant_q4k": [_P, _P, _I, _I, _P],
    "busfill_stream_status": [_P],
    "busfill_stream_status_ex": [_P, ctypes.POINTER(ctypes.c_uint)],
    "busfill_last_failure_detail": [],
    "busfill_status_string": [_I],
    "busfill_version": [],
    "busfill_set_option": [_I, _I],
    "busfill_probe_umma": [_P, _P, _P, _I, _P],
    "busfill_gemm_kernel_for": [_I, _I, _I],
    "busfill_gemm_launches": [_I, _I, _I, _I],
    "busfill_gemm_q4k_gather": [_P, _P, _I, _I, _I, _P, _P],
    "busfill_gemm_q4k_swiglu_gather": [_P, _P, _P, _I, _I, _I, _P, _P],
    "busfill_gather_wait": [_P, _P],
    "busfill_ipc_alloc": [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)],
    "busfill_ipc_free": [_P],
    "busfill_ipc_get_handle": [_P, _P],
    "busfill_ipc_open": [_P, ctypes.POINTER(ctypes.c_void_p)],
    "busfill_ipc_close": [_P],
}


def load_library(path: str | None = None):
    """Load libbusfill.so (once) and declare argument types. Raises if absent."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or library_path()
    if not os.path.exists(p):
        raise RuntimeError(f"libbusfill.so not found at {p}; build it with `python -m busfill_b200.build`")
    lib = ctypes.CDLL(p)
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = (ctypes.c_char_p if name == "busfill_status_string"
                      else ctypes.c_uint if name in ("busfill_last_failure_detail", "busfill_internal_allocations")
                      else ctypes.c_int)
    if path is None:
        _LIB = lib
    return lib


def _lib():
    if _LIB is None:
        load_library()
    return _LIB


def version() -> int:
    return _lib().busfill_version()


def set_pdl(enabled: bool) -> None:
    """Enable/disable programmatic dependent launch for the GEMMs (default on)."""
    _check(_lib().busfill_set_option(1, 1 if enabled else 0), "busfill_set_option")


def set_ksplit(csize: int) -> None:
    """Force the number of CTAs (cluster size, 1..8) that split each 128-row
    tile along K; 0 restores the library's own choice."""
    _check(_lib().busfill_set_option(2, int(csize)), "busfill_set_option")


def uses_prefill(m: int, n: int, k: int) -> bool:
    """True if a GEMM of m batch rows, n output columns and depth k runs the prefill kernel."""
    return _lib().busfill_gemm_kernel_for(int(m), int(n), int(k)) == 1


def gemm_launches(m: int, n: int, k: int, sm_count: int = 0) -> int:
    """Kernel launches of one plain GEMM call of that shape (busfill_gemm_launches)."""
    v = _lib().busfill_gemm_launches(int(m), int(n), int(k), int(sm_count))
    _check(min(v, 0), "busfill_gemm_launches")
    return v


def set_exact_kquant(on: bool) -> None:
    """BUSFILL_OPT_EXACT_KQUANT, kept for callers that set it: every K-quant
    GEMM operand is already fp16_rn(fp32 w), the CPU dequant's bits, so the
    option changes nothing."""
    _check(_lib().busfill_set_option(4, 1 if on else 0), "busfill_set_option")


def set_prefill_min_m(m: int) -> None:
    """GEMMs with at least `m` batch rows take the large-batch (prefill)
    kernel; 0 restores the default threshold."""
    _check(_lib().busfill_set_option(3, int(m)), "busfill_set_option")


def set_prefill_batch_tile(bt: int) -> None:
    """Batch rows per work item of the prefill kernel: 128 (two weight tiles)
    or 256 (one weight tile, MMA N = 256); 0 restores the choice by M."""
    _check(_lib().busfill_set_option(5, int(bt)), "busfill_set_option")


def set_sweep_ctas(n: int) -> None:
    """BUSFILL_OPT_SWEEP_CTAS: CTAs of a layer-sweep launch (0 = one per SM)."""
    _check(_lib().busfill_set_option(7, n), "busfill_set_option")


def set_prefill_pair(mode: int) -> None:
    """Prefill GEMMs on CTA pairs (256 x 256 items over a 2-CTA cluster):
    0 = from M = 256 (default), 1 = always (not the SwiGLU pairs), 2 = never."""
    _check(_lib().busfill_set_option(6, int(mode)), "busfill_set_option")


# ---------------------------------------------------------------------------
# torch-tensor wrappers
# ---------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def _check(status: int, where: str):
    if status != 0:
        raise BusfillError(status, where)


def _stream(stream):
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _need(t, dtype, name, ndim=2):
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != ndim or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous {ndim}-D tensor")


def gemm_q4_0(wq, ws, a, out=None, stream=None):
    """C[M, N] = A[M, K] @ deq(Wq, Ws)[N, K]^T for reference split-plane Q4_0; fp16 out."""
    torch = _torch()
    _need(wq, torch.uint8, "wq"); _need(ws, torch.float16, "ws"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = wq.shape[0]
    if wq.shape[1] * 2 != k or ws.shape != (n, k // 32):
        raise ValueError(f"shape mismatch: wq {tuple(wq.shape)}, ws {tuple(ws.shape)}, a {tuple(a.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q4_0(_ptr(wq), _ptr(ws), _ptr(a), _ptr(out), m, n, k, _stream(stream)),
           "busfill_gemm_q4_0")
    return out


def gemm_q4k(blocks, a, out=None, stream=None):
    """C[M, N] = A[M, K] @ deq(W)[N, K]^T for llama.cpp block_q4_K rows; fp16 out."""
    torch = _torch()
    _need(blocks, torch.uint8, "blocks"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = blocks.shape[0]
    if k % 256 or blocks.shape[1] != k // 256 * 144:
        raise ValueError(f"shape mismatch: blocks {tuple(blocks.shape)}, a {tuple(a.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q4k(_ptr(blocks), _ptr(a), _ptr(out), m, n, k, _stream(stream)), "busfill_gemm_q4k")
    return out


def gemm_q4_0_ggml(blocks, a, out=None, stream=None):
    """C[M, N] = A[M, K] @ deq(W)[N, K]^T for llama.cpp block_q4_0 rows
    (18-byte blocks, [N, K/32*18] u8); fp16 out. K % 256 == 0."""
    torch = _torch()
    _need(blocks, torch.uint8, "blocks"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = blocks.shape[0]
    if k % 256 or blocks.shape[1] != k // 32 * 18:
        raise ValueError(f"shape mismatch: blocks {tuple(blocks.shape)}, a {tuple(a.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q4_0_ggml(_ptr(blocks), _ptr(a), _ptr(out), m, n, k, _stream(stream)),
           "busfill_gemm_q4_0_ggml")
    return out


def gemm_q4k_swiglu(w_gate, w_up, a, out=None, stream=None):
    """h[M, N] = silu(A @ deq(Wg)^T) * (A @ deq(Wu)^T) for two llama.cpp
    block_q4_K weights [N, K/256*144] (ffn_gate, ffn_up); fp16 out."""
    torch = _torch()
    _need(w_gate, torch.uint8, "w_gate"); _need(w_up, torch.uint8, "w_up"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = w_gate.shape[0]
    if k % 256 or w_gate.shape[1] != k // 256 * 144 or tuple(w_up.shape) != tuple(w_gate.shape):
        raise ValueError(f"shape mismatch: w_gate {tuple(w_gate.shape)}, w_up {tuple(w_up.shape)}, a {tuple(a.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q4k_swiglu(_ptr(w_gate), _ptr(w_up), _ptr(a), _ptr(out), m, n, k, _stream(stream)),
           "busfill_gemm_q4k_swiglu")
    return out


class SweepOp(ctypes.Structure):
    """busfill_sweep_op: one GEMM of a layer sweep."""
    _fields_ = [("w", _P), ("w_up", _P), ("a", _P), ("c", _P), ("N", _I), ("K", _I), ("dep", _I)]


SWEEP_MAX_OPS = 8


def gemm_q4k_sweep(ops, stream=None):
    """Run up to SWEEP_MAX_OPS Q4_K GEMMs of one batch size M <= 32 as one
    launch (busfill_gemm_q4k_sweep). `ops` is a list of dicts with keys ``w``
    (block_q4_K rows [N, K/256*144]), ``a`` (fp16 [M, K]), ``out`` (fp16
    [M, N]) and optionally ``w_up`` (SwiGLU pair: out = silu(a w^T) * (a
    w_up^T)) and ``dep`` (index of the earlier op whose output ``a`` is).
    Returns the outputs."""
    torch = _torch()
    if not 1 <= len(ops) <= SWEEP_MAX_OPS:
        raise ValueError(f"1..{SWEEP_MAX_OPS} ops, got {len(ops)}")
    arr = (SweepOp * len(ops))()
    m = None
    for i, op in enumerate(ops):
        w, a, out, w_up = op["w"], op["a"], op["out"], op.get("w_up")
        _need(w, torch.uint8, "w"); _need(a, torch.float16, "a"); _need(out, torch.float16, "out")
        mi, k = a.shape
        n = w.shape[0]
        if m is None:
            m = mi
        if mi != m or k % 256 or w.shape[1] != k // 256 * 144 or tuple(out.shape) != (m, n):
            raise ValueError(f"op {i}: shape mismatch: w {tuple(w.shape)}, a {tuple(a.shape)}, out {tuple(out.shape)}")
        if w_up is not None:
            _need(w_up, torch.uint8, "w_up")
            if tuple(w_up.shape) != tuple(w.shape):
                raise ValueError(f"op {i}: w_up {tuple(w_up.shape)} != w {tuple(w.shape)}")
        arr[i].w, arr[i].a, arr[i].c = w.data_ptr(), a.data_ptr(), out.data_ptr()
        arr[i].w_up = w_up.data_ptr() if w_up is not None else None
        arr[i].N, arr[i].K, arr[i].dep = n, k, int(op.get("dep", -1))
    _check(_lib().busfill_gemm_q4k_sweep(arr, len(ops), m, _stream(stream)), "busfill_gemm_q4k_sweep")
    return [op["out"] for op in ops]


def gemm_q4k_noalloc(blocks, a, out, stream=None):
    """gemm_q4k through busfill_gemm_q4k_noalloc: the library allocates no
    device memory (its error words are a fixed 256-byte array in the library
    image), so `out` must be given. Calls whose kernels overlap on the GPU
    share that array and race on it."""
    torch = _torch()
    _need(blocks, torch.uint8, "blocks"); _need(a, torch.float16, "a"); _need(out, torch.float16, "out")
    m, k = a.shape
    n = blocks.shape[0]
    if k % 256 or blocks.shape[1] != k // 256 * 144 or tuple(out.shape) != (m, n):
        raise ValueError(f"shape mismatch: blocks {tuple(blocks.shape)}, a {tuple(a.shape)}, out {tuple(out.shape)}")
    _check(_lib().busfill_gemm_q4k_noalloc(_ptr(blocks), _ptr(a), _ptr(out), m, n, k, _stream(stream)),
           "busfill_gemm_q4k_noalloc")
    return out


def repack_q4k_planar(qs, d, dmin, scales12, stream=None):
    """Q4_K planes (qs u8 [N, K/2], d / dmin fp16 [N, K/256], scales12 u8
    [N, K/256*12]) -> llama.cpp block_q4_K rows u8 [N, K/256*144]."""
    torch = _torch()
    _need(qs, torch.uint8, "qs"); _need(d, torch.float16, "d"); _need(dmin, torch.float16, "dmin")
    _need(scales12, torch.uint8, "scales12")
    n, k = qs.shape[0], qs.shape[1] * 2
    blocks = torch.empty((n, k // 256 * 144), dtype=torch.uint8, device=qs.device)
    _check(_lib().busfill_repack_q4k_planar(_ptr(qs), _ptr(d), _ptr(dmin), _ptr(scales12), _ptr(blocks), n, k,
                                            _stream(stream)), "busfill_repack_q4k_planar")
    return blocks


def gemm_q4k_planar(qs, d, dmin, scales12, a, out=None, stream=None):
    """C[M, N] = A @ deq(W)^T with the Q4_K weight given as planes (see
    repack_q4k_planar); the library repacks per call into its own buffer."""
    torch = _torch()
    _need(qs, torch.uint8, "qs"); _need(d, torch.float16, "d"); _need(dmin, torch.float16, "dmin")
    _need(scales12, torch.uint8, "scales12"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = qs.shape[0]
    if qs.shape[1] * 2 != k or d.shape != (n, k // 256) or dmin.shape != (n, k // 256) or \
            scales12.shape != (n, k // 256 * 12):
        raise ValueError("shape mismatch between the Q4_K planes and a")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q4k_planar(_ptr(qs), _ptr(d), _ptr(dmin), _ptr(scales12), _ptr(a), _ptr(out), m, n,
                                          k, _stream(stream)), "busfill_gemm_q4k_planar")
    return out


class Tensor(ctypes.Structure):
    """ctypes mirror of busfill_tensor (a ggml-style tensor description)."""
    _fields_ = [("type", ctypes.c_int32), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                ("data", ctypes.c_void_p)]


TYPE_F16, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q5_K = 1, 2, 12, 13
_BLOCK = {TYPE_Q4_0: (32, 18), TYPE_Q4_K: (256, 144), TYPE_Q5_K: (256, 176)}


def tensor_desc(t, ggml_type, ne):
    """busfill_tensor of a CUDA tensor holding a packed ggml tensor of type
    `ggml_type` with ggml shape `ne` (innermost first); strides as ggml
    computes them for a contiguous tensor."""
    ne = list(ne) + [1] * (4 - len(ne))
    if ggml_type == TYPE_F16:
        nb0, row = 2, 2 * ne[0]
    else:
        qk, bs = _BLOCK[ggml_type]
        nb0, row = bs, ne[0] // qk * bs
    d = Tensor()
    d.type = ggml_type
    for i in range(4):
        d.ne[i] = ne[i]
    d.nb[0], d.nb[1] = nb0, row
    d.nb[2] = row * ne[1]
    d.nb[3] = d.nb[2] * ne[2]
    d.data = t.data_ptr()
    return d


def mul_mat(src0, src1, dst, stream=None):
    """busfill_mul_mat on three busfill_tensor descriptions (ggml_mul_mat)."""
    _check(_lib().busfill_mul_mat(ctypes.byref(src0), ctypes.byref(src1), ctypes.byref(dst), _stream(stream)),
           "busfill_mul_mat")


def busfill_q4(A, Wq, Ws, C, Bsz, K, N, stream=None):
    """The reference kernel surface busfill_q4(A, Wq, Ws, C, Bsz, K, N)
    (kernels/busfill_v1a.cu:41-46): fp32 C [Bsz, N], all Bsz rows computed."""
    torch = _torch()
    _need(A, torch.float16, "A"); _need(Wq, torch.uint8, "Wq"); _need(Ws, torch.float16, "Ws")
    _need(C, torch.float32, "C")
    _check(_lib().busfill_q4(_ptr(A), _ptr(Wq), _ptr(Ws), _ptr(C), Bsz, K, N, _stream(stream)), "busfill_q4")
    return C


def dequant_q4_0(wq, ws, out=None, stream=None):
    torch = _torch()
    _need(wq, torch.uint8, "wq"); _need(ws, torch.float16, "ws")
    n, k = wq.shape[0], wq.shape[1] * 2
    if out is None:
        out = torch.empty((n, k), dtype=torch.float16, device=wq.device)
    _check(_lib().busfill_dequant_q4_0(_ptr(wq), _ptr(ws), _ptr(out), n, k, _stream(stream)),
           "busfill_dequant_q4_0")
    return out


def dequant_q4_0_ggml(blocks, k, out=None, stream=None):
    torch = _torch()
    _need(blocks, torch.uint8, "blocks")
    n = blocks.shape[0]
    if out is None:
        out = torch.empty((n, k), dtype=torch.float16, device=blocks.device)
    _check(_lib().busfill_dequant_q4_0_ggml(_ptr(blocks), _ptr(out), n, k, _stream(stream)),
           "busfill_dequant_q4_0_ggml")
    return out


def dequant_q4k(blocks, k, out=None, stream=None):
    torch = _torch()
    _need(blocks, torch.uint8, "blocks")
    n = blocks.shape[0]
    if out is None:
        out = torch.empty((n, k), dtype=torch.float16, device=blocks.device)
    _check(_lib().busfill_dequant_q4k(_ptr(blocks), _ptr(out), n, k, _stream(stream)), "busfill_dequant_q4k")
    return out


def gemm_q5k(blocks, a, out=None, stream=None):
    """C[M, N] = A[M, K] @ deq(W)[N, K]^T for llama.cpp block_q5_K rows
    [N, K/256*176]; fp16 out."""
    torch = _torch()
    _need(blocks, torch.uint8, "blocks"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = blocks.shape[0]
    if k % 256 or blocks.shape[1] != k // 256 * 176:
        raise ValueError(f"shape mismatch: blocks {tuple(blocks.shape)}, a {tuple(a.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q5k(_ptr(blocks), _ptr(a), _ptr(out), m, n, k, _stream(stream)), "busfill_gemm_q5k")
    return out


def dequant_q5k(blocks, k, out=None, stream=None):
    torch = _torch()
    _need(blocks, torch.uint8, "blocks")
    n = blocks.shape[0]
    if out is None:
        out = torch.empty((n, k), dtype=torch.float16, device=blocks.device)
    _check(_lib().busfill_dequant_q5k(_ptr(blocks), _ptr(out), n, k, _stream(stream)), "busfill_dequant_q5k")
    return out


def repack_q6k(blocks, k, stream=None):
    """llama.cpp block_q6_K rows u8 [N, K/256*210] -> (body u8 [N, K/256*208],
    d fp16 [K/256, N]), the layout of gemm_q6k (busfill_repack_q6k)."""
    torch = _torch()
    _need(blocks, torch.uint8, "blocks")
    n = blocks.shape[0]
    if k % 256 or blocks.shape[1] != k // 256 * 210:
        raise ValueError(f"shape mismatch: blocks {tuple(blocks.shape)}, k {k}")
    body = torch.empty((n, k // 256 * 208), dtype=torch.uint8, device=blocks.device)
    d = torch.empty((k // 256, n), dtype=torch.float16, device=blocks.device)
    _check(_lib().busfill_repack_q6k(_ptr(blocks), _ptr(body), _ptr(d), n, k, _stream(stream)), "busfill_repack_q6k")
    return body, d


def gemm_q6k(body, d, a, out=None, stream=None):
    """C[M, N] = A[M, K] @ deq(W)[N, K]^T for Q6_K weights in the repacked
    layout (repack_q6k); fp16 out."""
    torch = _torch()
    _need(body, torch.uint8, "body"); _need(d, torch.float16, "d"); _need(a, torch.float16, "a")
    m, k = a.shape
    n = body.shape[0]
    if k % 256 or body.shape[1] != k // 256 * 208 or d.shape != (k // 256, n):
        raise ValueError(f"shape mismatch: body {tuple(body.shape)}, d {tuple(d.shape)}, a {tuple(a.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    _need(out, torch.float16, "out")
    _check(_lib().busfill_gemm_q6k(_ptr(body), _ptr(d), _ptr(a), _ptr(out), m, n, k, _stream(stream)),
           "busfill_gemm_q6k")
    return out


def dequant_q6k(body, d, k, out=None, stream=None):
    torch = _torch()
    _need(body, torch.uint8, "body"); _need(d, torch.float16, "d")
    n = body.shape[0]
    if out is None:
        out = torch.empty((n, k), dtype=torch.float16, device=body.device)
    _check(_lib().busfill_dequant_q6k(_ptr(body), _ptr(d), _ptr(out), n, k, _stream(stream)), "busfill_dequant_q6k")
    return out


def noalloc_status(stream=None):
    """(status, error_bits) of the no-allocation GEMMs' static error word
    (busfill_noalloc_status): synchronizes the stream, reads and clears it."""
    bits = ctypes.c_uint(0)
    st = _lib().busfill_noalloc_status(_stream(stream), ctypes.byref(bits))
    return st, bits.value


def internal_allocations() -> int:
    """Device allocations the library has made on its own so far."""
    return _lib().busfill_internal_allocations()


def stream_status(stream=None) -> int:
    """Synchronize the stream and return the device-side status code (0 = ok)."""
    return _lib().busfill_stream_status(_stream(stream))


def stream_status_bits(stream=None):
    """(status, error_bits): the device error word names the kernel roles whose
    bounded wait expired (see include/busfill.h)."""
    bits = ctypes.c_uint(0)
    st = _lib().busfill_stream_status_ex(_stream(stream), ctypes.byref(bits))
    return st, bits.value


def probe_umma(a, b, nb, stream=None):
    """tcgen05 operand-layout probe: returns fp32 [128, nb] = a[128,64] @ b[nb,64]^T."""
    torch = _torch()
    _need(a, torch.float16, "a"); _need(b, torch.float16, "b")
    d = torch.empty((128, nb), dtype=torch.float32, device=a.device)
    _check(_lib().busfill_probe_umma(_ptr(a), _ptr(b), _ptr(d), nb, _stream(stream)), "busfill_probe_umma")
    return d
