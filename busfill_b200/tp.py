"""Column split of one quantized weight across a process group.

Rank r of g owns weight rows [start, stop) of the N output columns (a
contiguous slice of the packed [N, ...] buffers, for Q4_0 planes and Q4_K
blocks alike), computes C_r[M, stop-start] = A @ deq(W_r)^T with the local
GEMM, and an all-gather over the group (NCCL over NVLink on B200 nodes)
assembles C[M, N]. Every rank needs the full activations A. This is the only
exchange on the path: no reduction, since the K dimension is never split
across ranks.

Shards are whole 128-row tiles (the GEMM's tile height); when N does not
divide evenly the last ranks get fewer rows and every rank pads its slice to
the largest shard for the gather.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

TILE_ROWS = 128


def shard_rows(n: int, world: int, rank: int, align: int = TILE_ROWS) -> tuple[int, int]:
    """Rows [start, stop) of an n-row weight that `rank` of `world` owns.

    Tiles of `align` rows are dealt out as evenly as possible; the extra
    tiles go to the last ranks, which also hold the partial last tile, so
    shards differ by less than one tile. A rank can own zero rows when there
    are fewer tiles than ranks.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n < 0 or align < 1:
        raise ValueError(f"n={n}, align={align}")
    tiles = (n + align - 1) // align
    base, extra = divmod(tiles, world)
    first_big = world - extra          # ranks >= first_big take base + 1 tiles
    t0 = rank * base + max(0, rank - first_big)
    t1 = t0 + base + (1 if rank >= first_big else 0)
    return min(t0 * align, n), min(t1 * align, n)


def max_shard_rows(n: int, world: int, align: int = TILE_ROWS) -> int:
    """Rows of the largest shard (the padded gather width)."""
    return max(stop - start for start, stop in (shard_rows(n, world, r, align) for r in range(world)))


def gather_columns(c_local, n: int, group=None, out=None):
    """All-gather column slices C_r[M, rows_r] (rank order) into C[M, n].

    `c_local` is this rank's slice; slices are padded to the largest shard so
    that one all_gather_into_tensor moves them all.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    m = c_local.shape[0]
    width = max_shard_rows(n, world)
    start, stop = shard_rows(n, world, rank)
    if c_local.shape != (m, stop - start):
        raise ValueError(f"local slice {tuple(c_local.shape)} != ({m}, {stop - start})")
    if stop - start == width and c_local.is_contiguous():
        send = c_local
    else:
        send = torch.zeros((m, width), dtype=c_local.dtype, device=c_local.device)
        send[:, : stop - start] = c_local
    recv = torch.empty((world, m, width), dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(recv.view(world * m, width), send, group=group)
    if out is None:
        out = torch.empty((m, n), dtype=c_local.dtype, device=c_local.device)
    if n == world * width:
        out.view(m, world, width).copy_(recv.permute(1, 0, 2))
    else:
        for r in range(world):
            s0, s1 = shard_rows(n, world, r)
            out[:, s0:s1] = recv[r, :, : s1 - s0]
    return out


def gemm_q4k_tp(blocks_local, a, n: int, group=None, out=None, local_out=None,
                local_gemm: Optional[Callable] = None):
    """C[M, n] = A @ deq(W)^T with W's rows split over `group`.

    `blocks_local` holds this rank's rows of the llama.cpp block_q4_K weight
    (shard_rows(n, world, rank)). `local_gemm(blocks, a) -> C_local` defaults
    to busfill_b200.gemm_q4k (the C ABI on this rank's GPU), writing into
    `local_out` when given.
    """
    from . import gemm_q4k

    if blocks_local.shape[0] == 0:
        c_local = _empty_slice(a)
    elif local_gemm is not None:
        c_local = local_gemm(blocks_local, a)
    else:
        c_local = gemm_q4k(blocks_local, a, out=local_out)
    return gather_columns(c_local, n, group=group, out=out)


def gemm_q4_0_tp(wq_local, ws_local, a, n: int, group=None, out=None, local_out=None,
                 local_gemm: Optional[Callable] = None):
    """As gemm_q4k_tp for the split-plane Q4_0 layout (wq [rows, K/2], ws [rows, K/32])."""
    from . import gemm_q4_0

    if wq_local.shape[0] == 0:
        c_local = _empty_slice(a)
    elif local_gemm is not None:
        c_local = local_gemm(wq_local, ws_local, a)
    else:
        c_local = gemm_q4_0(wq_local, ws_local, a, out=local_out)
    return gather_columns(c_local, n, group=group, out=out)


def _empty_slice(a):
    """The slice of a rank that owns no rows (fewer tiles than ranks)."""
    import torch

    return torch.empty((a.shape[0], 0), dtype=torch.float16, device=a.device)


# ---------------------------------------------------------------------------
# Column split with the all-gather fused into the GEMM epilogue
# ---------------------------------------------------------------------------
class Gather(ctypes.Structure):
    """ctypes mirror of busfill_gather (include/busfill.h)."""
    _fields_ = [("npeers", ctypes.c_int), ("col_off", ctypes.c_int), ("ldc", ctypes.c_int),
                ("out", ctypes.c_void_p * 8), ("flag", ctypes.c_void_p * 8),
                ("wait", ctypes.c_void_p), ("wait_gen", ctypes.c_void_p), ("nwait", ctypes.c_int),
                ("wait_tiles", ctypes.c_int * 8)]


class _DevArray:
    """A raw device pointer seen as a torch tensor (CUDA array interface)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class GatherSpace:
    """Output buffers, flags and counters of a sequence of gathered GEMM call
    sites, in one device allocation per rank that every rank maps (CUDA IPC).

    Site i owns, in every rank's allocation, a full output [rows_i, cols_i]
    fp16, one tile-counter word per source rank (rank r adds to word r), and
    four local words that count this site's waits (two as a GEMM consumer,
    two through `wait`). A site's output is written by every rank's GEMM for
    that site and read by later sites. Within one pass over the sites, the
    separate buffer per site keeps a rank from overwriting data that another
    rank has not read yet. Across passes it does not: a site must not be
    called again until every rank's consumers of its previous output have
    finished, e.g. because a later site's wait already orders the ranks, or
    because the caller puts a barrier between passes (as the tests and the
    benchmark do between graph replays).
    """

    _ALIGN = 256

    def __init__(self, sites, group=None):
        import torch
        import torch.distributed as dist

        from . import _check, _lib

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.sites = [(int(r), int(c)) for r, c in sites]
        off = 0
        self._off = []
        for rows, cols in self.sites:
            o_out = off
            off = _align(off + rows * cols * 2, self._ALIGN)
            o_flag = off
            off = _align(off + 4 * self.world, self._ALIGN)
            o_cnt = off
            off = _align(off + 16, self._ALIGN)
            self._off.append((o_out, o_flag, o_cnt))
        self.bytes = max(off, self._ALIGN)
        lib = _lib()
        base = ctypes.c_void_p()
        _check(lib.busfill_ipc_alloc(self.bytes, ctypes.byref(base)), "busfill_ipc_alloc")
        self._base = base.value
        handle = ctypes.create_string_buffer(64)
        _check(lib.busfill_ipc_get_handle(self._base, handle), "busfill_ipc_get_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.bases = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.bases.append(self._base)
                continue
            p = ctypes.c_void_p()
            hb = ctypes.create_string_buffer(h, 64)
            _check(lib.busfill_ipc_open(hb, ctypes.byref(p)), "busfill_ipc_open")
            self.bases.append(p.value)
        self._structs = {}
        self._torch = torch

    def output(self, site):
        """This rank's full output of `site` as a torch fp16 tensor [rows, cols]."""
        rows, cols = self.sites[site]
        return self._torch.as_tensor(_DevArray(self._base + self._off[site][0], (rows, cols), "<f2"),
                                     device=self._torch.device("cuda", self._torch.cuda.current_device()))

    def args(self, site, wait_site=None):
        """The busfill_gather struct of `site` on this rank (cached)."""
        key = (site, wait_site)
        g = self._structs.get(key)
        if g is not None:
            return g
        rows, cols = self.sites[site]
        start, stop = shard_rows(cols, self.world, self.rank)
        o_out, o_flag, o_cnt = self._off[site]
        g = Gather()
        g.npeers = self.world
        g.col_off = start
        g.ldc = cols
        for q in range(self.world):
            g.out[q] = self.bases[q] + o_out
            g.flag[q] = self.bases[q] + o_flag + 4 * self.rank
        if wait_site is not None:
            g.wait = self._base + self._off[wait_site][1]
            g.wait_gen = self._base + o_cnt          # this site's 2 words counting its waits on wait_site
            g.nwait = self.world
            for r in range(self.world):
                g.wait_tiles[r] = self._tiles(wait_site, r)
        self._structs[key] = g
        return g

    def _tiles(self, site, r):
        """128-row output tiles rank r writes per call of `site`."""
        s0, s1 = shard_rows(self.sites[site][1], self.world, r)
        return (s1 - s0 + TILE_ROWS - 1) // TILE_ROWS

    def wait(self, site, stream=None):
        """Make `stream` wait (on the device) until `site`'s gathered output is
        complete on this rank, for consumers that are not busfill GEMMs."""
        from . import _check, _lib, _stream
        key = ("wait", site)
        g = self._structs.get(key)
        if g is None:
            g = Gather()
            g.wait = self._base + self._off[site][1]
            g.wait_gen = self._base + self._off[site][2] + 8    # this site's standalone wait count (2 words)
            g.nwait = self.world
            for r in range(self.world):
                g.wait_tiles[r] = self._tiles(site, r)
            self._structs[key] = g
        _check(_lib().busfill_gather_wait(ctypes.byref(g), _stream(stream)), "busfill_gather_wait")

    def close(self):
        from . import _lib
        lib = _lib()
        for q, b in enumerate(self.bases):
            if q != self.rank and b:
                lib.busfill_ipc_close(b)
        if self._base:
            lib.busfill_ipc_free(self._base)
        self.bases, self._base = [], 0


def _align(x, a):
    return (x + a - 1) // a * a


def gemm_q4k_gather(blocks_local, a, space, site, wait_site=None, stream=None):
    """C = A @ deq(W)^T with W's rows split over the group and the all-gather
    done by the GEMM epilogue (busfill_gemm_q4k_gather); returns this rank's
    full output of `site`. `wait_site`: the site whose gathered output `a` is."""
    from . import _check, _lib, _ptr, _stream
    m, k = a.shape
    n = blocks_local.shape[0]
    g = space.args(site, wait_site)
    _check(_lib().busfill_gemm_q4k_gather(_ptr(blocks_local), _ptr(a), m, n, k, ctypes.byref(g), _stream(stream)),
           "busfill_gemm_q4k_gather")
    return space.output(site)


def gemm_q4k_swiglu_gather(w_gate_local, w_up_local, a, space, site, wait_site=None, stream=None):
    """busfill_gemm_q4k_swiglu on this rank's gate/up rows with the gathered output."""
    from . import _check, _lib, _ptr, _stream
    m, k = a.shape
    n = w_gate_local.shape[0]
    g = space.args(site, wait_site)
    _check(_lib().busfill_gemm_q4k_swiglu_gather(_ptr(w_gate_local), _ptr(w_up_local), _ptr(a), m, n, k,
                                                 ctypes.byref(g), _stream(stream)),
           "busfill_gemm_q4k_swiglu_gather")
    return space.output(site)
