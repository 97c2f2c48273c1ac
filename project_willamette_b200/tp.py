"""Tensor-parallel BitLinear and greedy lm-head across the GPUs of one box.

One process per GPU.  The reference runs a BitLinear as an independent dot
product per output row (src/model/bitlinear_sse2.rs:313-342 loops over rows
with one shared quantised input), so splitting the rows across GPUs and
gathering y is exact; its greedy head takes the first maximum of the logits
(src/model/lm_head.rs:161-176), which a vocab split reproduces with a
(max, lowest index) reduction of per-shard keys.

The exchange is fused into the library's kernels: each rank's kernels store
their output rows straight into every rank's symmetric block (CUDA IPC
mappings over NVLink) and bump arrival counters there; a kernel that reads a
gathered vector waits, bounded, on its own memory.  Handles are exchanged
once through any host channel -- ``torch.distributed`` (gloo or nccl) by
default.

Host-side helpers (``shard_rows``, ``order_keys``, ``reduce_keys``) are pure
numpy so the split and the reduction can be checked without a GPU.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Sequence

import numpy as np

from . import WillametteError
from ._abi import WL_TP_HANDLE_BYTES, WlI2sDevWeight, lib

__all__ = ["shard_rows", "order_keys", "reduce_keys", "decode_key", "TPGroup", "SymView"]


def shard_rows(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Contiguous row slice (first row, row count) of rank ``rank``.

    Rows are dealt in units of ``align`` (the stream kernel's 64-row box is a
    good unit), as evenly as possible, earlier ranks taking the remainder;
    the last unit may be partial.  Ranks past the end get an empty slice.
    """
    if world < 1 or not 0 <= rank < world or align < 1 or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank} align={align}")
    units = (n + align - 1) // align
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    r0, r1 = min(u0 * align, n), min(u1 * align, n)
    return r0, r1 - r0


def order_keys(logits: np.ndarray, row_offset: int = 0) -> np.ndarray:
    """64-bit keys whose unsigned maximum is the reference's greedy choice.

    High half: the f32 bits made monotone (-0.0 counted as +0.0); a NaN gets
    0 (never wins) except at global index 0, where the reference's scan keeps
    index 0 whatever follows, so it gets the largest key.  Low half:
    0xFFFFFFFF - index, so among equal values the lowest index wins.  The
    device kernels build the same keys.
    """
    v = np.array(logits, dtype=np.float32, copy=True).reshape(-1)
    rows = np.arange(v.size, dtype=np.uint64) + np.uint64(row_offset)
    nan = np.isnan(v)
    v[v == 0.0] = 0.0
    b = v.view(np.uint32).astype(np.uint64)
    hi = np.where(b & 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000)
    hi = np.where(nan, np.where(rows == 0, np.uint64(0xFFFFFFFF), np.uint64(0)), hi)
    return (hi.astype(np.uint64) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - rows)


def reduce_keys(keys: Sequence[int] | np.ndarray) -> int:
    """Combine per-shard maxima (empty shards contribute 0)."""
    k = np.asarray(keys, dtype=np.uint64).reshape(-1)
    return int(k.max()) if k.size else 0


def decode_key(key: int) -> int:
    return 0xFFFFFFFF - (int(key) & 0xFFFFFFFF)


class SymView:
    """A device array inside the group's symmetric block, exposed through
    ``__cuda_array_interface__`` (``torch.as_tensor(view, device=...)``)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str, owner: "TPGroup"):
        self.ptr, self.shape, self.typestr, self._owner = ptr, shape, typestr, owner

    @property
    def __cuda_array_interface__(self):
        return {"shape": self.shape, "typestr": self.typestr, "data": (self.ptr, False),
                "version": 2, "strides": None}


def _torch_exchange(handle: bytes, world: int) -> list[bytes]:
    import torch.distributed as dist
    out: list = [None] * world
    dist.all_gather_object(out, handle)
    return out


def _check(rc: int):
    if rc != 0:
        L = lib()
        raise WillametteError(rc, L.wl_last_error().decode(errors="replace"),
                              L.wl_last_error_tensor_type())


class TPGroup:
    """Symmetric block of ``sym_bytes`` on this rank's current device, mapped
    by every rank.  Every rank must make the same sequence of calls."""

    def __init__(self, rank: int, world: int, sym_bytes: int, device: int | None = None,
                 exchange: Callable[[bytes, int], list[bytes]] | None = None):
        L = lib()
        self.rank, self.world = rank, world
        self._g = C.c_void_p()
        _check(L.wl_init(rank if device is None else device))
        h = (C.c_uint8 * WL_TP_HANDLE_BYTES)()
        _check(L.wl_tp_create(rank, world, sym_bytes, C.byref(self._g), h))
        try:
            handles = (exchange or _torch_exchange)(bytes(h), world)
            if len(handles) != world or any(len(x) != WL_TP_HANDLE_BYTES for x in handles):
                raise WillametteError(8, "handle exchange returned the wrong shape", 0)
            allh = (C.c_uint8 * (WL_TP_HANDLE_BYTES * world)).from_buffer_copy(b"".join(handles))
            _check(L.wl_tp_connect(self._g, allh))
        except BaseException:
            # A peer that never joined (the exchange timed out or raised) or a
            # mapping that failed: free this rank's block and any peer mappings
            # now, not whenever the traceback lets go of this object.
            self.close()
            raise
        self.sym_bytes = sym_bytes

    def view(self, offset: int, shape, dtype=np.float32) -> SymView:
        """Array at byte ``offset`` of the symmetric region (same offset on
        every rank)."""
        dt = np.dtype(dtype)
        shape = (int(shape),) if np.isscalar(shape) else tuple(int(s) for s in shape)
        n = int(np.prod(shape)) * dt.itemsize
        if offset < 0 or offset + n > self.sym_bytes or offset % dt.itemsize:
            raise ValueError(f"view [{offset}, {offset + n}) outside the symmetric region")
        ptr = lib().wl_tp_buffer(self._g, offset)
        return SymView(ptr, shape, dt.str, self)

    def i2s_matvec(self, weights: Sequence[tuple[int, float, int, int]],
                   row_offsets: Sequence[int], in_dim: int, x_ptr: int,
                   wait_for_input: bool, stream: int = 0):
        """weights: (packed row-slice ptr, w_scale, slice rows, full-y ptr in
        the symmetric region, flags) per BitLinear sharing x."""
        arr = (WlI2sDevWeight * len(weights))()
        for i, w in enumerate(weights):
            packed, scale, rows, y = w[:4]
            arr[i].packed, arr[i].w_scale, arr[i].out_dim, arr[i].y = packed, scale, rows, y
            arr[i].acc, arr[i].flags = None, (w[4] if len(w) > 4 else 0)
        offs = (C.c_uint32 * len(weights))(*row_offsets)
        _check(lib().wl_tp_i2s_matvec_fused_f32(self._g, arr, offs, len(weights), in_dim, x_ptr,
                                                int(bool(wait_for_input)), stream))

    def stream_run(self, plan: int, stream: int = 0):
        _check(lib().wl_tp_i2s_stream_run(self._g, plan, stream))

    def wait(self, stream: int = 0):
        _check(lib().wl_tp_wait(self._g, stream))

    def lm_head_greedy(self, packed_shard: int, n_embd: int, vocab_shard: int, row_offset: int,
                       hidden_ptr: int, batch: int, ids_ptr: int, scratch_ptr: int,
                       stream: int = 0):
        _check(lib().wl_tp_q6k_lm_head_greedy(self._g, packed_shard, n_embd, vocab_shard,
                                              row_offset, hidden_ptr, batch, ids_ptr,
                                              scratch_ptr, stream))

    def close(self):
        if self._g:
            lib().wl_tp_destroy(self._g)
            self._g = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
