"""Row sharding of large matvecQ8 GEMVs over the GPUs of one node.

Rows are independent (ops/matvec/reference.ts:117-131 computes each output
from its own row), so a GEMV splits by output row with no exchange during
the dot products: GPU g holds rows [g*R, (g+1)*R) of every matrix, R =
ceil(N / G), computes its slice of y, and one all-gather over NVLink
assembles y on every GPU.  With a stack of matrices applied to one x, the
slices of all matrices are gathered in one collective; the gathered buffer is
rank-major, ``[G][matrices][R]``, and ``gathered_to_rows`` restores
``[matrices][N]``.
"""
from __future__ import annotations

import numpy as np


def shard_rows(N: int, world: int, rank: int):
    """(first row, row count, padded rows per rank) of `rank`'s shard."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"shard_rows: rank {rank} outside a world of {world}")
    per = -(-N // world)
    first = min(N, rank * per)
    count = max(0, min(N, first + per) - first)
    return first, count, per


def gathered_to_rows(gathered, world: int, matrices: int, N: int) -> np.ndarray:
    """``[world][matrices][per]`` (all-gather order) -> ``[matrices][N]``."""
    per = -(-N // world)
    g = np.asarray(gathered).reshape(world, matrices, per)
    return g.transpose(1, 0, 2).reshape(matrices, world * per)[:, :N]


def shard_bytes(N: int, K: int, world: int, rank: int, matrices: int = 1) -> int:
    """Algorithmic bytes one rank moves per pass over the stack: its codes,
    scales and outputs, and x once."""
    _, rows, _ = shard_rows(N, world, rank)
    W = (K + 3) // 4
    return matrices * rows * (4 * W + 8) + 4 * K


class RowShardGroup:
    """One process driving several GPUs of this node (xpu_dist_create): the
    row-sharded matvecQ8 stack without torch.distributed.  Device g of
    `devices` holds rows [g R, (g + 1) R) of every matrix, R = N / len(devices)."""

    def __init__(self, devices):
        import ctypes as C

        from ._lib import check, lib

        self._lib, self._check = lib(), check
        self.devices = [int(d) for d in devices]
        arr = (C.c_int32 * len(self.devices))(*self.devices)
        h = C.c_void_p()
        check(self._lib.xpu_dist_create(len(self.devices), arr, C.byref(h)))
        self._h = h

    def matvecQ8StackRowShard(self, weights, weight_stride: int, scales, vectors, count: int, N: int, K: int,
                              outputs) -> None:
        """weights/scales/vectors/outputs: one device pointer (or tensor,
        DeviceBuffer) per device; blocking; every outputs[g] gets [count][N]."""
        import ctypes as C

        from .ops import _ptr

        G = len(self.devices)
        arr = lambda xs: (C.c_void_p * G)(*[_ptr(x) for x in xs])
        self._check(self._lib.xpu_dist_matvec_q8_rowshard(self._h, arr(weights), weight_stride, arr(scales),
                                                          arr(vectors), count, N, K, arr(outputs)))

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.xpu_dist_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
