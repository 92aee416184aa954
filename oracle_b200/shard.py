"""Row sharding of weight matrices over the ranks of one node.

Every output row of a matvec (or GEMM) depends on its own weight row only, so a
matrix of N rows is split into `world` contiguous row ranges of equal size,
rank r owning rows [r * N / world, (r + 1) * N / world).  Each rank computes
its rows; one all-gather of the per-rank outputs (NCCL over NVLink) gives every
rank the whole output, in row order, bit-identical to one GPU.  Several
matrices of one step are packed into one per-rank buffer so that a single
all-gather serves them all:

    pack on rank r   = [y_0[rows of r] | y_1[rows of r] | ...]
    all-gather       -> gathered[r] = pack on rank r
    y_i              = concat over r of gathered[r][off_i : off_i + n_i / world]

This mirrors the north star's partitioning (weights row-wise by output
feature; NCCL only for the per-layer exchange of activations).  The layout
helpers here are plain Python so that they are tested on CPU (gloo ranks) as
well as used by the GPU benchmark.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class RowShard:
    rows: int        # rows of the whole matrix
    world: int
    rank: int

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a world of {self.world}")
        if self.rows % self.world:
            raise ValueError(f"{self.rows} rows do not split evenly over {self.world} ranks")

    @property
    def local_rows(self) -> int:
        return self.rows // self.world

    @property
    def begin(self) -> int:
        return self.rank * self.local_rows

    @property
    def end(self) -> int:
        return self.begin + self.local_rows

    def weight_slice(self, w: np.ndarray) -> np.ndarray:
        """This rank's rows of a (rows, row_bytes) GGML matrix."""
        if w.shape[0] != self.rows:
            raise ValueError("matrix row count does not match the shard plan")
        return w[self.begin:self.end]


class PackPlan:
    """Offsets of several row-sharded outputs inside one per-rank buffer."""

    def __init__(self, rows_per_matrix, world: int, rank: int):
        self.shards = [RowShard(n, world, rank) for n in rows_per_matrix]
        self.world = world
        self.offsets = []
        off = 0
        for s in self.shards:
            self.offsets.append(off)
            off += s.local_rows
        self.pack_len = off

    def unpack(self, gathered: np.ndarray) -> list[np.ndarray]:
        """Whole outputs from the all-gathered buffer (world x pack_len)."""
        g = np.asarray(gathered).reshape(self.world, self.pack_len)
        return [g[:, o:o + s.local_rows].reshape(-1) for o, s in zip(self.offsets, self.shards)]
