"""Batch x heads sharding of the attention op across GPUs (no communication).

Re-expresses the partitioning rule the reference left commented out
(``flash_hog/jax/_pallas_gpu.py:75-83``): only the ``batch`` and ``heads``
factors are sharded; ``queries``, ``keys`` and ``hidden`` stay whole on every
device. Every (batch, head) pair is independent in the forward, backward and
double backward, so a rank that owns a slice computes exactly the matching
slice of the unsharded result with no collective.
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class BatchHeadsSharding:
    """Splits (batch, heads) over ``world`` ranks as a ``batch_parts x head_parts`` grid.

    Batch is split first (largest divisor of ``world`` that divides ``batch``), the
    remaining factor splits heads; ``ValueError`` if ``world`` cannot be factored so.
    """

    batch: int
    heads: int
    world: int

    def __post_init__(self):
        if self.world < 1 or self.batch < 1 or self.heads < 1:
            raise ValueError("batch, heads and world must be >= 1")
        bp = max(d for d in range(1, self.world + 1) if self.world % d == 0 and self.batch % d == 0)
        hp = self.world // bp
        if self.heads % hp:
            raise ValueError(f"cannot shard batch={self.batch} x heads={self.heads} over {self.world} ranks")
        object.__setattr__(self, "batch_parts", bp)
        object.__setattr__(self, "head_parts", hp)

    def slices(self, rank: int):
        """(batch slice, head slice) owned by ``rank``."""
        if not 0 <= rank < self.world:
            raise ValueError("rank out of range")
        bi, hi = divmod(rank, self.head_parts)
        nb, nh = self.batch // self.batch_parts, self.heads // self.head_parts
        return slice(bi * nb, (bi + 1) * nb), slice(hi * nh, (hi + 1) * nh)

    def shard(self, x, rank: int):
        """This rank's view of a BTNH tensor."""
        sb, sh = self.slices(rank)
        return x[sb, :, sh]

    def shard_stats(self, v, rank: int):
        """This rank's view of a (B, N, T) statistics vector (e.g. the log-sum-exp)."""
        sb, sh = self.slices(rank)
        return v[sb, sh]
