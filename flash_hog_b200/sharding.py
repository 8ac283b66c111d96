"""Batch x heads sharding of the attention op across GPUs (no communication).

Re-expresses the partitioning rule the reference left commented out
(``flash_hog/jax/_pallas_gpu.py:75-83``): only the ``batch`` and ``heads``
factors are sharded; ``queries``, ``keys`` and ``hidden`` stay whole on every
device. Every (batch, head) pair is independent in the forward, backward and
double backward, so a rank that owns a slice computes exactly the matching
slice of the unsharded result with no collective.

``sharded_flash_bwdbwd`` is the caller: one process per GPU (torchrun), each
given the global batch, runs its own slice on its GPU's kernels and returns it
(optionally all-gathered into the global result over the process group).
"""

from __future__ import annotations

import dataclasses

import torch


@dataclasses.dataclass(frozen=True)
class BatchHeadsSharding:
    """Splits (batch, heads) over ``world`` ranks as a ``batch_parts x head_parts`` grid.

    Batch is split first (largest divisor of ``world`` that divides ``batch``), the
    remaining factor splits heads; ``ValueError`` if ``world`` cannot be factored so.
    With grouped-query attention (``kv_heads`` < ``heads``) the key/value heads are
    split by the same factor, so each rank keeps whole query groups: query head n
    uses key head n // (heads // kv_heads) on the same rank.
    """

    batch: int
    heads: int
    world: int
    kv_heads: int | None = None

    def __post_init__(self):
        kv = self.heads if self.kv_heads is None else self.kv_heads
        if self.world < 1 or self.batch < 1 or self.heads < 1 or kv < 1 or self.heads % kv:
            raise ValueError("batch, heads, kv_heads and world must be >= 1, heads a multiple of kv_heads")
        bp = max(d for d in range(1, self.world + 1) if self.world % d == 0 and self.batch % d == 0)
        hp = self.world // bp
        if self.heads % hp or kv % hp:
            raise ValueError(f"cannot shard batch={self.batch} x heads={self.heads} (kv_heads={kv}) "
                             f"over {self.world} ranks")
        object.__setattr__(self, "batch_parts", bp)
        object.__setattr__(self, "head_parts", hp)
        object.__setattr__(self, "kv", kv)

    def slices(self, rank: int):
        """(batch slice, head slice) owned by ``rank``."""
        if not 0 <= rank < self.world:
            raise ValueError("rank out of range")
        bi, hi = divmod(rank, self.head_parts)
        nb, nh = self.batch // self.batch_parts, self.heads // self.head_parts
        return slice(bi * nb, (bi + 1) * nb), slice(hi * nh, (hi + 1) * nh)

    def kv_slice(self, rank: int):
        """Key/value head slice owned by ``rank`` (the query heads' groups)."""
        _, sh = self.slices(rank)
        g = self.heads // self.kv
        return slice(sh.start // g, sh.stop // g)

    def shard(self, x, rank: int):
        """This rank's view of a query-side BTNH tensor."""
        sb, sh = self.slices(rank)
        return x[sb, :, sh]

    def shard_kv(self, x, rank: int):
        """This rank's view of a key-side BTNH tensor."""
        sb, _ = self.slices(rank)
        return x[sb, :, self.kv_slice(rank)]

    def shard_stats(self, v, rank: int):
        """This rank's view of a (B, N, T) statistics vector (e.g. the log-sum-exp)."""
        sb, sh = self.slices(rank)
        return v[sb, sh]


def _rank_world(group):
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def sharded_flash_bwdbwd(Q, K, V, O, dO, ddQ, ddK, ddV, L, mask_type=None, scale=None, *, rank=None, world=None,
                         device=None, gather=False, group=None):
    """The double backward of a global batch, sharded over batch x heads.

    Every rank passes the same global BTNH tensors (on the host or on any device)
    and the global log-sum-exp ``L`` (B, N, T). The rank copies its slice to
    ``device`` (default: the current CUDA device), runs ``flash_bwdbwd`` on it --
    the sm_100a kernels, no collective -- and returns ``(dQ2, dK2, dV2, ddO)`` for
    its slice together with the ``BatchHeadsSharding`` that says which slice that
    is. ``rank``/``world`` default to the process group's (0/1 without one).

    With ``gather=True`` the slices are all-gathered over ``group`` (NCCL under
    torchrun) and every rank returns the global result: a collective that serves
    callers who need the whole result everywhere, not the computation.
    """
    from flash_hog_b200._attention_impl import MaskType
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    mask_type = MaskType.NO_MASK if mask_type is None else mask_type
    r, w = _rank_world(group)
    rank = r if rank is None else rank
    world = w if world is None else world
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    sh = BatchHeadsSharding(Q.shape[0], Q.shape[2], world, K.shape[2])
    q_side = [sh.shard(x, rank) for x in (Q, O, dO, ddQ)]
    k_side = [sh.shard_kv(x, rank) for x in (K, V, ddK, ddV)]
    q, o, do, ddq = (x.to(device, non_blocking=True).contiguous() for x in q_side)
    k, v, ddk, ddv = (x.to(device, non_blocking=True).contiguous() for x in k_side)
    lse = sh.shard_stats(L, rank).to(device, non_blocking=True).contiguous()
    local = flash_bwdbwd(q, k, v, o, do, ddq, ddk, ddv, lse, mask_type=mask_type, scale=scale)
    if not gather:
        return local, sh
    return _gather(local, sh, world, group), sh


def _gather(local, sh: BatchHeadsSharding, world: int, group):
    """All-gathers every rank's (dQ2, dK2, dV2, ddO) slice into the global tensors."""
    import torch.distributed as dist

    out = []
    for i, t in enumerate(local):
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous(), group=group)
        b = t.shape[0] * sh.batch_parts
        h = t.shape[2] * sh.head_parts
        full = t.new_empty((b, t.shape[1], h, t.shape[3]))
        for r, p in enumerate(parts):
            sb, _ = sh.slices(r)
            hs = sh.kv_slice(r) if i in (1, 2) else sh.slices(r)[1]
            full[sb, :, hs] = p
        out.append(full)
    return tuple(out)
