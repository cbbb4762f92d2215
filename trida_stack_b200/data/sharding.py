"""Record-level sharding shared by the streaming datasets.

A DataLoader worker of a rank reads shard ``rank * workers + worker`` of ``world * workers``
(``worker_shard``).  ``EpochSampler`` deals an indexable collection of n records to the shards:
every epoch draws a fresh permutation from (seed, epoch), and shard s takes the positions s,
s + nshard, ... of it, wrapping around so that every shard gets ceil(n / nshard) records per epoch
(all ranks then run the same number of steps even when n is not a multiple of the shard count).
"""
import hashlib
import random

from torch.utils.data import get_worker_info


def worker_shard(rank, world):
    """(shard, number of shards) of the calling DataLoader worker of ``rank`` in ``world``."""
    info = get_worker_info()
    wid, nw = (info.id, info.num_workers) if info is not None else (0, 1)
    return rank * nw + wid, world * nw


def mix_seed(*parts):
    """A 64-bit seed from any printable parts (stable across processes and Python versions)."""
    return int.from_bytes(hashlib.sha256(":".join(map(str, parts)).encode()).digest()[:8], "little")


class EpochSampler:
    """Endless (epoch, record index) stream of one shard."""

    def __init__(self, n, shard, nshard, seed):
        if n <= 0:
            raise ValueError("nothing to sample")
        self.n, self.shard, self.nshard, self.seed = n, shard, nshard, seed

    def epoch(self, epoch):
        perm = list(range(self.n))
        random.Random(mix_seed(self.seed, "order", epoch)).shuffle(perm)
        per_shard = -(-self.n // self.nshard)
        return [perm[(self.shard + j * self.nshard) % self.n] for j in range(per_shard)]

    def __iter__(self):
        e = 0
        while True:
            for idx in self.epoch(e):
                yield e, idx
            e += 1
