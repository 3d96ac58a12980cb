"""Host logic of the multi-GPU run: which machines a rank owns, and the one collective.

Machines are independent, so ranks split them with no per-step exchange.  The run ends with one
all-gather of the per-machine state checksums (FNV-1a 64 of registers, PC and RAM, computed on
the device by ``qx_checksums``), XOR-combined into a single run checksum that does not depend on
the number of ranks.
"""

from __future__ import annotations

import numpy as np


def shard(machines: int, world: int, rank: int, weak: bool = False, seed: int = 1000) -> tuple[int, int]:
    """(machines on this rank, seed of its first program).  Strong: ``machines`` split evenly over
    the ranks (programs seed .. seed + machines - 1 overall); weak: every rank runs ``machines``."""
    if weak:
        b = machines
    else:
        if machines % world:
            raise ValueError(f"{machines} machines do not split evenly over {world} ranks")
        b = machines // world
    return b, seed + rank * b


def gather_checksums(sums, dist=None):
    """All ranks' checksums in rank order (one collective; ``dist`` None: a single rank)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return sums
    import torch

    world = dist.get_world_size()
    if dist.get_backend() == "nccl":
        out = torch.empty(world * sums.numel(), dtype=sums.dtype, device=sums.device)
        dist.all_gather_into_tensor(out, sums)
        return out
    parts = [torch.empty_like(sums) for _ in range(world)]
    dist.all_gather(parts, sums)
    return torch.cat(parts)


def combine(sums) -> int:
    """XOR of every machine's 64-bit checksum."""
    a = sums.cpu().numpy() if hasattr(sums, "cpu") else np.asarray(sums)
    return int(np.bitwise_xor.reduce(a.view(np.uint64))) if a.size else 0
