"""Host-side planning for bulk embedding: length-bucketed padded batches and
their assignment to GPUs.

The reference embeds one document per batch-1 forward (`Gatherer::next`,
src/lib.rs:929-1001; `embed_chunks`, src/lib.rs:1044-1135).  Documents are
independent, so this backend sorts them by token count, packs them into
padded batches of at most `max_tokens` (B * L) tokens and gives each GPU its
own batches: a replica per device, no collective on the data path.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Batch:
    docs: np.ndarray      # document indices, in row order
    L: int                # padded length (longest document of the batch)

    @property
    def padded_tokens(self) -> int:
        return len(self.docs) * self.L


def config4_lengths(n_docs: int = 131072, seed: int = 5, mu: float = 5.0, sigma: float = 0.7,
                    lo: int = 16, hi: int = 512) -> np.ndarray:
    """Document token counts of the bulk-embedding workload:
    clip(round(exp(N(mu, sigma))), lo, hi) from a seeded generator."""
    rng = np.random.default_rng(seed)
    return np.clip(np.rint(np.exp(rng.normal(mu, sigma, n_docs))), lo, hi).astype(np.int32)


def plan_batches(lengths: np.ndarray, max_tokens: int = 16384) -> list[Batch]:
    """Sort by length and cut into batches whose padded size stays within
    max_tokens (a single document longer than max_tokens gets its own batch)."""
    order = np.argsort(lengths, kind="stable")
    out: list[Batch] = []
    start = 0
    n = len(order)
    while start < n:
        end = start + 1
        L = int(lengths[order[start]])
        while end < n:
            L2 = int(lengths[order[end]])
            if (end - start + 1) * L2 > max_tokens:
                break
            L = L2
            end += 1
        out.append(Batch(order[start:end], L))
        start = end
    return out


def lpt_assign(costs, world: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of items with the given
    costs to `world` workers (largest first, each to the least-loaded worker;
    ties to the lowest worker index).  Returns the item indices per worker."""
    loads = np.zeros(world, np.int64)
    owners: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: -costs[i]):
        r = int(np.argmin(loads))
        owners[r].append(i)
        loads[r] += costs[i]
    return owners


def assign_batches(batches: list[Batch], world: int) -> list[list[int]]:
    """LPT assignment of batches to `world` ranks by padded token count.
    Returns the batch indices of each rank."""
    return lpt_assign([b.padded_tokens for b in batches], world)
