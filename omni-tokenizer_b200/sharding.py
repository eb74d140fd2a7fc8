"""Item sharding across GPUs for the batched hot path (one process per GPU).

The reference scales by running one Tokenizer per GPU
(python/omni_tokenizer/runtime.py:56, ``omni_model_load(..., device=N)``).  Items
(images, audio segments) are independent, so a batch splits across ranks with
no exchange step on the data path; only the host gathers the per-item results
at the end.

* :func:`even_split` -- contiguous near-equal ranges, for fixed-size items
  (SigLIP-shaped image batches).
* :func:`balanced_bins` -- greedy longest-processing-time-first assignment of
  variable-length items to the least-loaded rank, cost ``L**2`` by default (the
  attention work of a segment of L tokens), for varlen audio batches.  Each
  rank's indices come back in their original order.
* :func:`gather_results` -- host-side reassembly of per-rank results in the
  original item order over a ``torch.distributed`` process group (CPU objects;
  works with ``gloo`` and ``nccl`` groups alike).

Rank failures surface as exceptions: a rank that never reaches the gather makes
the others' collective fail after the process group's timeout.
"""

from __future__ import annotations

from typing import Callable, Iterable, List, Sequence


def even_split(n_items: int, world: int) -> List[range]:
    """Contiguous ranges covering ``range(n_items)``; sizes differ by at most one."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if n_items < 0:
        raise ValueError("n_items must be >= 0")
    base, extra = divmod(n_items, world)
    out, start = [], 0
    for r in range(world):
        size = base + (1 if r < extra else 0)
        out.append(range(start, start + size))
        start += size
    return out


def balanced_bins(lengths: Sequence[int], world: int,
                  cost: Callable[[int], float] = lambda n: float(n) * float(n)) -> List[List[int]]:
    """Assign item indices to ``world`` bins, longest first, each to the least-loaded bin.

    Ties (equal cost, equal load) resolve to the lower index, so the result is
    deterministic.  Returns per-bin index lists sorted ascending.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-cost(int(lengths[i])), i))
    loads = [0.0] * world
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        b = min(range(world), key=lambda k: (loads[k], k))
        bins[b].append(i)
        loads[b] += cost(int(lengths[i]))
    return [sorted(b) for b in bins]


def bin_loads(lengths: Sequence[int], bins: Iterable[Sequence[int]],
              cost: Callable[[int], float] = lambda n: float(n) * float(n)) -> List[float]:
    """Total cost per bin (for reporting the balance of a partition)."""
    return [sum(cost(int(lengths[i])) for i in b) for b in bins]


def gather_results(indices: Sequence[int], results: Sequence, n_items: int, group=None) -> list:
    """Reassemble ``results[k]`` (this rank's result for item ``indices[k]``) into a
    list of all ``n_items`` results, in item order, on every rank.

    Without an initialised process group this is the single-process case and the
    local results must already cover every item.
    """
    if len(indices) != len(results):
        raise ValueError("indices and results differ in length")
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        world = dist.get_world_size(group)
        parts = [None] * world
        dist.all_gather_object(parts, (list(indices), list(results)), group=group)
    else:
        parts = [(list(indices), list(results))]
    out = [None] * n_items
    seen = 0
    for idx, res in parts:
        for i, r in zip(idx, res):
            if out[i] is not None:
                raise ValueError(f"item {i} produced by two ranks")
            out[i] = r
            seen += 1
    if seen != n_items:
        raise ValueError(f"gathered {seen} of {n_items} items")
    return out
