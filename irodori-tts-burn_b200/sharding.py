"""Utterance-level sharding across GPUs (no collective on the data path).

Independent utterances are assigned to ranks by greedy longest-processing-
time-first bin packing on a per-utterance cost model of the DiT work
(row-forwards x tokens x (per-token GEMM work + attention over the valid
keys)).  Each rank then samples its bin as one ragged batch.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple


def utterance_cost(seq_len: int, text_len: int, ref_frames: int, model_dim: int = 2048, layers: int = 24,
                   hidden: int = 5888, cfg_rows: float = 1.5) -> float:
    """FLOPs of one utterance's sampling per step (relative units):
    S * [L * (gemm_per_token + 4 * D * Skv)] * rows, with Skv = S + text + ref + 1."""
    D, F = model_dim, hidden
    gemm = 2 * D * (4 * D) + 2 * D * D + 2 * D * (2 * F) + 2 * F * D
    skv = seq_len + text_len + ref_frames + 1
    return seq_len * layers * (gemm + 4 * D * skv) * cfg_rows


def lpt_bins(costs: Sequence[float], nbins: int) -> List[List[int]]:
    """Greedy LPT: sort by decreasing cost, put each item into the currently
    lightest bin (ties -> lowest bin index).  Deterministic."""
    if nbins <= 0:
        raise ValueError("nbins must be > 0")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0.0] * nbins
    bins: List[List[int]] = [[] for _ in range(nbins)]
    for i in order:
        b = min(range(nbins), key=lambda j: (loads[j], j))
        bins[b].append(i)
        loads[b] += costs[i]
    return [sorted(b) for b in bins]


def shard_for_rank(costs: Sequence[float], rank: int, world: int) -> List[int]:
    return lpt_bins(costs, world)[rank]


def imbalance(costs: Sequence[float], bins: List[List[int]]) -> Tuple[float, float]:
    """(max bin load / mean bin load, max load)."""
    loads = [sum(costs[i] for i in b) for b in bins]
    mean = sum(loads) / len(loads)
    return (max(loads) / mean if mean > 0 else 1.0), max(loads)


# ---------------------------------------------------------------------------
# Rank plumbing shared by bench.py and the multi-rank tests
# ---------------------------------------------------------------------------

def init_rank_group(backend: str, timeout_s: float, device=None):
    """Join the job's process group (env:// rendezvous: RANK, WORLD_SIZE,
    MASTER_ADDR, MASTER_PORT) with a short collective timeout, so that the
    surviving ranks of a job whose rank died end their next collective with an
    error instead of waiting for it.  Returns the ``torch.distributed``
    module."""
    import datetime

    import torch.distributed as dist
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist


def max_over_ranks(dist, value: float, device=None) -> float:
    """Barrier, then the maximum of ``value`` over all ranks (the timing
    reduction of a multi-GPU step: the job takes as long as its slowest
    rank).  Raises if a rank has left the job."""
    import torch
    dist.barrier()
    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
