"""Partition of an operator call across ranks (one process per GPU).

All three recurrent operators are independent per batch row, per channel
(SelectiveScanFn) and per head (Mamba3SisoFn, GatedDeltaNet2Fn); GatedDeltaNet2Fn
is also independent per value column, given the key-side inputs. A call over a
global batch therefore splits into disjoint shards with no exchange between
them: each rank runs the same operator on its own slice, and the global output
is the concatenation of the shards' outputs along the split axis. The data path
has no collective; the only collectives are the host-side barrier and the
max-over-ranks reduction of the timings, plus an optional gather used to check
results (never inside a timed region).

Layouts follow the reference operators (row-major, batch first):
  SelectiveScanFn   u, delta, z, out [B, D, L]; B, C [B, G, N, L] (variable)
  GatedDeltaNet2Fn  q, k, g, beta [B, T, H, K]; v, w, out [B, T, H, V];
                    initial_state [B, H, K, V]
  Mamba3SisoFn      Q, K [B, T, G, N]; V, Z, out [B, T, H, P];
                    ADT, DT, Trap [B, H, T]; Angles [B, T, H, A]
"""

from __future__ import annotations

# Per-rank input seed: rank r's batch block is generated with
# seed + RANK_SEED_STRIDE * r, so every rank builds its own block without
# materialising the others. (The benchmark's ranks also draw their shared
# per-channel / per-head parameters from their own seed, i.e. each runs an
# independent call of the per-GPU shape; the multi-rank tests take those
# parameters from rank 0 so that the shards form one global call.)
RANK_SEED_STRIDE = 1000

# Batch axis of every batch-carrying input / the output, per operator.
_BATCH_AXIS = {
    "ss": {"u": 0, "delta": 0, "B": 0, "C": 0, "z": 0, "out": 0},
    "gdn": {"q": 0, "k": 0, "v": 0, "g": 0, "beta": 0, "w": 0, "initial_state": 0, "out": 0},
    "m3": {"Q": 0, "K": 0, "V": 0, "ADT": 0, "DT": 0, "Trap": 0, "Angles": 0, "Z": 0, "out": 0},
}


def rank_seed(seed: int, rank: int) -> int:
    return seed + RANK_SEED_STRIDE * rank


def block_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced split of n units: rank r gets [start, stop)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _slice_axis(a, axis, start, stop):
    index = [slice(None)] * a.ndim
    index[axis] = slice(start, stop)
    return a[tuple(index)]


def shard_batch(op: str, inputs: dict, world: int, rank: int) -> dict:
    """Rank `rank`'s batch slice of a global input dict (numpy or torch arrays).

    Inputs without a batch axis (A, D, delta_bias, Q_bias, K_bias, scale, ...)
    are shared by every shard and passed through unchanged."""
    axes = _BATCH_AXIS[op]
    batch = next(inputs[k].shape[axes[k]] for k in axes if inputs.get(k) is not None and k != "out")
    start, stop = block_range(batch, world, rank)
    out = {}
    for k, a in inputs.items():
        batched = a is not None and k in axes
        if op == "ss" and k in ("B", "C") and batched:
            batched = a.ndim >= 3  # constant B / C are [D, N], shared by every batch row
        out[k] = _slice_axis(a, axes[k], start, stop) if batched else a
    return out


# Head (GatedDeltaNet2Fn, Mamba3SisoFn) or channel (SelectiveScanFn) axis of
# every input that carries one; the other inputs are shared by all shards.
_UNIT_AXIS = {
    "ss": {"u": 1, "delta": 1, "z": 1, "A": 0, "D": 0, "delta_bias": 0, "out": 1},
    "gdn": {"q": 2, "k": 2, "v": 2, "g": 2, "beta": 2, "w": 2, "initial_state": 1, "out": 2},
    "m3": {"V": 2, "Z": 2, "ADT": 1, "DT": 1, "Trap": 1, "Q_bias": 0, "K_bias": 0, "Angles": 2, "D": 0,
           "out": 2},
}


def shard_units(op: str, inputs: dict, world: int, rank: int, prefer: str = "batch") -> tuple[dict, str]:
    """Rank `rank`'s share of one global call, split over batch rows when the
    batch divides evenly over the ranks (and `prefer` is "batch"), otherwise
    over channels (SelectiveScanFn) or heads (the other two). Returns (inputs,
    axis name).

    Channel and head shards keep every batch row: the per-channel / per-head
    parameters (A, D, delta_bias; Q_bias, K_bias, D) are sliced with them, and
    the inputs shared across channels or heads (SelectiveScanFn's B and C,
    Mamba3SisoFn's Q and K with one Q/K group) are passed whole. A Mamba-3
    head split needs nheads_qk == 1 or a split that keeps whole Q/K groups."""
    axes = _BATCH_AXIS[op]
    batch = next(inputs[k].shape[axes[k]] for k in axes if inputs.get(k) is not None and k != "out")
    if prefer == "batch" and batch % world == 0:
        return shard_batch(op, inputs, world, rank), "batch"
    uax = _UNIT_AXIS[op]
    probe = {"ss": "u", "gdn": "q", "m3": "V"}[op]
    n = inputs[probe].shape[uax[probe]]
    if op == "m3" and inputs["Q"].shape[2] != 1:
        raise ValueError("Mamba3SisoFn head shards need nheads_qk == 1")
    start, stop = block_range(n, world, rank)
    out = {}
    for k, a in inputs.items():
        sliced = a is not None and k in uax and hasattr(a, "ndim") and a.ndim > uax[k]
        out[k] = _slice_axis(a, uax[k], start, stop) if sliced else a
    return out, "channel" if op == "ss" else "head"


def shard_value_columns(inputs: dict, world: int, rank: int) -> dict:
    """GatedDeltaNet2Fn split over value columns: v, w and initial_state are
    sliced on V; the key-side inputs are shared (each shard re-reads them)."""
    V = inputs["v"].shape[3]
    start, stop = block_range(V, world, rank)
    out = dict(inputs)
    out["v"] = inputs["v"][..., start:stop]
    out["w"] = inputs["w"][..., start:stop]
    if inputs.get("initial_state") is not None:
        out["initial_state"] = inputs["initial_state"][..., start:stop]
    return out


def concat_shards(parts, axis: int):
    """Global output from the shards' outputs, in rank order."""
    first = parts[0]
    if hasattr(first, "detach"):
        import torch

        return torch.cat(list(parts), dim=axis)
    import numpy as np

    return np.concatenate(list(parts), axis=axis)


def max_over_ranks(value: float, device=None) -> float:
    """All-reduce MAX of a per-rank timing (the job takes as long as its slowest rank)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_shards(part, axis: int, device=None):
    """All-gather every rank's output shard and concatenate them (for checking
    results outside the timed region; shards must have equal shapes)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return part
    t = part if hasattr(part, "detach") else torch.from_numpy(part)
    if device is not None:
        t = t.to(device)
    bufs = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(bufs, t.contiguous())
    return torch.cat(bufs, dim=axis)
