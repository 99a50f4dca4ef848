"""Multi-rank path on CPU: two `gloo` ranks run disjoint shards of one call.

Each rank builds its own seeded batch block (as `bench.py --gpus N` does on
each GPU), runs the CPU restatement of the operator on it, and the gathered
shards must equal the single-process result over the concatenated global
input bit for bit (the operators are independent per batch row, head and
value column). The same ranks check the max-over-ranks timing reduction and
the value-column split of GatedDeltaNet2Fn.
"""

import os
import socket

import numpy as np
import pytest

from conftest import load_package

xm = load_package()
from xmetai_onnx_plugins_b200 import shard  # noqa: E402
from xmetai_onnx_plugins_b200 import workloads as W  # noqa: E402

WORLD = 2
SS_BLOCK = dict(batch=1, dim=32, dstate=16, seqlen=64)
GDN_BLOCK = dict(B=1, T=24, H=2, K=32, V=16)
M3_BLOCK = dict(B=1, T=40, H=2, G=1, N=16, P=8, A=8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gen(op, seed):
    if op == "ss":
        return W.ss_inputs(seed=seed, **SS_BLOCK)
    if op == "gdn":
        return W.gdn_inputs(seed=seed, **GDN_BLOCK)
    return W.m3_inputs(seed=seed, **M3_BLOCK)


def _block(op, rank):
    """Rank `rank`'s batch block: batch-carrying inputs from the rank's seed,
    the shared per-channel / per-head parameters from rank 0's."""
    x = _gen(op, shard.rank_seed(7, rank))
    shared = _gen(op, shard.rank_seed(7, 0))
    for k, a in shared.items():
        if k not in shard._BATCH_AXIS[op] or (op == "ss" and isinstance(a, np.ndarray) and a.ndim < 3):
            x[k] = a
    return x


def _run_oracle(op, x):
    import oracle

    if op == "ss":
        return oracle.ss(*[x[k] for k in W.SS_ORDER], softplus=True, precision="f32", nthreads=1)
    if op == "gdn":
        return oracle.gdn(*[x[k] for k in W.GDN_ORDER], scale=x["scale"], precision="f32", nthreads=1)
    return oracle.m3(*[x[k] for k in W.M3_ORDER], precision="f32", nthreads=1)


def _global(op):
    blocks = [_block(op, r) for r in range(WORLD)]
    out = {}
    for k, a in blocks[0].items():
        if isinstance(a, np.ndarray) and k in shard._BATCH_AXIS[op] and not (op == "ss" and a.ndim < 3):
            out[k] = np.concatenate([b[k] for b in blocks], axis=0)
        else:
            out[k] = a
    return out


def _worker(rank, port, result_dir):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        # timing reduction: every rank sees the slowest rank's figure
        got = shard.max_over_ranks(1.5 + rank)
        assert got == 1.5 + (WORLD - 1), got
        for op in ("ss", "gdn", "m3"):
            part = _run_oracle(op, _block(op, rank))
            full = shard.gather_shards(torch.from_numpy(np.ascontiguousarray(part)), axis=0)
            if rank == 0:
                np.save(os.path.join(result_dir, f"{op}_gathered.npy"), full.numpy())
        # a batch-1 call split over channels (SS) or heads (GDN, M3), as
        # `bench.py --gpus N` splits a configuration whose batch N does not divide
        for op in ("ss", "gdn", "m3"):
            part, axis = shard.shard_units(op, _gen(op, 7), WORLD, rank)
            assert axis == ("channel" if op == "ss" else "head")
            out = _run_oracle(op, part)
            ax = 1 if op == "ss" else 2
            full = shard.gather_shards(torch.from_numpy(np.ascontiguousarray(out)), axis=ax)
            if rank == 0:
                np.save(os.path.join(result_dir, f"{op}_units.npy"), full.numpy())
        # value-column split of one GDN call: each rank owns half of V
        g = _global("gdn")
        part = _run_oracle("gdn", shard.shard_value_columns(g, WORLD, rank))
        full = shard.gather_shards(torch.from_numpy(np.ascontiguousarray(part)).movedim(3, 0), axis=0)
        if rank == 0:
            np.save(os.path.join(result_dir, "gdn_vsplit.npy"), full.movedim(0, 3).contiguous().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_block_range_covers_units():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [shard.block_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.block_range(4, 2, 2)


def test_shard_batch_slices_blocks():
    g = _global("ss")
    for r in range(WORLD):
        s = shard.shard_batch("ss", g, WORLD, r)
        b = _block("ss", r)
        for k in W.SS_ORDER:
            if b[k] is None:
                assert s[k] is None
            else:
                np.testing.assert_array_equal(s[k], b[k])


def test_two_gloo_ranks_match_single_process(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True, start_method="spawn")
    for op in ("ss", "gdn", "m3"):
        want = _run_oracle(op, _global(op))
        got = np.load(tmp_path / f"{op}_gathered.npy")
        np.testing.assert_array_equal(got, want)
    want = _run_oracle("gdn", _global("gdn"))
    np.testing.assert_array_equal(np.load(tmp_path / "gdn_vsplit.npy"), want)
    for op in ("ss", "gdn", "m3"):
        np.testing.assert_array_equal(np.load(tmp_path / f"{op}_units.npy"), _run_oracle(op, _gen(op, 7)))


def test_shard_units_splits_batch_when_it_divides_else_units():
    """Three ranks over a batch of 2: channel / head shards that cover every
    unit once, with the per-unit parameters sliced alongside."""
    for op in ("ss", "gdn", "m3"):
        x = _global(op)
        parts = [shard.shard_units(op, x, 3, r) for r in range(3)]
        assert {a for _, a in parts} == {"channel" if op == "ss" else "head"}
        want = _run_oracle(op, x)
        ax = 1 if op == "ss" else 2
        probe = {"ss": "u", "gdn": "q", "m3": "V"}[op]
        assert sum(p[probe].shape[ax] for p, _ in parts) == x[probe].shape[ax]
        got = np.concatenate([_run_oracle(op, p) for p, _ in parts if p[probe].shape[ax] > 0], axis=ax)
        np.testing.assert_array_equal(got, want)
        assert shard.shard_units(op, x, 2, 1)[1] == "batch"
        # a unit split asked for although the batch divides (the Mamba-3 batch-32 sweep over heads)
        parts = [shard.shard_units(op, x, 2, r, prefer="unit") for r in range(2)]
        assert {a for _, a in parts} == {"channel" if op == "ss" else "head"}
        got = np.concatenate([_run_oracle(op, p) for p, _ in parts], axis=ax)
        np.testing.assert_array_equal(got, want)
