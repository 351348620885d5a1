"""Host logic of point-sharded engine groups, on CPU with gloo ranks.

A sharded epoch relies on three facts this file checks without a GPU:
  * the shard rule (Python mirror and the C ABI's cpde_shard_range) tiles every
    sample range exactly once, remainder spread over the first ranks;
  * summing per-shard losses and weight gradients over ranks (the NCCL
    all-reduce of the epoch) reproduces the whole-data epoch, here with the
    float64 oracle on each rank and a gloo all-reduce, world size 2;
  * the first bad sample found by an integer minimum over ranks of
    (global sample, component) keys is the one a single device reports;
and that the NCCL group id reaches every rank through a torch.distributed
broadcast. Tolerance: 1e-12 relative (float64 sums in a different order).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cpde_b200 import native, sharding
from cpde_b200.expressions import quadrature_inputs
from oracle import jets


def test_shard_rule_matches_library_and_tiles_samples():
    for total in (0, 1, 2, 7, 10, 729, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.shard_range(total, r, world) for r in range(world)]
            assert spans == [native.shard_range(total, r, world) for r in range(world)]
            covered = [s for lo, n in spans for s in range(lo, lo + n)] if total < 1000 else None
            if covered is not None:
                assert covered == list(range(total))
            sizes = [n for _, n in spans]
            assert sum(sizes) == total and max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)
    assert sharding.shard_range(10, 0, 4) == (0, 3) and sharding.shard_range(10, 3, 4) == (8, 2)
    with pytest.raises(ValueError):
        sharding.shard_range(5, 2, 2)


def _key(sample, component):
    # same packing as bad_entry_key in cpde_b200/csrc/collectives.hpp
    return (sample << 32) + (component + 2 ** 31)


def _unkey(key):
    return key >> 32, (key & 0xFFFFFFFF) - 2 ** 31


def _problem():
    rng = np.random.default_rng(5)
    table = np.array([(0, 0, 0), (1, 1, 0), (1, 0, 1), (2, 2, 0), (2, 1, 1), (2, 0, 2)], np.int32)
    layers, linear = [2, 16, 16, 1], [1, 0, 0, 1]
    P = 37
    pts = rng.uniform(-1, 1, (P, 2))
    x = quadrature_inputs(pts, table)
    weights = [rng.normal(size=h * (w + 1)) / np.sqrt(w) for w, h in zip(layers[:-1], layers[1:])]
    target = rng.normal(size=(len(table), 1, P))
    mw = rng.uniform(0.5, 1.5, (len(table), 1, P))
    return table, layers, linear, x, weights, target, mw


def _epoch(table, layers, linear, x, weights, target, mw):
    schema = jets.Schema(table[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    loss, dout = jets.matching(acts[-1], target, mw)
    return loss, jets.backward(schema, weights, layers, linear, pre, acts, dout)


def _first_bad(values):
    """(sample, component) of the first non-finite residual, samples first."""
    bad = np.argwhere(~np.isfinite(values.transpose(2, 0, 1).reshape(values.shape[2], -1)))
    return (int(bad[0][0]), int(bad[0][1])) if len(bad) else (2 ** 31 - 1, 2 ** 31 - 1)


def _rank(rank, world, port, queue):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        table, layers, linear, x, weights, target, mw = _problem()
        P = x.shape[2]
        lo, n = sharding.shard_range(P, rank, world)
        part = slice(lo, lo + n)
        loss, grads = _epoch(table, layers, linear, x[..., part], weights, target[..., part], mw[..., part])
        flat = torch.tensor(np.concatenate([[loss]] + grads), dtype=torch.float64)
        dist.all_reduce(flat)
        # a planted non-finite target in two samples: the group minimum of the
        # global keys must name the earlier one
        planted = target.copy()
        planted[3, 0, 30] = np.nan
        planted[1, 0, 12] = np.inf
        residual = planted[..., part] - x[:1, :1, part]
        sample, component = _first_bad(residual)
        key = _key(sample + lo if sample != 2 ** 31 - 1 else sample, component)
        keys = torch.tensor([key], dtype=torch.int64)
        dist.all_reduce(keys, op=dist.ReduceOp.MIN)
        uid = sharding.exchange_id(make_id=lambda: bytes(range(128)))
        queue.put((rank, flat.numpy(), _unkey(int(keys[0])), uid))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_sum_to_the_whole_epoch():
    world = 2
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    table, layers, linear, x, weights, target, mw = _problem()
    loss, grads = _epoch(table, layers, linear, x, weights, target, mw)
    whole = np.concatenate([[loss]] + grads)
    planted = target.copy()
    planted[3, 0, 30] = np.nan
    planted[1, 0, 12] = np.inf
    expected_bad = _first_bad(planted - x[:1, :1, :])
    for rank, summed, bad, uid in results:
        assert np.allclose(summed, whole, rtol=1e-12, atol=1e-12 * np.abs(whole).max())
        assert bad == expected_bad == (12, 1)
        assert uid == bytes(range(128))
    assert np.array_equal(results[0][1], results[1][1])
