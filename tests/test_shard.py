"""Sharded input-split BaB over gloo ranks on the CPU (host logic only): a
synthetic engine with a deterministic per-box closure rule stands in for
the GPU bounds, so the sharded tree must match the single-process tree leaf
for leaf."""
import os
import socket
import types

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vibecheck_nn_b200 import shard
from vibecheck_nn_b200.bab import (BabConfig, LocalState, StepResult, Worklist,
                                   local_iteration)


class SyntheticEngine:
    """Closes a box when a Lipschitz lower bound of f(x) = const + sin(7 x0) +
    cos(5 x1) - 0.5 x2^2 over it is > 0; boxes narrower than ``w_min`` are
    degenerate; others bisect their widest side (lowest index on ties).  A
    box whose centre has f < -``sat_below`` yields that centre as a witness."""

    def __init__(self, batch=64, const=2.6, w_min=1e-3, sat_below=None, budget=120.0,
                 n_in=3):
        self.cfg = BabConfig(types.SimpleNamespace(input_split_batch_size=batch,
                                                   total_timeout=budget))
        self.device = torch.device('cpu')
        self.n_in = n_in
        self.const = const
        self.w_min = w_min
        self.sat_below = sat_below

    def root(self):
        return (torch.full((self.n_in,), -1.0, dtype=torch.float32),
                torch.full((self.n_in,), 1.0, dtype=torch.float32))

    def process(self, xl, xh, n_iter, batch_size=None, timer=None):
        xl64, xh64 = xl.double(), xh.double()
        c = (xl64 + xh64) / 2
        r = (xh64 - xl64) / 2
        f = self.const + torch.sin(7 * c[:, 0]) + torch.cos(5 * c[:, 1]) - 0.5 * c[:, 2] ** 2
        if self.sat_below is not None:
            hit = (f < -self.sat_below).nonzero()
            if hit.numel():
                return StepResult(None, None, 0, 0, c[int(hit[0])].numpy())
        lower = f - 7 * r[:, 0] - 5 * r[:, 1] - r[:, 2] * (c[:, 2].abs() + r[:, 2])
        width = (xh - xl).max(dim=1).values
        closed = lower > 0
        degen = ~closed & (width <= self.w_min)
        keep = ~closed & ~degen
        xl_k, xh_k = xl[keep], xh[keep]
        dim = (xh_k - xl_k).argmax(dim=1)
        mid = (xl_k.gather(1, dim[:, None]) + xh_k.gather(1, dim[:, None])) / 2
        lo_h = xh_k.clone()
        lo_h.scatter_(1, dim[:, None], mid)
        hi_l = xl_k.clone()
        hi_l.scatter_(1, dim[:, None], mid)
        n = int(keep.sum())
        return StepResult((xl_k, lo_h), (hi_l, xh_k), n, int(degen.sum()))


def single_run(engine):
    st = LocalState(Worklist(*engine.root()), engine.cfg.batch_size)
    while st.wl:
        local_iteration(engine, st)
        if st.witness is not None:
            return 'sat', st
    return ('verified' if st.n_open == 0 else 'unknown'), st


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, kwargs, run_kwargs, out):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=__import__('datetime').timedelta(seconds=60))
    try:
        eng = SyntheticEngine(**kwargs)
        verdict, det = shard.input_split_sharded(eng, **run_kwargs)
        w = det.get('witness')
        out.put((rank, verdict, det['batched_n_leaves'], det['shard_leaves'],
                 det.get('shard_transfers', 0), None if w is None else list(w)))
    finally:
        dist.destroy_process_group()


def sharded_run(world, kwargs, run_kwargs=None):
    ctx = mp.get_context('spawn')
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), kwargs, run_kwargs or {}, q),
                       nprocs=world, join=True, start_method='spawn')
    res = sorted(q.get() for _ in range(world))
    return res


def test_rebalance_plan():
    assert shard.rebalance_plan([10, 10], 4) == []
    assert shard.rebalance_plan([100, 0], 4) == [(0, 1, 50)]
    assert shard.rebalance_plan([0, 100, 30, 31], 4) == [(1, 0, 50)]
    plan = shard.rebalance_plan([200, 0, 180, 1], 8)
    assert plan == [(0, 1, 100), (2, 3, 89)]


def test_deal_round_robin():
    wl = Worklist.empty()
    wl.push(torch.arange(10.).reshape(5, 2), torch.arange(10.).reshape(5, 2) + 1)
    parts = []
    for r in range(3):
        w2 = Worklist.empty()
        w2.push(torch.arange(10.).reshape(5, 2), torch.arange(10.).reshape(5, 2) + 1)
        d = shard.deal(w2, r, 3, 2, 'cpu')
        parts.append(d.pop(d.size())[0][:, 0].tolist() if d.size() else [])
    assert parts == [[0.0, 6.0], [2.0, 8.0], [4.0]]


@pytest.mark.parametrize('world', [2, 3])
def test_sharded_tree_matches_single_process(world):
    kw = dict(batch=64)
    verdict, st = single_run(SyntheticEngine(**kw))
    assert verdict == 'verified' and st.n_leaves > 2000  # a tree worth sharding
    res = sharded_run(world, kw, dict(per_rank=8, sync_every=4))
    for rank, v, n, per, _, _ in res:
        assert v == verdict
        assert n == st.n_leaves
        assert sum(per) == st.n_leaves
        assert min(per) > 0  # every rank did work


def test_sharded_rebalances_and_degenerate_leaves_stay_open():
    kw = dict(batch=16, const=2.45, w_min=0.05)
    verdict, st = single_run(SyntheticEngine(**kw))
    assert verdict == 'unknown' and st.n_open > 0
    res = sharded_run(2, kw, dict(per_rank=1, sync_every=2))
    for _, v, n, _, transfers, _ in res:
        assert v == 'unknown' and n == st.n_leaves
    assert res[0][4] == res[1][4]  # every rank saw the same plans


def test_sharded_sat_broadcasts_witness():
    kw = dict(batch=32, const=2.0, w_min=0.05, sat_below=0.3)
    verdict, st = single_run(SyntheticEngine(**kw))
    assert verdict == 'sat'
    res = sharded_run(2, kw, dict(per_rank=4, sync_every=2))
    wits = [tuple(r[5]) for r in res]
    assert all(r[1] == 'sat' for r in res)
    assert wits[0] == wits[1]
    x = np.asarray(wits[0])
    assert 2.0 + np.sin(7 * x[0]) + np.cos(5 * x[1]) - 0.5 * x[2] ** 2 < -0.3


def test_sharded_global_timeout_is_consistent():
    res = sharded_run(2, dict(batch=8, budget=0.0), dict(per_rank=1, sync_every=1))
    assert {r[1] for r in res} == {'unknown'}
