"""Sharded input-split BaB on GPUs over NCCL: the reference's cfg1 leaf count
on one rank, and on two GPUs when the box has them."""
import datetime
import os
import socket
import types

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_golden
from vibecheck_nn_b200 import shard, workloads as wk
from vibecheck_nn_b200.bab import LinearSpec

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _cfg1_problem(seed, device):
    w = wk.cfg1(seed)
    gg = wk.mlp_gg(w['layers'], device)
    spec = LinearSpec(w['xl'], w['xh'], [[('pair', 1, 0)]])
    st = wk.reference_bab_settings(input_split_batch_size=2048, input_split_crown_intermediate=True,
                                   disable_sat_finding=True, total_timeout=600.0)
    return gg, spec, st


def _worker(rank, world, port, seed, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device('cuda', rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        gg, spec, st = _cfg1_problem(seed, dev)
        verdict, det = shard._input_split_batched_sharded(None, spec, st, gg, dev,
                                                          torch.float32, per_rank=16)
        out.put((rank, verdict, det['batched_n_leaves'], det['shard_leaves']))
    finally:
        dist.destroy_process_group()


def _run(world, seed):
    ctx = mp.get_context('spawn')
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _port(), seed, q), nprocs=world, join=True,
                       start_method='spawn')
    return sorted(q.get() for _ in range(world))


def test_sharded_one_rank_matches_reference_leaf_count():
    g = load_golden('bab_cfg1_seed0')
    res = _run(1, 0)
    assert res[0][1] == str(g['verdict_ci1'])
    assert res[0][2] == int(g['n_leaves_ci1'])


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason='needs two GPUs')
def test_sharded_two_gpus_same_tree():
    g = load_golden('bab_cfg1_seed0')
    res = _run(2, 0)
    for rank, verdict, n, per in res:
        assert verdict == str(g['verdict_ci1'])
        assert n == int(g['n_leaves_ci1'])
        assert min(per) > 0
