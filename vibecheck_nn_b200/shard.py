"""Input-split BaB sharded over ranks (one process per GPU).

Leaves of the input-split tree are independent: whether a leaf closes, is
clipped or is split (and along which dimension) depends only on that leaf's
box, so the tree -- and its leaf count -- does not depend on which rank bounds
which leaf.  The sharded driver therefore

1. expands the root identically on every rank (the same deterministic
   kernels on the same boxes) until the worklist holds at least
   ``world * per_rank`` leaves, counting that work once (on rank 0);
2. deals the worklist round-robin: leaf i goes to rank i % world;
3. runs the single-GPU iteration (``bab.local_iteration``) on each rank's own
   worklist in rounds of ``sync_every`` iterations; after each round one
   ``all_gather`` of a 6-word status per rank (worklist size, leaves, open
   degenerate leaves, witness flag, time-out flag, out-of-memory flag) gives
   every rank the same view, from which each decides identically whether to
   stop and how to rebalance;
4. rebalances: while the fullest worklist holds more than twice the emptiest
   plus one batch, the fullest rank sends half the difference to the
   emptiest (point-to-point send / recv of the boxes); plans are computed
   from the gathered sizes, so every rank agrees on them;
5. finishes when every worklist is empty (``verified`` unless some leaf was
   degenerate), when a rank found a witness (it is broadcast from the lowest
   such rank: ``sat``), on the global time budget or on worklist overflow
   (the sum over ranks against ``input_split_batched_max_worklist``).

Every rank takes the same collective steps in the same order, including on
the exit paths.  The engine is any object with ``process(xl, xh, n_iter)``,
``root()``, ``n_in``, ``device`` and ``cfg`` (``bab.BoundEngine`` on a GPU; the
CPU tests use a synthetic one over ``gloo``).
"""
from __future__ import annotations

import time
import types

import numpy as np
import torch
import torch.distributed as dist

from .bab import LocalState, Worklist, local_iteration

F32 = torch.float32
# status words
S_WL, S_LEAVES, S_OPEN, S_SAT, S_TIMEOUT, S_OOM = range(6)


def expand_root(engine, st, target):
    """Run the single-GPU loop until the worklist holds >= target leaves or
    the tree is exhausted (identically on every rank)."""
    while st.wl and st.wl.size() < target:
        local_iteration(engine, st)
        if st.oom or st.witness is not None:
            return


def deal(wl, rank, world, n_in, device):
    """Keep leaf i of the worklist (in pop order) when i % world == rank."""
    n = wl.size()
    if n == 0:
        return Worklist.empty(n_in, device)
    xl, xh = wl.pop(n)
    idx = torch.arange(rank, n, world, device=xl.device)
    out = Worklist.empty(n_in, device)
    if idx.numel():
        out.push(xl.index_select(0, idx).contiguous(), xh.index_select(0, idx).contiguous())
    return out


def rebalance_plan(sizes, batch):
    """Transfers [(src, dst, count)] from the gathered worklist sizes: the
    fullest rank sends half the difference to the emptiest while the fullest
    holds more than twice the emptiest plus one batch; each rank takes part in
    at most one transfer per round."""
    sizes = list(int(v) for v in sizes)
    order = sorted(range(len(sizes)), key=lambda r: (sizes[r], r))
    plan = []
    lo_i, hi_i = 0, len(order) - 1
    while lo_i < hi_i:
        lo_r, hi_r = order[lo_i], order[hi_i]
        if sizes[hi_r] <= 2 * sizes[lo_r] + batch:
            break
        cnt = (sizes[hi_r] - sizes[lo_r]) // 2
        plan.append((hi_r, lo_r, cnt))
        lo_i += 1
        hi_i -= 1
    return plan


def _transfer(wl, plan, rank, n_in, device, group):
    for src, dst, cnt in plan:
        if rank == src:
            xl, xh = wl.pop(cnt)
            dist.send(torch.cat([xl, xh], 1).contiguous(), dst, group=group)
        elif rank == dst:
            buf = torch.empty((cnt, 2 * n_in), dtype=F32, device=device)
            dist.recv(buf, src, group=group)
            wl.push(buf[:, :n_in].contiguous(), buf[:, n_in:].contiguous())


def _gather_status(status, world, device, group):
    mine = torch.as_tensor(status, dtype=torch.int64, device=device)
    allv = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allv, mine, group=group)
    return torch.stack(allv).cpu().numpy()


def _broadcast_witness(st, src, n_in, device, group, rank):
    buf = torch.zeros(n_in, dtype=torch.float64, device=device)
    if rank == src:
        buf.copy_(torch.as_tensor(np.asarray(st.witness, np.float64).reshape(-1)))
    dist.broadcast(buf, src, group=group)
    return buf.cpu().numpy()


def input_split_sharded(engine, group=None, per_rank=64, sync_every=8, t_start=None):
    """Sharded worklist BaB over the process group; returns (verdict,
    details) -- the single-GPU driver's keys, with global counts, plus
    ``shard_leaves`` (per rank), ``shard_transfers``, ``shard_rounds`` and
    this rank's host seconds in the root expansion (``shard_expand_s``), the
    status all_gather including the wait for the slowest rank
    (``shard_sync_s``) and the rebalancing send / recv (``shard_transfer_s``)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    cfg = engine.cfg
    device = engine.device
    n_in = engine.n_in
    t_start = time.perf_counter() if t_start is None else t_start
    sync = (lambda: torch.cuda.synchronize(device)) if torch.device(device).type == 'cuda' \
        else (lambda: None)
    st = LocalState(Worklist(*engine.root()), cfg.batch_size)
    t0 = time.perf_counter()
    expand_root(engine, st, world * per_rank)
    sync()
    t_expand = time.perf_counter() - t0
    t_sync = t_transfer = 0.0
    if rank != 0:  # the expansion ran on every rank; count it once
        st.n_leaves = 0
        st.n_open = 0
    if st.witness is None and not st.oom:
        st.wl = deal(st.wl, rank, world, n_in, device)
    n_transfers = 0
    rounds = 0
    while True:
        if st.witness is None and not st.oom:
            for _ in range(sync_every):
                if not st.wl or time.perf_counter() - t_start > cfg.total_budget - 0.5:
                    break
                local_iteration(engine, st)
                if st.oom or st.witness is not None:
                    break
        timed_out = time.perf_counter() - t_start > cfg.total_budget - 0.5
        status = [st.wl.size(), st.n_leaves, st.n_open, int(st.witness is not None),
                  int(timed_out), int(st.oom)]
        t0 = time.perf_counter()
        allv = _gather_status(status, world, device, group)
        t_sync += time.perf_counter() - t0
        rounds += 1
        tot = allv.sum(0)
        details = {'batched_n_leaves': int(tot[S_LEAVES]), 'batched_n_iters': st.n_iters,
                   'shard_leaves': [int(v) for v in allv[:, S_LEAVES]],
                   'shard_transfers': n_transfers, 'shard_rounds': rounds,
                   'batched_batch_size': st.batch_size, 'shard_expand_s': t_expand,
                   'shard_sync_s': t_sync, 'shard_transfer_s': t_transfer}
        if tot[S_SAT] > 0:
            src = int(np.nonzero(allv[:, S_SAT])[0][0])
            wit = _broadcast_witness(st, src, n_in, device, group, rank)
            return 'sat', dict(details, phase='batched_leaf_pgd', witness=wit)
        if tot[S_OOM] > 0:
            return 'unknown', dict(details, phase='batched_oom')
        if tot[S_WL] > cfg.max_worklist:
            return 'unknown', dict(details, phase='batched_worklist_overflow',
                                   worklist_size=int(tot[S_WL]))
        if tot[S_WL] == 0:
            if tot[S_OPEN] == 0:
                return 'verified', dict(details, phase='batched_verified')
            return 'unknown', dict(details, phase='batched_timeout', batched_worklist_left=0,
                                   batched_open_degenerate=int(tot[S_OPEN]))
        if tot[S_TIMEOUT] > 0:
            return 'unknown', dict(details, phase='batched_timeout',
                                   batched_worklist_left=int(tot[S_WL]),
                                   batched_open_degenerate=int(tot[S_OPEN] + tot[S_WL]))
        plan = rebalance_plan(allv[:, S_WL], cfg.batch_size)
        if plan:
            t0 = time.perf_counter()
            _transfer(st.wl, plan, rank, n_in, device, group)
            sync()
            t_transfer += time.perf_counter() - t0
            n_transfers += len(plan)


def _agree_on_witness(sat, wit, n_in, device, group):
    """Every rank ran the same root attack; agree on its outcome anyway (a
    wall-time budget can end it differently per rank) so that no rank enters
    the BaB collectives alone.  Returns the witness of the lowest rank that
    found one, or None."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    flags = _gather_status([int(bool(sat))], world, device, group)[:, 0]
    if not flags.any():
        return None
    src = int(np.nonzero(flags)[0][0])
    st = types.SimpleNamespace(witness=wit)
    return _broadcast_witness(st, src, n_in, device, group, rank)


def _input_split_batched_sharded(graph, spec, settings, gg, device, dtype, group=None,
                                 per_rank=64, sync_every=8):
    """``_input_split_batched`` (verify_graph.py:12466) over the ranks of
    ``group`` (default: the world), one GPU per rank: the same verdict and,
    with alpha-CROWN and leaf PGD off, the same leaf count as one GPU."""
    from .bab import make_engine
    from .ops import _dev
    device = _dev(device)
    t_start = time.perf_counter()
    engine = make_engine(spec, gg, settings, device)
    cfg = engine.cfg
    if cfg.sat_finding and cfg.pgd_phase0:
        from .pgd import root_pgd
        sat, wit, phase = root_pgd(spec, gg, engine.n_output, device, settings)
        wit = _agree_on_witness(sat, wit, engine.n_in, device, group)
        if wit is not None:
            return 'sat', {'phase': phase or 'batched_pgd', 'witness': wit}
    if not engine.queries:
        return 'verified', {'phase': 'batched_no_queries'}
    return input_split_sharded(engine, group, per_rank=per_rank, sync_every=sync_every,
                               t_start=t_start)
