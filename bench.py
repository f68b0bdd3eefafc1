#!/usr/bin/env python
"""Benchmark: CROWN subdomain-bound throughput (cfg2) on B200.

Workload (the headline metric's single-GPU config):
a seeded 5->[50]x6->5 fp32 ReLU MLP (ACAS-Xu shape), 65,536 sub-boxes per
step (centre U(-0.5,0.5), half-width U(0.001,0.1)), 4 spec rows with
coefficients in {-1,0,1}; one step = IBP intermediate bounds + CROWN
back-substitution for every box (one fused kernel launch, vcb_mlp_crown).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg2|cfg1|cfg3|cfg4]

``--config`` selects another BASELINE config on its own metric: cfg1 the
input-split BaB time-to-verdict (N > 1: the sharded driver, strong scaling),
cfg3 alpha-CROWN over 1,024 ReLU-split domains, cfg4 conv CROWN over 256
domains, cfg5 one BaB iteration (tcgen05 zonotope + CROWN + split) over
leaves of the depth-18 input-split tree of the 3072->[1024]x8->10 MLP.

N > 1 runs under torchrun, one rank per GPU; every rank bounds its own
65,536 boxes (weak scaling, no data-path collective); the time is the max
over ranks.  ``--impl reference`` times the reference's own CPU path
(its torch code, installed under baseline/_ref by ``pip install --target``)
in one single-threaded process per host core on a bounded sample of the same
workload, or the numpy restatement in oracle/ when the reference is not
installed.  The default cfg2 line also carries a ``cfg1`` record: the
input-split BaB time-to-verdict on this GPU and the reference's own CPU
driver on the same problem at 1 thread and at a thread per core.  Prints one
JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'subdomain bounds/sec (CROWN, batched input-split)'
UNIT = 'subdomains/s'
N_BOXES = 65536
N_Q = 4
FLUSH_BYTES = 256 << 20  # > 126 MB L2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=200)
    ap.add_argument('--warmup', type=int, default=10)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--config', default='cfg2', choices=['cfg2', 'cfg1', 'cfg3', 'cfg4', 'cfg5'],
                    help='cfg2 (default) is the headline; the others time the '
                         'remaining BASELINE configs on their own metrics')
    ap.add_argument('--cfg5-leaves', type=int, default=64,
                    help='cfg5: leaves per GPU per step (the default is the workload; fewer '
                         'make a small case for counter captures)')
    ap.add_argument('--full', action='store_true',
                    help='cfg5: the whole input-split BaB through the sharded driver '
                         '(worklist bound 262,144 leaves) instead of single iterations')
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU legs: the reference's own torch CPU path when it is installed under
# baseline/_ref (pip install --target of the reference), else the oracle
# (numpy restatement of the reference algorithm)
# ---------------------------------------------------------------------------

REF_DIR = os.path.join(ROOT, 'baseline', '_ref')
_WORKER = {}


def reference_installed():
    return os.path.isfile(os.path.join(REF_DIR, 'vibecheck', 'verify_graph.py'))


def _pool_init(threads):
    """Spawned worker: its torch / BLAS thread count, fixed before torch is
    imported."""
    for k in ('OMP_NUM_THREADS', 'MKL_NUM_THREADS', 'OPENBLAS_NUM_THREADS'):
        os.environ[k] = str(threads)
    import torch
    torch.set_num_threads(threads)


def _reference_modules():
    """The installed reference's modules (gurobipy is only imported by its
    LP/MILP code, which these paths do not reach: an empty stand-in)."""
    import types
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    sys.modules.setdefault('gurobipy', types.ModuleType('gurobipy'))
    from vibecheck import settings as vs, spec as vspec, verify_graph as vg, verify_zono_bnb as vz
    return vz, vg, vs, vspec


def _cpu_worker(args):
    """Seconds to bound cfg2 boxes [lo, hi): 'reference' = the reference's
    _ibp_forward_graph_batched + _spec_backward_graph_batched on the CPU
    (verify_zono_bnb.py:1066, :4270), 'port' = oracle/bounds.py."""
    kind, lo, hi = args
    if 'w' not in _WORKER:
        from vibecheck_nn_b200 import workloads as wk
        _WORKER['w'] = wk.cfg2(seed=0, n_boxes=N_BOXES, n_q=N_Q)
    w = _WORKER['w']
    if kind == 'port':
        from oracle import bounds as ob
        if 'gg' not in _WORKER:
            from vibecheck_nn_b200 import workloads as wk
            _WORKER['gg'] = wk.mlp_gg(w['layers'])
        gg = _WORKER['gg']
        t0 = time.perf_counter()
        sb = ob.ibp_forward_batched(w['xl'][lo:hi], w['xh'][lo:hi], gg)
        ob.spec_backward_batched(sb, w['xl'][lo:hi], w['xh'][lo:hi], gg,
                                 w['spec_W'], w['spec_b'])
        return time.perf_counter() - t0
    import torch
    if 'ref' not in _WORKER:
        from vibecheck_nn_b200 import workloads as wk
        vz = _reference_modules()[0]
        _WORKER['ref'] = (vz, wk.mlp_gg(w['layers'], 'cpu', torch.float32),
                          wk.spec_ew_from(w['spec_W'], w['spec_b'], 'cpu'),
                          torch.as_tensor(w['xl']), torch.as_tensor(w['xh']))
    vz, gg, spec_ew, xl, xh = _WORKER['ref']
    t0 = time.perf_counter()
    sb = vz._ibp_forward_graph_batched(xl[lo:hi], xh[lo:hi], gg, 'cpu', torch.float32)
    vz._spec_backward_graph_batched(sb, xl[lo:hi], xh[lo:hi], gg, spec_ew, 'cpu',
                                    torch.float32)
    return time.perf_counter() - t0


def cpu_rate(pool, procs, sample, kind):
    """Boxes/s of `kind` on `sample` boxes split over `procs` processes."""
    per = (sample + procs - 1) // procs
    chunks = [(kind, i * per, min(sample, (i + 1) * per)) for i in range(procs)]
    t0 = time.perf_counter()
    pool.map(_cpu_worker, chunks)
    return sample / (time.perf_counter() - t0)


def make_pool(procs, threads=1, kinds=('port',)):
    import multiprocessing as mp
    pool = mp.get_context('spawn').Pool(procs, initializer=_pool_init, initargs=(threads,))
    for kind in kinds:
        pool.map(_cpu_worker, [(kind, 0, 64)] * procs)  # import + warm each worker
    return pool


class CpuPools:
    """Spawned CPU workers, started before the first GPU call: all cores as
    single-threaded processes, one single-threaded process, and (reference
    only) one process with a torch thread per core."""

    def __init__(self):
        self.cores = os.cpu_count() or 1
        self.ref = reference_installed()
        kinds = ('reference', 'port') if self.ref else ('port',)
        self.procs = make_pool(self.cores, 1, kinds)
        self.one = make_pool(1, 1, kinds[:1])
        self.threaded = make_pool(1, self.cores, ('reference',)) if self.ref else None

    def close(self):
        for p in (self.procs, self.one, self.threaded):
            if p is not None:
                p.close()


def _median_rate(pool, procs, sample, kind, budget_s):
    rates = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or len(rates) < 2:
        rates.append(cpu_rate(pool, procs, sample, kind))
    return statistics.median(rates), len(rates)


def cpu_baseline(pools, budget_s=6.0):
    """The reference's CPU throughput on cfg2 boxes: its torch path in one
    process per core (the value), in one single-threaded process and with a
    torch thread per core in one process, next to the numpy port."""
    c = pools.cores
    port, n_port = _median_rate(pools.procs, c, 4096 * c, 'port', budget_s)
    if not pools.ref:
        return {'value': port, 'unit': UNIT, 'cores': c, 'kind': 'port',
                'sample': f'{4096 * c} cfg2 boxes per repetition, {n_port} repetitions '
                          f'(median), numpy oracle (oracle/bounds.py) in {c} spawn processes; '
                          f'the reference is not installed under baseline/_ref'}
    procs, n1 = _median_rate(pools.procs, c, 4096 * c, 'reference', budget_s)
    one, n2 = _median_rate(pools.one, 1, 4096, 'reference', budget_s)
    thr, n3 = _median_rate(pools.threaded, 1, 4096 * c, 'reference', budget_s)
    return {'value': procs, 'unit': UNIT, 'cores': c, 'kind': 'reference',
            'sample': f'{4096 * c} cfg2 boxes per repetition, {n1} repetitions (median): the '
                      f'reference\'s _ibp_forward_graph_batched + _spec_backward_graph_batched '
                      f'on the CPU (torch, fp32) in {c} spawn processes of 1 thread',
            'one_thread': {'value': one, 'sample': f'4096 boxes, {n2} repetitions'},
            'threads_in_one_process': {'value': thr, 'threads': c,
                                       'sample': f'{4096 * c} boxes, {n3} repetitions'},
            'port': {'value': port, 'cores': c, 'kind': 'port',
                     'sample': f'numpy oracle, {4096 * c} boxes, {n_port} repetitions'}}


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    kind = 'reference' if reference_installed() else 'port'
    pool = make_pool(cores, 1, (kind,))
    sample = 4096 * cores
    for _ in range(args.warmup):
        cpu_rate(pool, cores, sample, kind)
    rates = [cpu_rate(pool, cores, sample, kind) for _ in range(args.steps)]
    pool.close()
    v = statistics.median(rates)
    what = ("the reference's own CPU path (_ibp_forward_graph_batched + "
            "_spec_backward_graph_batched, torch fp32, installed under baseline/_ref)"
            if kind == 'reference' else 'the numpy oracle (oracle/bounds.py)')
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': v, 'unit': UNIT,
        'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': 1000.0 * N_BOXES / v, 'higher_is_better': True,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded)',
        'config': config_dict(args.gpus),
        'cpu_baseline': {'value': v, 'unit': UNIT, 'cores': cores, 'kind': kind,
                         'sample': f'each step: {sample} cfg2 boxes, {what}, in {cores} '
                                   f'spawn processes of 1 thread'},
        'e2e': {'value': v, 'unit': UNIT, 'h2d_bytes_per_step': 0,
                'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(n):
    return {'workload': 'cfg2: CROWN microbench, 5x[50]x6x5 fp32 ReLU MLP, '
                        'IBP intermediates + CROWN back-substitution',
            'boxes_per_gpu': N_BOXES, 'spec_rows': N_Q,
            'global_batch': N_BOXES * n,
            'l2': 'flushed (256 MiB write) between timed steps',
            'parallelism': f'{n} GPU(s), boxes sharded, no data-path collective'}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """SM clock and clock-event reasons sampled while the timed region runs.

    In-process NVML (read-only queries) polled every ~1 ms from a thread, so
    even a timed region of a few milliseconds gets samples; `nvidia-smi -lms`
    (which needs hundreds of milliseconds to start) is the fallback when NVML
    is not importable.  The sampler starts before the region and has taken its
    first sample before __enter__ returns."""
    FIELDS = ('clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,'
              'clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,'
              'clocks_event_reasons.sw_power_cap')
    REASONS = (('hw_slowdown', 0x8), ('hw_thermal_slowdown', 0x40),
               ('sw_thermal_slowdown', 0x20), ('sw_power_cap', 0x4))

    def __init__(self, gpu_id, period_s=0.001):
        self.gpu_id = gpu_id
        self.period = period_s
        self.proc = None
        self.lines = []
        self.samples = []  # (sm MHz, max sm MHz, reason bits)
        self._stop = threading.Event()
        self._first = threading.Event()
        self.t = None
        self.nv = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        gid = str(self.gpu_id)
        if gid.startswith('GPU-'):
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(gid)
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(int(gid))

    def _poll(self, nv, h):
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while True:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), float(mx), int(rs)))
            except Exception:  # noqa: BLE001 -- a failed read only loses a sample
                pass
            self._first.set()
            if self._stop.wait(self.period):
                break

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            self.nv = nv
            self.t = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.t.start()
            self._first.wait(5.0)
            return self
        except Exception:  # noqa: BLE001 -- no NVML: fall back to nvidia-smi
            self.t = None
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', '-i', str(self.gpu_id),
                 f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                 '-lms', '20'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        elif self.t is not None:
            self.t.join(timeout=5)
            try:
                self.nv.nvmlShutdown()
            except Exception:  # noqa: BLE001 -- releasing NVML is best effort
                pass

    def summary(self):
        sm, mx, reasons = [], [], set()
        for s_, m_, bits in self.samples:
            sm.append(s_)
            mx.append(m_)
            for nm, bit in self.REASONS:
                if bits & bit:
                    reasons.add(nm)
        names = [nm for nm, _ in self.REASONS]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(',')]
            if len(parts) != 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[2:]):
                if v.lower() == 'active':
                    reasons.add(nm)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [],
                    'samples': 0}
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': max(mx),
                'reasons': sorted(reasons), 'samples': len(sm),
                'source': 'nvml' if self.samples else 'nvidia-smi'}


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

def read_traffic(kernel):
    """Per-launch DRAM bytes of a cfg2 kernel from bench_traffic.json (one
    ncu capture per kernel, the command recorded beside the figure)."""
    try:
        with open(os.path.join(ROOT, 'bench_traffic.json')) as f:
            return float(json.load(f)[kernel]['bytes_per_launch'])
    except (OSError, KeyError, ValueError):
        return None


def measured_fp32_peak(dev):
    """TFLOP/s of the FFMA probe kernel (vcb_probe_ffma) on this GPU now."""
    import torch
    from vibecheck_nn_b200 import _lib
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * 8
    iters = 4096
    out = torch.empty(blocks * 256, device=dev)
    st = _lib.stream_of(dev)
    best = 0.0
    for _ in range(5):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        _lib.check(_lib.lib().vcb_probe_ffma(_lib.ptr(out), blocks, iters, st))
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        best = max(best, blocks * 256.0 * iters * 128 / (ms * 1e-3) / 1e12)
    return best


def _lib_path(desc, B, Q):
    """1 when vcb_mlp_crown runs the tensor-core kernel for (B, Q)."""
    from vibecheck_nn_b200 import _lib
    return _lib.lib().vcb_mlp_crown_path(desc.struct, B, Q)


def roofline_cfg2(tc_path, achieved, ffma_peak, flop_per_box):
    """Roofline of the cfg2 step's kernel.  The tensor-core kernel is judged
    against the 3xTF32 rate the tensor cores can deliver (measured bf16 dense
    peak / 2 for TF32 / 3 products); the SIMT kernel against the FFMA peak
    measured live."""
    if not tc_path:
        return {'bound': 'fp32_simt', 'achieved': achieved, 'peak': ffma_peak,
                'unit': 'TFLOP/s', 'frac': achieved / ffma_peak if ffma_peak else None,
                'traffic': read_traffic('crown_mlp_kernel'),
                'kernel': 'vcb_mlp_crown (crown_mlp_kernel)', 'flop_per_box': flop_per_box,
                'peak_source': 'measured live: vcb_probe_ffma FFMA loop (MEASURED_PEAKS.json '
                               'has no FP32 SIMT figure)'}
    peak, source = tf32x3_peak()
    return {'bound': 'tensor', 'achieved': achieved, 'peak': peak, 'unit': 'TFLOP/s',
            'frac': achieved / peak, 'traffic': read_traffic('crown_tc_kernel'),
            'kernel': 'vcb_mlp_crown (crown_tc_kernel, tcgen05 3xTF32), timed as the whole '
                      'call: crown_tc_kernel 89 %, crown_tie_kernel 9 %, crown_tc_images 2 %',
            'flop_per_box': flop_per_box,
            'frac_of_ffma_peak': achieved / ffma_peak if ffma_peak else None,
            'peak_source': source}


def tf32x3_peak():
    """fp32-equivalent rate of 3xTF32 on the tensor cores: the measured bf16
    dense peak / 2 (TF32 rate) / 3 (products per fp32 product)."""
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, 'MEASURED_PEAKS.json')))
    except (OSError, ValueError):
        pass
    bf16 = peaks.get('bf16_tflops')
    if bf16:
        return bf16 / 6.0, ('of measured: MEASURED_PEAKS.json bf16_tflops / 2 (TF32 rate) / 3 '
                            '(3xTF32 products)')
    return 1590.0 / 6.0, 'of fallback: 1590 TFLOP/s bf16 / 2 / 3'


def run_ours(args):
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    pools = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        pools = CpuPools()  # spawned before the first GPU call
    dev = torch.device(f'cuda:{local}')
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=120),
                                device_id=dev)
    from vibecheck_nn_b200 import ops, workloads as wk
    w = wk.cfg2(seed=0, n_boxes=N_BOXES, n_q=N_Q)
    gg = wk.mlp_gg(w['layers'], dev)
    spec = ops.spec_matrix(wk.spec_ew_from(w['spec_W'], w['spec_b'], dev), dev)
    xl = torch.as_tensor(w['xl'], device=dev)
    xh = torch.as_tensor(w['xh'], device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return ops.ibp_crown_batched(xl, xh, gg, spec, dev)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    peak = measured_fp32_peak(dev)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    props = torch.cuda.get_device_properties(dev)
    gpu_id = getattr(props, 'uuid', None)
    gpu_id = f'GPU-{gpu_id}' if gpu_id is not None else local
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(gpu_id) as clk:
        t_wall0 = time.perf_counter()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        t_wall = time.perf_counter() - t_wall0
    if world > 1:
        dist.barrier()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    t_ms = sum(per_step)
    t_max = torch.tensor([t_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    t_max = float(t_max.item())
    value = world * N_BOXES * args.steps / (t_max * 1e-3)

    # ---- e2e through the public API with host buffers (pinned): every step
    # copies its boxes in, bounds them and reads the bounds back; steps
    # alternate between two streams so one step's copies overlap the other's
    # kernel (each stream has its own device and host buffers)
    xl_h = torch.as_tensor(w['xl']).pin_memory()
    xh_h = torch.as_tensor(w['xh']).pin_memory()
    lanes = [torch.cuda.Stream(dev) for _ in range(2)]
    bufs = [(torch.empty_like(xl), torch.empty_like(xh),
             torch.empty((N_BOXES, N_Q), dtype=torch.float32).pin_memory()) for _ in lanes]

    def e2e_step(i):
        lane = lanes[i % 2]
        xl_d, xh_d, lb_h = bufs[i % 2]
        with torch.cuda.stream(lane):
            xl_d.copy_(xl_h, non_blocking=True)
            xh_d.copy_(xh_h, non_blocking=True)
            lb_h.copy_(ops.ibp_crown_batched(xl_d, xh_d, gg, spec, dev), non_blocking=True)

    for lane in lanes:
        lane.wait_stream(stream)
    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for lane in lanes:
        lane.wait_stream(stream)
    for i in range(args.steps):
        e2e_step(i)
    for lane in lanes:
        stream.wait_stream(lane)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        dist.barrier()
    e2e_value = world * N_BOXES * args.steps / (float(e2e_ms.item()) * 1e-3)

    sum_w = sum(a * b for a, b in zip((5,) + (50,) * 6, (50,) * 6 + (5,)))
    flop_per_box = (4 + 2 * N_Q) * sum_w
    mean_ms = t_ms / args.steps
    achieved = N_BOXES * flop_per_box / (mean_ms * 1e-3) / 1e12
    desc = ops.mlp_desc(gg, dev)
    tc_path = bool(_lib_path(desc, N_BOXES, N_Q))
    cfg1 = cfg1_record(dev, gpu_id) if world == 1 else None
    cpu = None
    if pools is not None:
        cpu = cpu_baseline(pools)
        if pools.ref:
            cfg1.update(cfg1_reference_cpu(pools))
        pools.close()
    if rank == 0:
        line = {
            'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': t_max / args.steps, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded numpy rng; no public dataset for this path)',
            'config': config_dict(world),
            'e2e': {'value': e2e_value, 'unit': UNIT,
                    'h2d_bytes_per_step': int(xl_h.numel() * 4 * 2),
                    'd2h_bytes_per_step': int(N_BOXES * N_Q * 4),
                    'pipelining': 'steps alternate between 2 CUDA streams'},
            # per step: crown_tc_images, crown_tc_kernel, crown_tie_kernel (tensor-core
            # route) or crown_mlp_kernel (SIMT route)
            'gpu_launches': (3 if tc_path else 1) * args.steps,
            'roofline': roofline_cfg2(tc_path, achieved, peak, flop_per_box),
            'clocks': clk.summary(),
            'wall_s_timed_region': t_wall,
        }
        if cpu is not None:
            line['cpu_baseline'] = cpu
        if cfg1 is not None:
            line['cfg1'] = cfg1
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _cfg1_problem(dev):
    from vibecheck_nn_b200 import bab, workloads as wk
    w = wk.cfg1(0)
    spec = bab.LinearSpec(w['xl'], w['xh'], [[('pair', 1, 0)]])
    st = wk.reference_bab_settings(input_split_batch_size=2048,
                                   input_split_crown_intermediate=True, total_timeout=600.0)
    return w, spec, st, wk.mlp_gg(w['layers'], dev)


def _cfg1_reference_worker(budget_s):
    """Verdicts of the reference's own input-split driver on cfg1 on the CPU
    (_input_split_batched, verify_graph.py:9947, default_settings with the
    bench's overrides, root PGD included) for about budget_s seconds:
    (verdict, leaves, seconds per verdict, verdicts)."""
    import contextlib
    import types
    import torch
    from vibecheck_nn_b200 import workloads as wk
    _, vg, vs, vspec = _reference_modules()
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], 'cpu', torch.float32)
    spec = vspec.VNNSpec(x_lo=w['xl'].astype('float64'), x_hi=w['xh'].astype('float64'),
                         disjuncts=[vspec.Conjunct([vspec.PairwiseConstraint(pred=1, comp=0)])])
    st = vs.default_settings(device='cpu', bits=32, input_split_batched_enabled=True,
                             input_split_batch_size=2048, input_split_crown_intermediate=True,
                             total_timeout=600.0)
    times = []
    t0 = time.perf_counter()
    with open(os.devnull, 'w') as null, contextlib.redirect_stdout(null):  # progress lines
        while not times or (time.perf_counter() - t0 < budget_s and len(times) < 5):
            t = time.perf_counter()
            verdict, det = vg._input_split_batched(types.SimpleNamespace(onnx_path=None), spec,
                                                   st, gg, torch.device('cpu'), torch.float32)
            times.append(time.perf_counter() - t)
    return verdict, int(det.get('batched_n_leaves', -1)), statistics.median(times), len(times)


def cfg1_record(dev, gpu_id, n_verdicts=10):
    """cfg1 time-to-verdict on this GPU: 3 warm-up verdicts, then n_verdicts
    timed with CUDA events, L2 flushed before each."""
    import torch
    from vibecheck_nn_b200 import bab
    w, spec, st, gg = _cfg1_problem(dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        bab._input_split_batched(None, spec, st, gg, dev, torch.float32)
    torch.cuda.synchronize(dev)
    ms = []
    # the driver's host loop shares the interpreter with the sampler thread:
    # poll every 20 ms, not every 1 ms, so that sampling does not slow it
    with ClockSampler(gpu_id, period_s=0.02) as clk:
        for _ in range(n_verdicts):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            verdict, det = bab._input_split_batched(None, spec, st, gg, dev, torch.float32)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms.append(e0.elapsed_time(e1))
    rec = {'workload': 'cfg1: 5x[50]x6x5 MLP, y0 - y1 <= d, input-split BaB, leaf batch 2048, '
                       'CROWN intermediates, root PGD included',
           'verdict': verdict, 'leaves': det['batched_n_leaves'],
           'iterations': det['batched_n_iters'], 'ms': statistics.median(ms),
           'ms_all': ms, 'clocks': clk.summary()}
    return rec


def cfg1_reference_cpu(pools, limit_s=60.0):
    """The reference's own CPU driver on cfg1 at 1 thread and with a torch
    thread per core (each bounded by limit_s; a leg that runs out reports
    its limit instead of a time)."""
    import multiprocessing as mp
    out = {}
    for key, pool, threads in (('reference_cpu_1_thread', pools.one, 1),
                               ('reference_cpu_all_threads', pools.threaded, pools.cores)):
        job = pool.apply_async(_cfg1_reference_worker, (8.0,))
        try:
            v, leaves, s_, n = job.get(timeout=limit_s)
            out[key] = {'verdict': v, 'leaves': leaves, 'ms': 1e3 * s_, 'verdicts': n,
                        'threads': threads}
        except mp.TimeoutError:
            pool.terminate()
            out[key] = {'ms': None, 'threads': threads,
                        'note': f'no verdict within {limit_s:.0f} s'}
    return out


# ---------------------------------------------------------------------------
# other BASELINE configs (cfg1, cfg3, cfg4)
# ---------------------------------------------------------------------------

def _setup_dist():
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    dev = torch.device(f'cuda:{local}')
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=300), device_id=dev)
    return rank, world, local, dev


def _time_steps(dev, step, args, world, flush, min_warmup=3, clock_period=0.001):
    """W warm-up steps, then K timed steps (CUDA events, L2 flushed before
    each); returns (per-step ms, clocks summary, max-over-ranks total ms).
    clock_period: seconds between clock samples (host-driven steps take a
    longer one, so that the sampler thread does not slow their host loop)."""
    import torch
    import torch.distributed as dist
    for _ in range(max(min_warmup, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    props = torch.cuda.get_device_properties(dev)
    gid = getattr(props, 'uuid', None)
    gid = f'GPU-{gid}' if gid is not None else dev.index
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(gid, period_s=clock_period) as clk:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    per = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    tot = torch.tensor([sum(per)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    return per, clk.summary(), float(tot.item())


def _cpu_cfg1(budget_s=15.0):
    from oracle import bab as obab
    from vibecheck_nn_b200 import workloads as wk
    w = wk.cfg1(0)
    t0 = time.perf_counter()
    _, det = obab.input_split_bab(wk.mlp_gg(w['layers']), w['xl'], w['xh'], w['spec_W'],
                                  w['spec_b'], batch_size=2048, crown_intermediate=True,
                                  timeout=budget_s)
    return det['batched_n_leaves'] / (time.perf_counter() - t0)


def run_cfg1(args):
    import torch
    import torch.distributed as dist
    import types
    rank, world, _, dev = _setup_dist()
    from vibecheck_nn_b200 import bab, shard, workloads as wk
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], dev)
    spec = bab.LinearSpec(w['xl'], w['xh'], [[('pair', 1, 0)]])
    st = wk.reference_bab_settings(input_split_batch_size=2048, input_split_crown_intermediate=True,
                                   total_timeout=600.0)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    res = {}

    def step():
        if world > 1:
            res['v'] = shard._input_split_batched_sharded(None, spec, st, gg, dev, torch.float32)
        else:
            res['v'] = bab._input_split_batched(None, spec, st, gg, dev, torch.float32)

    per, clocks, t_max = _time_steps(dev, step, args, world, flush, clock_period=0.02)
    verdict, det = res['v']
    n_leaves = det['batched_n_leaves']
    ms = t_max / args.steps
    if rank == 0:
        line = {
            'metric': 'BaB time-to-verdict (cfg1, input-split, CROWN intermediates)',
            'value': ms / 1e3, 'unit': 's', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': False,
            'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded numpy rng)',
            'config': {'workload': 'cfg1: 5x[50]x6x5 MLP, y0 - y1 <= d, input-split BaB, '
                                   'leaf batch 2048, root PGD included',
                       'verdict': verdict, 'leaves': n_leaves,
                       'leaves_per_s': n_leaves / (ms / 1e3),
                       'l2': 'flushed (256 MiB write) before each verdict',
                       'parallelism': f'{world} GPU(s), leaves sharded' if world > 1
                       else '1 GPU'},
            'clocks': clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            rate = _cpu_cfg1()
            port = {'value': n_leaves / rate, 'unit': 's', 'cores': 1, 'kind': 'port',
                    'sample': f'oracle/bab.py input-split BaB for 15 s ({rate:.0f} leaves/s, '
                              f'numpy), extrapolated to the {n_leaves} leaves of the verdict'}
            line['cpu_baseline'] = port
            if reference_installed():
                cores = os.cpu_count() or 1
                pools = types.SimpleNamespace(one=make_pool(1, 1, ()), cores=cores,
                                              threaded=make_pool(1, cores, ()))
                ref = cfg1_reference_cpu(pools)
                pools.one.close()
                pools.threaded.close()
                legs = [v for v in ref.values() if v.get('ms') is not None]
                if legs:
                    best = min(legs, key=lambda v: v['ms'])
                    line['cpu_baseline'] = {
                        'value': best['ms'] / 1e3, 'unit': 's', 'cores': best['threads'],
                        'kind': 'reference',
                        'sample': "the reference's own _input_split_batched on the CPU "
                                  f"(torch fp32, installed under baseline/_ref), median of "
                                  f"{best['verdicts']} verdict(s) ({best['verdict']}, "
                                  f"{best['leaves']} leaves) at {best['threads']} thread(s)",
                        'legs': ref, 'port': port}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _domains(xl1, xh1, root_lo, root_hi, n_split):
    import numpy as np
    from vibecheck_nn_b200 import workloads as wk
    picked, clamps = wk.split_domains(root_lo, root_hi, n_split)
    Dn = 1 << len(picked)
    xl = np.broadcast_to(xl1, (Dn, xl1.size)).copy()
    xh = np.broadcast_to(xh1, (Dn, xh1.size)).copy()
    return xl, xh, clamps


def run_cfg34(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    rank, world, _, dev = _setup_dist()
    from vibecheck_nn_b200 import graph, ops, wide, workloads as wk
    from oracle import bounds as ob
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    T = lambda a: torch.as_tensor(a, device=dev)  # noqa: E731
    if args.config == 'cfg3':
        w = wk.cfg3(0)
        gg = wk.mlp_gg(w['layers'], dev)
        wn = wide.wide_net(gg, dev)
        root = wide.wide_ibp(wn, T(w['xl'][None]), T(w['xh'][None]))
        xl, xh, clamps = _domains(w['xl'], w['xh'], {L: v[0][0].cpu().numpy() for L, v in root.items()},
                                  {L: v[1][0].cpu().numpy() for L, v in root.items()}, 10)
        Dn = xl.shape[0]
        dims = wk.CFG3_DIMS
        sw = sum(a * b for a, b in zip(dims[:-1], dims[1:]))
        Q = w['spec_W'].shape[0]
        flop = 20 * Dn * 4 * Q * sw + 4 * sw * Dn
        tcl = {L: (T(c[0]), T(c[1])) for L, c in clamps.items()}
        xld, xhd = T(xl).float(), T(xh).float()  # resident in HBM before the timed region
        sWd, sbd = T(w['spec_W']).float(), T(w['spec_b']).float()

        def step():
            return wide.alpha_crown_domains(xld, xhd, gg, sWd, sbd, tcl, dev,
                                            n_iters=20, lr=0.1)

        def cpu():
            ggc = wk.mlp_gg(w['layers'])
            n = 16
            cc = {L: (c[0][:n], c[1][:n]) for L, c in clamps.items()}
            t0 = time.perf_counter()
            ob.alpha_beta_crown_domains(xl[:n], xh[:n], ggc, w['spec_W'], w['spec_b'], cc,
                                        n_iters=20, lr=0.1)
            return n / (time.perf_counter() - t0), f'{n} domains x 20 iterations, numpy oracle'
        metric = 'alpha-CROWN domains/s (cfg3: 20 Adam iterations, 9 spec rows)'
        workload = ('cfg3: 784x[256]x6x10 MLP, 1024 ReLU-split domains (10 widest unstable '
                    'neurons), IBP intermediates, min-area alpha init, Adam lr 0.1 x 20')
    else:
        w = wk.cfg4(0)
        gg = wk.cnn_gg(w['params'], dev)
        G = graph.graph_net(gg, dev)
        root = graph.graph_ibp(G, T(w['xl'][None]), T(w['xh'][None]))
        xl, xh, clamps = _domains(w['xl'], w['xh'], {L: v[0][0].cpu().numpy() for L, v in root.items()},
                                  {L: v[1][0].cpu().numpy() for L, v in root.items()}, 8)
        Dn = xl.shape[0]
        SW, Sb = wk.margin_rows(10, 3)
        flop = Dn * (4 * 926_696 + 2 * 9 * 926_696)
        tcl = {L: (T(c[0]), T(c[1])) for L, c in clamps.items()}
        xlt, xht = T(xl), T(xh)
        spec_ew = wk.spec_ew_from(SW, Sb, dev)

        def step():
            sb = ops._ibp_forward_graph_batched(xlt, xht, gg, dev, torch.float32,
                                                relu_clamps=tcl)
            return ops._spec_backward_graph_batched(sb, xlt, xht, gg, spec_ew, dev,
                                                    torch.float32)

        def cpu():
            ggc = wk.cnn_gg(w['params'])
            n = 16
            cc = {L: (c[0][:n], c[1][:n]) for L, c in clamps.items()}
            t0 = time.perf_counter()
            sbr = ob.ibp_forward_batched(xl[:n], xh[:n], ggc, relu_clamps=cc)
            ob.spec_backward_batched(sbr, xl[:n], xh[:n], ggc, SW, Sb)
            return n / (time.perf_counter() - t0), f'{n} domains, numpy oracle'
        metric = 'conv CROWN domains/s (cfg4: IBP intermediates + CROWN through conv-transpose)'
        workload = ('cfg4: CNN 3x32x32 -> conv16 4x4 s2 -> conv32 4x4 s2 -> fc100 -> fc10, '
                    '256 ReLU-split domains, 9 margin rows')
    per, clocks, t_max = _time_steps(dev, step, args, world, flush)
    ms = t_max / args.steps
    peak = measured_fp32_peak(dev)
    achieved = flop / (statistics.mean(per) * 1e-3) / 1e12
    if rank == 0:
        line = {
            'metric': metric, 'value': world * Dn / (ms / 1e3), 'unit': 'domains/s',
            'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms,
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded numpy rng)',
            'config': {'workload': workload, 'domains_per_gpu': Dn,
                       'l2': 'flushed (256 MiB write) between timed steps',
                       'parallelism': f'{world} GPU(s), domains sharded'},
            'roofline': {'bound': 'fp32_simt', 'achieved': achieved, 'peak': peak,
                         'unit': 'TFLOP/s', 'frac': achieved / peak if peak else None,
                         'traffic': None, 'flop_per_step': flop,
                         'peak_source': 'measured live: vcb_probe_ffma'},
            'clocks': clocks,
        }
        if args.config == 'cfg3' and wide.last_stats.get('path') == 'tc':
            tpk, src = tf32x3_peak()
            line['roofline'] = {
                'bound': 'tensor', 'achieved': achieved, 'peak': tpk, 'unit': 'TFLOP/s',
                'frac': achieved / tpk, 'traffic': None, 'flop_per_step': flop,
                'kernel': 'alpha loop on tcgen05 3xTF32 GEMMs with fused epilogues '
                          '(vcb_wtc_*), one CUDA graph per call; the step also runs the '
                          'SIMT wide IBP',
                'frac_of_ffma_peak': achieved / peak if peak else None, 'peak_source': src}
        if world == 1 and not args.no_cpu_baseline:
            rate, sample = cpu()
            line['cpu_baseline'] = {'value': rate, 'unit': 'domains/s',
                                    'cores': os.cpu_count(), 'kind': 'port',
                                    'sample': sample + ' (numpy BLAS threads)'}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_cfg5(args, per_step=64):
    import numpy as np
    import torch
    import torch.distributed as dist
    import types
    rank, world, _, dev = _setup_dist()
    from vibecheck_nn_b200 import bab, workloads as wk
    from oracle import bounds as ob
    w = wk.cfg5(0)
    gg = wk.mlp_gg(w['layers'], dev)
    t = w['true_label']
    spec = bab.LinearSpec(w['xl'], w['xh'], wk.robustness_disjuncts(10, t))
    st = wk.reference_bab_settings(input_split_batch_size=per_step, disable_sat_finding=True)
    eng = bab.make_engine(spec, gg, st, dev)
    assert isinstance(eng, bab.WideBoundEngine)
    n_batches = max(3, args.warmup) + args.steps
    base = rank * n_batches * per_step
    batches = []
    for i in range(n_batches):
        lo, hi = wk.cfg5_leaves(w['xl'], w['xh'], base + i * per_step, per_step)
        batches.append((torch.as_tensor(lo, device=dev), torch.as_tensor(hi, device=dev)))
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    it = {'i': 0}

    def step():
        xl_b, xh_b = batches[it['i'] % n_batches]
        it['i'] += 1
        return eng.process(xl_b, xh_b, 0)

    for _ in range(max(3, args.warmup)):
        step()
    eng.stats = {}
    per, clocks, t_max = _time_steps(dev, step, types.SimpleNamespace(warmup=0, steps=args.steps),
                                     world, flush, min_warmup=0)
    torch.cuda.synchronize(dev)
    stats = eng.stats
    gemm_ms = sum(a.elapsed_time(b) for a, b in stats['gemm_events'])
    achieved = stats['gemm_flop'] / (gemm_ms * 1e-3) / 1e12
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, 'MEASURED_PEAKS.json')))
    except (OSError, ValueError):
        pass
    bf16 = peaks.get('bf16_tflops')
    peak = bf16 / 6.0 if bf16 else 1590.0 / 6.0
    ms = t_max / args.steps
    if rank == 0:
        line = {
            'metric': 'cfg5 leaves/s (zonotope + CROWN spec bound + split, one BaB iteration)',
            'value': world * per_step / (ms / 1e3), 'unit': 'leaves/s', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms,
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded numpy rng)',
            'config': {'workload': 'cfg5: 3072x[1024]x8x10 MLP, eps 1/255 box, leaves of the '
                                   'depth-18 input-split tree, 9 robustness disjuncts',
                       'leaves_per_step_per_gpu': per_step,
                       'l2': 'inputs and generator matrices far larger than L2; flushed too',
                       'parallelism': f'{world} GPU(s), leaves sharded'},
            'roofline': {'bound': 'tensor', 'achieved': achieved, 'peak': peak,
                         'unit': 'TFLOP/s (fp32-equivalent, 3xTF32)',
                         'frac': achieved / peak, 'traffic': None,
                         'kernel': 'vcb_tc_gemm (tc_gemm_kernel), zonotope generator GEMMs',
                         'gemm_share_of_step': gemm_ms / sum(per),
                         'peak_source': 'MEASURED_PEAKS.json bf16_tflops / 2 (TF32 rate) / 3 '
                                        '(three MMAs per fp32 product)' if bf16 else
                                        'fallback 1590 / 6'},
            'clocks': clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            ggc = wk.mlp_gg(w['layers'])
            n = 2
            lo, hi = wk.cfg5_leaves(w['xl'], w['xh'], 0, n)
            W_q, b_q = wk.margin_rows(10, t)
            t0 = time.perf_counter()
            sb, _ = ob.forward_zonotope_batched(lo, hi, ggc)
            ob.spec_backward_batched(sb, lo, hi, ggc, W_q, b_q)
            rate = n / (time.perf_counter() - t0)
            line['cpu_baseline'] = {'value': rate, 'unit': 'leaves/s', 'cores': os.cpu_count(),
                                    'kind': 'port',
                                    'sample': f'{n} leaves: numpy oracle zonotope + CROWN '
                                              '(BLAS threads)'}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_cfg5_full(args, per_rank=64):
    """cfg5's stated workload end to end: the input-split BaB of the cfg5
    robustness property through the sharded driver
    (shard._input_split_batched_sharded: root expansion on every rank, leaves
    dealt round-robin, NCCL all_gather of the status and send / recv
    rebalancing every 8 iterations) with per_rank leaves per GPU iteration,
    the worklist bounded at 262,144 leaves (the size of the depth-18 tree),
    root PGD off.  One timed run after one warm-up batch; the time is the max
    over ranks of CUDA events around the driver."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    dev = torch.device(f'cuda:{local}')
    torch.cuda.set_device(dev)
    os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
    os.environ.setdefault('MASTER_PORT', '29533')
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=timedelta(seconds=600),
                            device_id=dev)
    from vibecheck_nn_b200 import bab, shard, workloads as wk
    w = wk.cfg5(0)
    gg = wk.mlp_gg(w['layers'], dev)
    spec = bab.LinearSpec(w['xl'], w['xh'], wk.robustness_disjuncts(10, w['true_label']))
    max_wl = 262_144
    st = wk.reference_bab_settings(input_split_batch_size=per_rank, disable_sat_finding=True,
                                   input_split_batched_max_worklist=max_wl,
                                   total_timeout=3600.0)
    eng = bab.make_engine(spec, gg, st, dev)
    lo, hi = wk.cfg5_leaves(w['xl'], w['xh'], 0, per_rank)
    eng.process(torch.as_tensor(lo, device=dev), torch.as_tensor(hi, device=dev), 0)
    del eng
    props = torch.cuda.get_device_properties(dev)
    gid = getattr(props, 'uuid', None)
    gid = f'GPU-{gid}' if gid is not None else local
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(gid) as clk:
        e0.record(stream)
        verdict, det = shard._input_split_batched_sharded(None, spec, st, gg, dev,
                                                          torch.float32, per_rank=per_rank)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    mine = torch.tensor([e0.elapsed_time(e1) / 1e3, det.get('shard_expand_s', 0.0),
                         det.get('shard_sync_s', 0.0), det.get('shard_transfer_s', 0.0)],
                        dtype=torch.float64, device=dev)
    allv = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allv, mine)
    per = torch.stack(allv).cpu().numpy()
    t = float(per[:, 0].max())
    leaves = int(det['batched_n_leaves'])
    if rank == 0:
        line = {
            'metric': 'cfg5 leaves/s (sharded input-split BaB, full run)',
            'value': leaves / t, 'unit': 'leaves/s', 'n_gpus': world, 'steps': 1,
            'warmup': 1, 'ms_per_step': 1e3 * t, 'higher_is_better': True,
            'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded numpy rng)',
            'config': {'workload': 'cfg5: 3072x[1024]x8x10 MLP, eps 1/255 box, 9 robustness '
                                   'disjuncts, input-split BaB (zonotope intermediates + '
                                   'CROWN spec bound, widest-dimension bisection) until the '
                                   f'worklist exceeds {max_wl} leaves',
                       'leaves_per_gpu_iteration': per_rank, 'parallelism':
                           f'{world} GPU(s): leaves dealt round-robin, NCCL status all_gather '
                           'and send/recv rebalancing every 8 iterations'},
            'verdict': verdict, 'phase': det.get('phase'), 'leaves': leaves,
            'worklist_at_stop': det.get('worklist_size'),
            'shard_leaves': det.get('shard_leaves'), 'shard_rounds': det.get('shard_rounds'),
            'shard_transfers': det.get('shard_transfers'),
            'phases_s': {'total_per_rank': per[:, 0].tolist(),
                         'root_expansion_per_rank': per[:, 1].tolist(),
                         'status_all_gather_incl_wait_per_rank': per[:, 2].tolist(),
                         'rebalance_send_recv_per_rank': per[:, 3].tolist()},
            'clocks': clk.summary(),
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == 'reference':
        run_reference(args)
    elif args.config == 'cfg1':
        run_cfg1(args)
    elif args.config in ('cfg3', 'cfg4'):
        run_cfg34(args)
    elif args.config == 'cfg5' and args.full:
        run_cfg5_full(args)
    elif args.config == 'cfg5':
        run_cfg5(args, per_step=args.cfg5_leaves)
    else:
        run_ours(args)


if __name__ == '__main__':
    main()
