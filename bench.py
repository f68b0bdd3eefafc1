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
over ranks.  ``--impl reference`` times the CPU restatement of the
reference's algorithm (oracle/, numpy, all host cores) on a bounded sample of
the same workload.  Prints one JSON line on rank 0.
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
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU leg: the oracle (numpy restatement of the reference algorithm)
# ---------------------------------------------------------------------------

_WORKER = {}


def _cpu_worker(args):
    os.environ['OMP_NUM_THREADS'] = '1'
    os.environ['OPENBLAS_NUM_THREADS'] = '1'
    lo, hi = args
    from oracle import bounds as ob
    if 'w' not in _WORKER:
        from vibecheck_nn_b200 import workloads as wk
        _WORKER['w'] = wk.cfg2(seed=0, n_boxes=N_BOXES, n_q=N_Q)
        _WORKER['gg'] = wk.mlp_gg(_WORKER['w']['layers'])
    w, gg = _WORKER['w'], _WORKER['gg']
    t0 = time.perf_counter()
    sb = ob.ibp_forward_batched(w['xl'][lo:hi], w['xh'][lo:hi], gg)
    ob.spec_backward_batched(sb, w['xl'][lo:hi], w['xh'][lo:hi], gg,
                             w['spec_W'], w['spec_b'])
    return time.perf_counter() - t0


def cpu_rate(pool, cores, sample):
    """Boxes/s of the oracle on `sample` boxes split over `cores` processes."""
    per = (sample + cores - 1) // cores
    chunks = [(i * per, min(sample, (i + 1) * per)) for i in range(cores)]
    t0 = time.perf_counter()
    pool.map(_cpu_worker, chunks)
    return sample / (time.perf_counter() - t0)


def make_pool():
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    pool = mp.get_context('spawn').Pool(cores)
    pool.map(_cpu_worker, [(0, 64)] * cores)  # import + warm each worker
    return pool, cores


def cpu_baseline(pool, cores, budget_s=12.0):
    sample = 4096 * cores
    rates = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or len(rates) < 2:
        rates.append(cpu_rate(pool, cores, sample))
    return {'value': statistics.median(rates), 'unit': UNIT, 'cores': cores,
            'kind': 'port',
            'sample': f'{sample} of the 65,536 cfg2 boxes per repetition, '
                      f'{len(rates)} repetitions (median), numpy oracle '
                      f'(oracle/bounds.py) in {cores} spawn processes'}


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    pool, cores = make_pool()
    sample = 4096 * cores
    for _ in range(args.warmup):
        cpu_rate(pool, cores, sample)
    rates = [cpu_rate(pool, cores, sample) for _ in range(args.steps)]
    pool.close()
    v = statistics.median(rates)
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': v, 'unit': UNIT,
        'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': 1000.0 * N_BOXES / v, 'higher_is_better': True,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded)',
        'config': config_dict(args.gpus),
        'cpu_baseline': {'value': v, 'unit': UNIT, 'cores': cores,
                         'kind': 'port',
                         'sample': f'each step: {sample} cfg2 boxes, numpy '
                                   f'oracle in {cores} spawn processes'},
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
            'kernel': 'vcb_mlp_crown (crown_tc_kernel, tcgen05 3xTF32; the step also runs '
                      'crown_tc_images, <1% of its time)',
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
    pool = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        pool, cores = make_pool()  # spawn before the first GPU call
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
    cpu = None
    if pool is not None:
        cpu = cpu_baseline(pool, cores)
        pool.close()
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
            'gpu_launches': (2 if tc_path else 1) * args.steps,
            'roofline': roofline_cfg2(tc_path, achieved, peak, flop_per_box),
            'clocks': clk.summary(),
            'wall_s_timed_region': t_wall,
        }
        if cpu is not None:
            line['cpu_baseline'] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


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


def _time_steps(dev, step, args, world, flush, min_warmup=3):
    """W warm-up steps, then K timed steps (CUDA events, L2 flushed before
    each); returns (per-step ms, clocks summary, max-over-ranks total ms)."""
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
    with ClockSampler(gid) as clk:
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

    per, clocks, t_max = _time_steps(dev, step, args, world, flush)
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
            line['cpu_baseline'] = {
                'value': n_leaves / rate, 'unit': 's', 'cores': 1, 'kind': 'port',
                'sample': f'oracle/bab.py input-split BaB for 15 s ({rate:.0f} leaves/s, '
                          f'numpy), extrapolated to the {n_leaves} leaves of the verdict'}
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


def main():
    args = parse()
    if args.impl == 'reference':
        run_reference(args)
    elif args.config == 'cfg1':
        run_cfg1(args)
    elif args.config in ('cfg3', 'cfg4'):
        run_cfg34(args)
    elif args.config == 'cfg5':
        run_cfg5(args)
    else:
        run_ours(args)


if __name__ == '__main__':
    main()
