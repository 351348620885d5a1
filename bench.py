"""Benchmark of the cPDE epoch on B200s (driver contract: one JSON line on rank 0).

Workload: MLP 2->128->128->128->128->1 sigmoid,
float32, weights N(0, 1/fan_in) from seed 0 with zero biases, 65,536 points
uniform in [0,1]^2 (seed 1), every pure and mixed derivative through order 6
(28 rows), squared-error matching against sin(2 pi x) exp(-y) and its
derivatives with unit weights. One step = one fixed-weight epoch: forward of
all rows, loss, output adjoints and the weight gradients of every layer (the
reference's op-90 epoch, docs/benchmarks/fourier-timing.patch). Each rank
processes its own 65,536 points (weak scaling); for N > 1 the ranks exchange
gradients with one NCCL all-reduce per epoch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS = [2, 128, 128, 128, 128, 1]
ORDER = 6
POINTS = 65536
METRIC = 'points*derivs/s (2->128^4->1 sigmoid, order 6 all mixed, fixed-weight epoch)'
UNIT = 'points*derivs/s'


def workload(points=POINTS, order=ORDER, seed=1):
    from cpde_b200.expressions import all_mixed, glorot_like, quadrature_inputs
    t = all_mixed(order, 'xy')
    pts = np.random.default_rng(seed).uniform(0, 1, (points, 2))
    x = quadrature_inputs(pts, t)
    targets = np.zeros((len(t), 1, points), np.float32)
    for i, (_, a, b) in enumerate(t):
        targets[i, 0] = ((2 * np.pi) ** a * np.sin(2 * np.pi * pts[:, 0] + a * np.pi / 2)
                         * (-1.0) ** b * np.exp(-pts[:, 1]))
    return t, x, targets, glorot_like(LAYERS, seed=0)


def gemm_flops(points, rows):
    """Algorithmic GEMM FLOPs of one epoch (forward, weight and input gradients)."""
    pairs = list(zip(LAYERS[:-1], LAYERS[1:]))
    fwd = sum(2 * a * b for a, b in pairs)
    wgrad = sum(2 * (a + 1) * b for a, b in pairs)
    dgrad = sum(2 * a * b for a, b in pairs[1:])
    return points * rows * fwd, points * rows * dgrad, points * rows * wgrad


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.path = Path(tempfile.mkstemp(suffix='.csv')[1])
        query = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
                 'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
                 'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={index}', f'--query-gpu={query}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait()
        rows = [line.split(', ') for line in self.path.read_text().splitlines() if line.strip()]
        self.path.unlink()
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == 'Active'})
        return dict(sm_mhz=statistics.median(sm) if sm else None,
                    sm_max_mhz=float(rows[0][2]) if rows[0][2].replace('.', '').isdigit() else None,
                    samples=len(rows), reasons=reasons)


def measured_peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        return json.loads(path.read_text()), 'measured'
    return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0}, 'fallback'


# Algorithmic HBM bytes of one launch of each kernel on the config-2 network
# (2->128^4->1, C = points x rows columns, 4-byte floats): what the kernel
# must read and write at least once. forward: X_{l-1} in, Y_l out; backward:
# dZ_l and Y_{l-1} in, dZ_{l-1} out; backward_input: dZ_2, Y_1 and the inputs
# in; weight_gradient: dZ_l and Y_{l-1} in; head: Y_4 in, dZ_4 out, targets
# in; input_forward: inputs in, Y_1 out. Tensor-core kernels also carry
# 2 x 128 x 128 x C algorithmic FLOPs per launch (3 TF32 passes each).
def algorithmic_bytes(points, rows):
    c = points * rows * 4
    return {'forward_ws': (128 + 128) * c, 'backward_ws': (128 + 2 * 128) * c, 'backward_input_ws': (2 * 128 + 2) * c,
            'weight_gradient_ws': (128 + 128) * c, 'head_matching': (2 * 128 + 2) * c, 'input_forward': (2 + 128) * c,
            'forward_tc': (128 + 128) * c, 'backward_tc': (128 + 2 * 128) * c, 'backward_input_tc': (2 * 128 + 2) * c,
            'weight_gradient_tc': (128 + 128) * c}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch measured
# by ncu on the same kernels at 16,384 points and scaled x4 to a 65,536-point
# launch (the traffic is linear in the columns).
MEASURED_TRAFFIC = {'forward_ws': int(4 * (234.98 + 183.97) * 1e6), 'weight_gradient_ws': int(4 * (469.79 + 4.07) * 1e6),
                    'backward_ws': int(4 * (469.87 + 199.63) * 1e6), 'backward_input_ws': int(4 * (473.57 + 3.77) * 1e6),
                    'head_matching': int(4 * (236.82 + 187.90) * 1e6), 'input_forward': int(4 * (3.71 + 174.55) * 1e6)}


def hbm_roofline(kernels, steps, points, rows, peaks, source):
    """Achieved HBM bandwidth of every kernel class (algorithmic bytes per
    launch / mean launch time) and the roofline object of the class with the
    largest share of the step."""
    bytes_per_launch = algorithmic_bytes(points, rows)
    total = sum(v[1] for v in kernels.values())
    peak = peaks['hbm_gbs']
    rows_out = {}
    for name, (count, ms) in kernels.items():
        if name not in bytes_per_launch or count == 0:
            continue
        per_launch_s = ms / count / 1000
        achieved = bytes_per_launch[name] / per_launch_s / 1e9
        rows_out[name] = dict(achieved=achieved, frac=achieved / peak, share=ms / total,
                              ms_per_launch=per_launch_s * 1000, algorithmic_bytes=bytes_per_launch[name])
    if not rows_out:
        return None, rows_out
    top = max(rows_out, key=lambda k: rows_out[k]['share'])
    t = rows_out[top]
    roofline = dict(kernel=top, bound='hbm', achieved=t['achieved'], peak=peak, unit='GB/s', frac=t['frac'],
                    traffic=MEASURED_TRAFFIC.get(top), share=t['share'],
                    peak_source=f'hbm_gbs of MEASURED_PEAKS.json ({source}): {peak} GB/s, of measured',
                    algorithmic_bytes_per_launch=t['algorithmic_bytes'])
    return roofline, rows_out


def cpu_baseline(points=128, steps=2):
    """Reference CPU server (built from the reference's own sources) on a
    bounded sample of the same workload; serial engine, 1 core."""
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cpu_server'
    if not exe.exists():
        return None
    from cpde_b200.client import Data, Network, Session
    t, x, targets, weights = workload(points)
    with Session(exe) as s:
        net = Network(s, LAYERS, weights=weights)
        inp = Data(s, x, t)
        tgt = Data(s, targets, t)
        cost = net.matching(inp, tgt, np.ones((1, len(t)), np.float32))
        wall, _, _, _ = net.benchmark(cost, warm=0, iterations=1, batches=steps)
    ms = float(np.median(wall))
    return dict(value=points * len(t) / (ms / 1000), unit=UNIT, cores=1, kind='reference',
                sample=f'{points} of the {POINTS} points, {steps} op-90 epochs, median; '
                       'cpde_ref_cpu_server (oracle/Makefile), serial CPU backend',
                ms_per_epoch_sample=ms)


def reference_cuda(device, points=POINTS, iterations=3, batches=3):
    """The reference's own CUDA server, built for sm_100a from its sources by
    oracle/Makefile, timed with its op-90 command on the same GPU and workload."""
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cuda_server'
    if not exe.exists():
        return None
    from cpde_b200.client import Data, Network, Session
    t, x, targets, weights = workload(points)
    env = dict(os.environ)
    env.pop('NVIDIA_TF32_OVERRIDE', None)
    with Session(exe, device=device, env=env) as s:
        net = Network(s, LAYERS, weights=weights)
        inp = Data(s, x, t)
        tgt = Data(s, targets, t)
        cost = net.matching(inp, tgt, np.ones((1, len(t)), np.float32))
        wall, gpu, loss, _ = net.benchmark(cost, warm=1, iterations=iterations, batches=batches)
    ms = float(np.median(gpu))
    return dict(ms_per_epoch=ms, value=points * len(t) / (ms / 1000), unit=UNIT, loss=loss,
                how='oracle/_ref/cpde_ref_cuda_server (reference sources, nvcc sm_100a, cuBLAS FP32), '
                    f'op 90, median of {batches} batches x {iterations} epochs, device time')


def config3_inputs(points=262144):
    """Config 3's interior cost: points uniform in the unit disk (seed 2), rows
    u, u_y, u_x, u_yy, u_xx, integral of (u_xx + u_yy + 1)^2 with weights pi/N,
    net 2 -> 64^3 -> 1 sigmoid with N(0, 1/fan_in) weights (seed 0)."""
    from cpde_b200.expressions import Expression, quadrature_inputs, table
    rng = np.random.default_rng(2)
    r, th = np.sqrt(rng.uniform(size=points)), 2 * np.pi * rng.uniform(size=points)
    t = table(['xx', 'yy'], 'xy')
    x = quadrature_inputs(np.stack([r * np.cos(th), r * np.sin(th)], 1), t)
    layers = [2, 64, 64, 64, 1]
    g = np.random.default_rng(0)
    weights = [np.concatenate([g.normal(0, 1 / np.sqrt(a), (b, a)).ravel(order='F'), np.zeros(b)]).astype(np.float32)
               for a, b in zip(layers[:-1], layers[1:])]
    expr = Expression('(u_xx+u_yy+1)**2', table=t, variables='xy', outputs='u', count=points)
    return t, x, layers, weights, expr, np.full(points, np.pi / points)


def config3_integral(device, engine=None, iterations=10, batches=3):
    """ms/epoch (op 90: forward, integral cost, weight gradients) of config 3's
    interior cost on this engine and on the reference CUDA server, same GPU."""
    from cpde_b200 import native
    from cpde_b200.client import Data, Network, Session
    t, x, layers, weights, expr, qw = config3_inputs()
    own = engine or native.Engine(device)
    try:
        net = own.network(layers, weights)
        data = own.data(x, t)
        cost = own.integral(net, data, len(qw), np.asarray(expr.nodes, np.int32), np.asarray(expr.constants),
                            expr.field_array(), qw)
        _, dev, loss, _ = own.benchmark(net, cost, 3, iterations, batches, len(layers) - 1)
        for kind, h in ((2, cost), (0, data), (1, net)):
            own.release(kind, h)
    finally:
        if engine is None:
            own.close()
    out = dict(workload='config 3 interior: 262,144 points in the unit disk, rows u,u_x,u_y,u_xx,u_yy, '
                        'integral of (u_xx+u_yy+1)^2, 2->64^3->1 sigmoid, op-90 epochs, median device ms',
               ms=float(np.median(dev)), loss=loss, points_derivs_per_s=len(qw) * len(t) / (float(np.median(dev)) / 1e3))
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cuda_server'
    if exe.exists():
        env = dict(os.environ)
        env.pop('NVIDIA_TF32_OVERRIDE', None)
        with Session(exe, device=device, env=env) as s:
            rnet = Network(s, layers, weights=weights)
            rd = Data(s, x, t)
            rc = rnet.integral(rd, expr, weights=qw)
            _, rdev, rloss, _ = rnet.benchmark(rc, warm=3, iterations=iterations, batches=batches)
        out.update(reference_cuda_ms=float(np.median(rdev)), reference_loss=rloss,
                   speedup_vs_reference_cuda=float(np.median(rdev)) / out['ms'])
    return out


PUBLISHED_RTX3090_MS = [0.41, 0.68, 1.10, 1.72, 2.40, 3.59, 5.65]  # docs/benchmarks/fourier-rtx3090.md:23-29


def published_inputs(order):
    """The reference's published benchmark workload, regenerated from its
    description (scripts/benchmark_fourier_performance.py:20-38): 27 x 27 grid
    on [-1, 1]^2, all mixed derivatives through `order`, a 10 x 10 Fourier
    target with coefficients from seed 2026, rows weighted by the inverse
    variance of their targets, and the front end's seed-3407 initialisation
    (uniform +-2/sqrt(fan_in) weights, +-0.1 biases; cpde/api.py:277-280)."""
    from cpde_b200.expressions import all_mixed, quadrature_inputs
    t = all_mixed(order, 'xy')
    g = np.linspace(-1, 1, 27)
    gx, gy = np.meshgrid(g, g, indexing='ij')
    pts = np.column_stack((gx.ravel(), gy.ravel())).astype(np.float32).astype(np.float64)
    x, y = pts.T
    coef = np.random.default_rng(2026).uniform(-1, 1, (4, 10, 10))
    target = np.zeros((len(t), len(pts)))
    for row, (_, dx, dy) in enumerate(t):
        for n in range(1, 11):
            for k in range(1, 11):
                a, b, c, d = coef[:, n - 1, k - 1] * n ** int(dx) * k ** int(dy) / (n * k)
                sx, cx = np.sin(n * x + dx * np.pi / 2), np.cos(n * x + dx * np.pi / 2)
                sy, cy = np.sin(k * y + dy * np.pi / 2), np.cos(k * y + dy * np.pi / 2)
                target[row] += a * sx * sy + b * sx * cy + c * cx * sy + d * cx * cy
    weights = (1 / target.std(axis=1) ** 2).astype(np.float32)
    rng = np.random.default_rng(3407)
    init = [np.concatenate((rng.uniform(-2 / np.sqrt(w), 2 / np.sqrt(w), h * w),
                            rng.uniform(-.1, .1, h))).astype(np.float32)
            for w, h in zip(LAYERS[:-1], LAYERS[1:])]
    return t, quadrature_inputs(pts, t), target[:, None, :].astype(np.float32), weights, init


def published_workload(device, engine=None, iterations=50, batches=5):
    """ms/epoch (op-90 epochs: forward, loss, weight gradients) of this engine
    and of the reference CUDA server on the same GPU, orders 0..6."""
    from cpde_b200 import native
    from cpde_b200.client import Data, Network, Session
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cuda_server'
    rows = []
    own = engine or native.Engine(device)
    ref = Session(exe, device=device) if exe.exists() else None
    try:
        for order in range(7):
            t, x, target, weights, init = published_inputs(order)
            R = len(t)
            net = own.network(LAYERS, init)
            data = own.data(x, t)
            tgt = own.data(target, t)
            cost = own.matching(net, data, tgt, list(range(R)), list(range(R)), 1, weights[:, None, None])
            _, dev, loss, _ = own.benchmark(net, cost, 10, iterations, batches, len(LAYERS) - 1)
            entry = dict(order=order, rows=R, ms=float(np.median(dev)), loss=loss,
                         rtx3090_reference_ms=PUBLISHED_RTX3090_MS[order])
            for kind, h in ((2, cost), (0, tgt), (0, data), (1, net)):
                own.release(kind, h)
            if ref is not None:
                rnet = Network(ref, LAYERS, weights=init)
                rd, rt = Data(ref, x, t), Data(ref, target, t)
                rc = rnet.matching(rd, rt, weights[None, :])
                _, rdev, rloss, _ = rnet.benchmark(rc, 10, iterations, batches)
                entry.update(reference_cuda_ms=float(np.median(rdev)), reference_loss=rloss,
                             speedup_vs_reference_cuda=float(np.median(rdev)) / entry['ms'])
                rc.close(); rt.close(); rd.close(); rnet.close()
            rows.append(entry)
    finally:
        if ref is not None:
            ref.close()
        if engine is None:
            own.close()
    return dict(workload='27x27 grid on [-1,1]^2, 2->128^4->1 sigmoid, all mixed derivatives through the order, '
                         'Fourier matching (scripts/benchmark_fourier_performance.py), op-90 epochs, '
                         f'median of {batches} batches x {iterations}, device time; reference = the reference '
                         'CUDA server built for sm_100a on the same GPU',
                orders=rows)


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    steps = max(1, args.steps)
    base = cpu_baseline(points=args.reference_points, steps=steps)
    if base is None:
        print(json.dumps({'impl': 'reference', 'unavailable': 'oracle/_ref/cpde_ref_cpu_server is not built'}))
        return
    line = dict(metric=METRIC, value=base['value'], unit=UNIT, n_gpus=args.gpus, steps=steps, warmup=0,
                ms_per_step=base['ms_per_epoch_sample'], higher_is_better=True, scaling='weak', vs_baseline=None,
                dtype='f32', data='synthetic', impl='reference',
                config=dict(workload='config 2 (65,536 pts, order 6, 2->128^4->1), bounded sample',
                            sample_points=args.reference_points),
                cpu_baseline=dict(value=base['value'], unit=UNIT, cores=1, kind='reference',
                                  sample=base['sample']),
                e2e=dict(value=base['value'], unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line))


def run_b200(args):
    import torch
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=120), device_id=torch.device('cuda', local))
    from cpde_b200 import native, sharding
    # N > 1: one point-sharded group; every rank submits the whole N x points
    # workload and keeps its own contiguous shard of it
    engine = sharding.engine(local) if dist is not None else native.Engine(local)
    engine.set_tier(args.tier)
    t, x, targets, weights = workload(args.points * world)
    net = engine.network(LAYERS, weights)
    inp = engine.data(x, t)
    tgt = engine.data(targets, t)
    R = len(t)
    rows = list(range(R))
    cost = engine.matching(net, inp, tgt, rows, rows, 1, np.ones((R, 1, 1), np.float32))
    params = sum((a + 1) * b for a, b in zip(LAYERS[:-1], LAYERS[1:]))
    stream = torch.cuda.ExternalStream(engine.stream())

    def sync_all():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        engine.epoch(net, [cost])
    sync_all()
    engine.timing(True)
    engine.timing_report()
    clocks = Clocks(local)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_all()
    start.record(stream)
    for _ in range(args.steps):
        engine.epoch(net, [cost])
    stop.record(stream)
    torch.cuda.synchronize()
    clock = clocks.stop()
    ms = start.elapsed_time(stop) / args.steps
    kernels = engine.timing_report()
    engine.timing(False)
    if dist is not None:
        m = torch.tensor([ms], device='cuda')
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    value = world * args.points * R / (ms / 1000)

    # end to end through the public API: pinned host inputs in, objective and gradient out
    # pinned host copies already in the engine's (derivative, sample, channel) layout
    pinned_x = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).pin_memory()
    pinned_t = torch.from_numpy(np.ascontiguousarray(targets.transpose(0, 2, 1))).pin_memory()
    host_grad = np.zeros(params, np.float32)
    sync_all()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        engine.replace_raw(inp, pinned_x.data_ptr(), pinned_x.numel())
        engine.replace_raw(tgt, pinned_t.data_ptr(), pinned_t.numel())
        engine.epoch(net, [cost])
        loss, host_grad = engine.epoch_result(net, params)
    sync_all()
    e2e_ms = (time.perf_counter() - t0) * 1000 / args.steps
    if dist is not None:
        m = torch.tensor([e2e_ms], device='cuda')
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        e2e_ms = float(m.item())

    fwd, dgrad, wgrad = gemm_flops(args.points, R)
    peaks, source = measured_peaks()
    launches = sum(v[0] for v in kernels.values()) // args.steps
    roofline, kernel_rooflines = hbm_roofline(kernels, args.steps, args.points, R, peaks, source)
    if rank == 0:
        line = dict(metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
                    ms_per_step=ms, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='f32',
                    data='synthetic',
                    config=dict(workload='config 2: 65,536 pts/GPU, order 6 (28 rows), 2->128^4->1 sigmoid',
                                points_per_gpu=args.points, rows=R, l2='inputs larger than L2 (1 GB per layer)',
                                parallelism=f'dp{world}'),
                    e2e=dict(value=world * args.points * R / (e2e_ms / 1000), unit=UNIT,
                             h2d_bytes_per_step=int(pinned_x.numel() * 4 + pinned_t.numel() * 4),
                             d2h_bytes_per_step=int(world * (params * 4 + 8)), timer='host wall clock',
                             note='all ranks together copy the whole input once per step (each its shard) '
                                  'and each rank reads the all-reduced objective and gradient'),
                    gpu_launches=int(launches), roofline=roofline, kernel_rooflines=kernel_rooflines, clocks=clock,
                    kernels={k: dict(launches=v[0] // args.steps, ms_per_step=v[1] / args.steps)
                             for k, v in sorted(kernels.items())},
                    gemm_gflop_per_step=(fwd + dgrad + wgrad) / 1e9, loss=loss)
        if world == 1 and not args.no_cpu_baseline:
            line['cpu_baseline'] = cpu_baseline()
        if world == 1 and not args.no_reference_cuda:
            line['published_workload'] = published_workload(local, engine)
            line['config3_integral'] = config3_integral(local, engine)
            engine.close()
            ref = reference_cuda(local, args.points)
            if ref is not None:
                ref['speedup_of_value'] = value / ref['value']
                line['reference_cuda_same_gpu'] = ref
        print(json.dumps(line))
    engine.close()
    if dist is not None:
        dist.destroy_process_group()


def main():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    p.add_argument('--points', type=int, default=POINTS)
    p.add_argument('--reference-points', type=int, default=128)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-reference-cuda', action='store_true')
    p.add_argument('--tier', type=int, default=0, help='0 automatic, 1 generic, 2 tensor cores')
    args = p.parse_args()
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
