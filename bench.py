"""Benchmark of the cPDE epoch on B200s (driver contract: one JSON line on rank 0).

Workload (config 2, the headline configuration): MLP 2->128->128->128->128->1 sigmoid,
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
    """nvidia-smi sampling (every 50 ms) around the timed region. The sampler
    is started before the warm-up steps, so that nvidia-smi's own start-up
    does not overlap the timed steps (it added about 0.3 ms per step when it
    did); ``stop(window)`` keeps the samples whose timestamps fall inside the
    host wall-clock window of the timed region (or the first one after its
    start when the region is shorter than the sampling period)."""

    def __init__(self, index):
        self.path = Path(tempfile.mkstemp(suffix='.csv')[1])
        query = ('timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
                 'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
                 'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={index}', f'--query-gpu={query}',
                                          '--format=csv,noheader,nounits', '-lms', '50'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self, window=None):
        if self.proc is None:
            return None
        import datetime
        self.proc.terminate()
        self.proc.wait()
        rows = [line.split(', ') for line in self.path.read_text().splitlines() if line.strip()]
        self.path.unlink()

        def when(r):
            try:
                return datetime.datetime.strptime(r[0].strip(), '%Y/%m/%d %H:%M:%S.%f').timestamp()
            except ValueError:
                return None
        if window is not None:
            t0, t1 = window
            stamped = [(when(r), r) for r in rows]
            inside = [r for t, r in stamped if t is not None and t0 <= t <= t1]
            after = [r for t, r in stamped if t is not None and t >= t0]
            rows = inside or after[:1] or rows
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in rows for n, v in zip(names, r[6:10]) if v.strip() == 'Active'})
        return dict(sm_mhz=statistics.median(sm) if sm else None,
                    sm_max_mhz=float(rows[0][3]) if rows[0][3].replace('.', '').isdigit() else None,
                    samples=len(rows), reasons=reasons, interval_ms=50)


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


def cpu_baseline(points=512, steps=2, processes=None):
    """Reference CPU server (built from the reference's own sources by
    oracle/Makefile) on a bounded sample of the same workload. The build used
    is the one with the reference's CPDE_CPU_CBLAS option linked against the
    OpenBLAS that numpy ships (this image has no system CBLAS; 6.4x faster
    than the portable serial BLAS on a 256-point config-2 epoch, same loss);
    the portable serial build stands in where that one is absent. The
    server's jet, cost and reduction kernels are single-threaded, so it uses
    the host's cores the way the path shards: one server process per core
    (one BLAS thread each), each on its own `points`-point slice, all running
    their op-90 epochs at once; the throughput is the sum over processes
    (capped at 64 processes)."""
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cpu_server_blas'
    blas = exe.exists()
    if not blas:
        exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cpu_server'
    if not exe.exists():
        return None
    env = dict(os.environ)
    env['OPENBLAS_NUM_THREADS'] = '1'
    import threading
    from cpde_b200.client import Data, Network, Session
    if processes is None:
        processes = max(1, min(64, len(os.sched_getaffinity(0))))
    t, x, targets, weights = workload(points * processes)
    R = len(t)
    start = threading.Barrier(processes)
    results = [None] * processes

    def run(i):
        sl = slice(i * points, (i + 1) * points)
        with Session(exe, env=env) as s:
            net = Network(s, LAYERS, weights=weights)
            inp = Data(s, x[:, :, sl], t)
            tgt = Data(s, targets[:, :, sl], t)
            cost = net.matching(inp, tgt, np.ones((1, R), np.float32))
            start.wait()
            wall, _, _, _ = net.benchmark(cost, warm=0, iterations=1, batches=steps)
        results[i] = float(np.median(wall))

    threads = [threading.Thread(target=run, args=(i,)) for i in range(processes)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    ms = max(results)
    return dict(value=sum(points * R / (r / 1000) for r in results), unit=UNIT, cores=processes, kind='reference',
                sample=f'{processes} concurrent {exe.name} processes (oracle/Makefile, CPU backend, '
                       + ('CPDE_CPU_CBLAS against numpy\'s OpenBLAS, one BLAS thread each' if blas else
                          'portable serial BLAS') +
                       f', one per core), each on its own {points} of the workload\'s points, {steps} op-90 '
                       'epochs, median per process, throughput summed',
                ms_per_epoch_sample=ms)


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


class Workload:
    """One configuration: derivative table, input jets, network and cost,
    buildable on this engine (C ABI, cpde_b200.native) and on a reference
    server session (wire protocol, cpde_b200.client). ``cost`` is
    ('matching', targets, row_weights) | ('integral', nodes, constants,
    fields, quadrature_weights) | ('polynomial', terms, coefficients, rhs,
    point_weights); per-point arrays have the points on their last axis."""

    def __init__(self, name, t, x, layers, linear, weights, cost, chunk=0, reference_chunk=None):
        self.name, self.t, self.x, self.layers, self.linear = name, t, x, layers, linear
        self.weights, self.cost, self.chunk = weights, cost, chunk
        # the reference server refuses chunks whose activation buffers pass
        # its int32 size limit (cuda/cpde_server.cu:23-25), so wide networks
        # give it smaller chunks than this engine's
        self.reference_chunk = chunk if reference_chunk is None else reference_chunk

    @property
    def points(self):
        return self.x.shape[2]

    def subset(self, n):
        """The first n points (every per-point array sliced the same way)."""
        if n >= self.points:
            return self
        kind, *a = self.cost
        if kind == 'matching':
            cost = (kind, a[0][:, :, :n], a[1])
        elif kind == 'integral':
            cost = (kind, a[0], a[1], a[2][:, :n], a[3][:n])
        else:
            cost = (kind, a[0], a[1][:, :n], a[2][:, :n], a[3][:n])
        return Workload(self.name, self.t, self.x[:, :, :n], self.layers, self.linear, self.weights, cost,
                        min(self.chunk, n) if self.chunk else 0,
                        min(self.reference_chunk, n) if self.reference_chunk else 0)

    def own(self, e):
        """(net, data, cost) on a native engine."""
        net = e.network(self.layers, self.weights, self.linear)
        data = e.data(self.x, self.t)
        kind, *a = self.cost
        R = len(self.t)
        if kind == 'matching':
            tgt = e.data(a[0], self.t)
            cost = e.matching(net, data, tgt, list(range(R)), list(range(R)), 1, a[1], chunk=self.chunk)
        elif kind == 'integral':
            cost = e.integral(net, data, self.points, a[0], a[1], a[2], a[3], chunk=self.chunk)
        else:
            cost = e.polynomial(net, data, list(range(R)), 1, a[0], a[1], a[2], a[3], chunk=self.chunk)
        return net, data, cost

    def reference(self, session):
        """(net, data, cost) on a reference server; a tanh network goes there
        as its exact sigmoid reparametrisation (the reference has no tanh)."""
        from types import SimpleNamespace

        from cpde_b200.client import Data, Network
        from cpde_b200.expressions import tanh_as_sigmoid
        linear, weights = tanh_as_sigmoid(self.layers, self.linear, self.weights)
        net = Network(session, self.layers, weights=weights, linear=linear)
        data = Data(session, self.x, self.t)
        kind, *a = self.cost
        chunk = self.reference_chunk
        if kind == 'matching':
            cost = net.matching(data, Data(session, a[0], self.t), a[1][:, 0, :].T, chunk=chunk)
        elif kind == 'integral':
            expr = SimpleNamespace(nodes=a[0], constants=a[1], field_array=lambda: a[2], count=self.points)
            cost = net.integral(data, expr, weights=a[3], chunk=chunk)
        else:
            poly = [{(comp,): a[1][k] for k, (_, comp, _) in enumerate(a[0])}]
            cost = net.polynomial(data, poly, rhs=a[2], weights=a[3][None, :], chunk=chunk)
        return net, data, cost

    def reference_gradients(self, grads):
        from cpde_b200.expressions import sigmoid_gradients_to_tanh
        return sigmoid_gradients_to_tanh(self.layers, self.linear, grads)


def config2_workload(points=POINTS):
    t, x, targets, weights = workload(points)
    return Workload('config 2', t, x, LAYERS, [1, 0, 0, 0, 0, 1], weights,
                    ('matching', targets, np.ones((len(t), 1, 1), np.float32)))


def generic_workload(points=POINTS):
    """A schema the fused tiers do not compile ahead of time (3D, all mixed
    derivatives through order 2: 10 rows), on the config-2 widths: it runs the
    generic tier (FFMA GEMMs plus table-driven jet kernels), the path every
    user schema outside the generated ones takes. Matching against
    f = sin(2 pi x) exp(-y) cos(pi z) and its derivatives, points uniform in
    [0,1]^3 (seed 5)."""
    from cpde_b200.expressions import all_mixed, glorot_like, quadrature_inputs
    t = all_mixed(2, 'xyz')
    pts = np.random.default_rng(5).uniform(0, 1, (points, 3))
    targets = np.zeros((len(t), 1, points), np.float32)
    for i, (_, a, b, c) in enumerate(t):
        targets[i, 0] = ((2 * np.pi) ** a * np.sin(2 * np.pi * pts[:, 0] + a * np.pi / 2) * (-1.0) ** b
                         * np.exp(-pts[:, 1]) * np.pi ** c * np.cos(np.pi * pts[:, 2] + c * np.pi / 2))
    layers = [3, 128, 128, 128, 1]
    return Workload('generic tier: 3->128^3->1 sigmoid, 3D order 2 all mixed (10 rows)', t,
                    quadrature_inputs(pts, t), layers, [1, 0, 0, 0, 1], glorot_like(layers, seed=0),
                    ('matching', targets, np.ones((len(t), 1, 1), np.float32)))


def config3_workload(points=262144):
    t, x, layers, weights, expr, qw = config3_inputs(points)
    return Workload('config 3 interior', t, x, layers, [1, 0, 0, 0, 1], weights,
                    ('integral', np.asarray(expr.nodes, np.int32), np.asarray(expr.constants), expr.field_array(), qw))


def config4_workload(points=1048576, chunk=262144, reference_chunk=65536):
    t, x, layers, linear, weights, expr, qw = config4_inputs(points)
    return Workload('config 4', t, x, layers, linear, weights,
                    ('integral', np.asarray(expr.nodes, np.int32), np.asarray(expr.constants), expr.field_array(), qw),
                    chunk, reference_chunk)


def config5_workload(points=4194304, chunk=131072, reference_chunk=32768):
    t, x, layers, linear, weights, terms, coeffs, rhs, pw = config5_inputs(points)
    return Workload('config 5', t, x, layers, linear, weights, ('polynomial', terms, coeffs, rhs, pw), chunk,
                    reference_chunk)


def epoch_gemm_flops(layers, rows, points):
    """Algorithmic GEMM FLOPs of one epoch: forward, weight gradient (bias
    column included) and input gradient of every layer but the first."""
    pairs = list(zip(layers[:-1], layers[1:]))
    return 2 * rows * points * (sum(a * b for a, b in pairs) + sum((a + 1) * b for a, b in pairs)
                                + sum(a * b for a, b in pairs[1:]))


def tensor_roofline(w, ms, peaks, source):
    """The epoch's GEMM work against the tensor cores' TF32 rate: a 3xTF32
    product is three TF32 MMAs, so the algorithmic ceiling is a third of the
    TF32 rate, which is half the dense bf16 rate (sustained figure of
    MEASURED_PEAKS.json: the epoch runs for seconds under the power cap)."""
    flops = epoch_gemm_flops(w.layers, len(w.t), w.points)
    bf16 = peaks.get('bf16_tflops_sustained', peaks['bf16_tflops'])
    peak = bf16 / 2 / 3
    achieved = flops / (ms / 1e3) / 1e12
    return dict(bound='tensor', achieved=achieved, peak=peak, unit='TFLOP/s', frac=achieved / peak,
                gemm_tflop_per_epoch=flops / 1e12,
                peak_source=f'bf16_tflops_sustained of MEASURED_PEAKS.json ({source}) {bf16} / 2 (TF32) / 3 '
                            '(3xTF32 passes), of measured')


def _layer_errors(actual, expected):
    return [float(np.linalg.norm(np.asarray(a, np.float64) - np.asarray(b, np.float64)) /
                  max(np.linalg.norm(np.asarray(b, np.float64)), 1e-300)) for a, b in zip(actual, expected)]


def _row_errors(actual, expected):
    a = np.asarray(actual, np.float64).reshape(len(actual), -1)
    b = np.asarray(expected, np.float64).reshape(len(expected), -1)
    norm = np.linalg.norm(b, axis=1)
    return np.linalg.norm(a - b, axis=1) / np.where(norm > 0, norm, 1.0)


def same_gpu_comparison(device, w, warm=1, iterations=3, batches=1, reference_points=None, sample_points=4096,
                        kernels=False, tier=0):
    """op-90 epochs (forward, cost, output adjoints, weight gradients) of one
    workload on this engine and on the reference CUDA server (built from the
    reference's sources for sm_100a by oracle/Makefile) on the same GPU, with
    parity: per-layer normwise relative error of the op-90 weight gradients
    and per-row normwise relative error of op-4 outputs on the first
    ``sample_points`` points, this engine against the reference. The
    reference runs on the first ``reference_points`` points when that is
    smaller than the workload (its time is then scaled by the point ratio and
    marked extrapolated); the gradients are compared on that same subset."""
    from cpde_b200 import native
    from cpde_b200.client import Session
    L = len(w.layers) - 1
    R = len(w.t)
    sub = w.subset(reference_points or w.points)
    sample = w.subset(sample_points)
    out = dict(workload=w.name, points=w.points, rows=R, layers=w.layers, chunk=w.chunk or w.points, tier=tier)
    with native.Engine(device) as e:
        e.set_tier(tier)
        net, data, cost = w.own(e)
        _, dev, loss, grads = e.benchmark(net, cost, warm, iterations, batches, L)
        out.update(ms=float(np.median(dev)), loss=loss, points_derivs_per_s=w.points * R / (float(np.median(dev)) / 1e3))
        if kernels:
            e.timing(True)
            e.timing_report()
            e.epoch(net, [cost])
            e.epoch_result(net, sum(np.asarray(x).size for x in w.weights))
            rep = e.timing_report()
            e.timing(False)
            out['kernels'] = {k: dict(launches=v[0], ms=round(v[1], 4)) for k, v in sorted(rep.items())}
        for kind, h in ((2, cost), (0, data), (1, net)):
            e.release(kind, h)
        if sub is not w:
            net, data, cost = sub.own(e)
            _, _, sub_loss, grads = e.benchmark(net, cost, 0, 1, 1, L)
        else:
            sub_loss = loss
        net, data, _ = sample.own(e)
        own_rows = e.download(e.evaluate(net, data, chunk=sample.chunk))
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cuda_server'
    if not exe.exists():
        return out
    env = dict(os.environ)
    env.pop('NVIDIA_TF32_OVERRIDE', None)
    try:
        with Session(exe, device=device, env=env) as s:
            rnet, _, rcost = sub.reference(s)
            _, rdev, rloss, rgrads = rnet.benchmark(rcost, warm=warm, iterations=iterations, batches=batches)
            rnet, rdata, _ = sample.reference(s)
            ref_rows = rnet.eval(rdata, chunk=sample.reference_chunk).to_numpy()
    except Exception as exc:  # the reference server exits on CUDA errors (e.g. out of memory)
        out['reference_error'] = f'{type(exc).__name__}: {exc}'
        return out
    rgrads = w.reference_gradients(rgrads)
    ref_ms = float(np.median(rdev)) * w.points / sub.points
    out.update(reference_cuda_ms=ref_ms, speedup_vs_reference_cuda=ref_ms / out['ms'],
               reference_loss=rloss,
               reference_how=('oracle/_ref/cpde_ref_cuda_server (reference sources, nvcc sm_100a, cuBLAS FP32), '
                              f'op 90, median of {batches} x {iterations} epochs, device time'
                              + (f'; timed on the first {sub.points} points and scaled by {w.points / sub.points:g} '
                                 '(extrapolated: the epoch is linear in the points)' if sub is not w else '')),
               parity=dict(points=sub.points, loss_relative=abs(sub_loss - rloss) / abs(rloss),
                           gradient_layer_errors=_layer_errors(grads, rgrads),
                           output_points=sample.points, output_row_error_max=float(_row_errors(own_rows, ref_rows).max()),
                           against='reference CUDA server (float32, cuBLAS) on the same inputs'))
    out['parity']['gradient_error_max'] = max(out['parity']['gradient_layer_errors'])
    return out


def config4_inputs(points=1048576):
    """Config 4: 3D biharmonic residual (Delta^2 u - g)^2 with
    g = sin(pi x) sin(pi y) sin(pi z) as a field, every pure and mixed
    derivative through order 4 (35 rows) on points uniform in [0,1]^3
    (seed 3), quadrature weights 1/N, net 3 -> 256^5 -> 1 tanh with
    N(0, 1/fan_in) weights (seed 0)."""
    from cpde_b200.expressions import Expression, all_mixed, glorot_like, quadrature_inputs
    pts = np.random.default_rng(3).uniform(0, 1, (points, 3))
    t = all_mixed(4, 'xyz')
    x = quadrature_inputs(pts, t)
    layers = [3, 256, 256, 256, 256, 256, 1]
    linear = [1, 2, 2, 2, 2, 2, 1]
    g = np.sin(np.pi * pts[:, 0]) * np.sin(np.pi * pts[:, 1]) * np.sin(np.pi * pts[:, 2])
    expr = Expression('(u_xxxx+u_yyyy+u_zzzz+2*u_xxyy+2*u_xxzz+2*u_yyzz-g)**2', table=t, variables='xyz',
                      outputs='u', parameters={'g': g}, count=points)
    return t, x, layers, linear, glorot_like(layers, seed=0), expr, np.full(points, 1.0 / points)


def config5_inputs(points=4194304):
    """Config 5: value plus pure derivatives through order 6 along 4 axes
    (25 rows) on points uniform in [-1,1]^4 (seed 4), one polynomial residual
    sum_a u_{a^6} (unit coefficients, rhs 0) with per-point weights U(0,1)
    from the same generator, net 4 -> 512^6 -> 1 sigmoid (seed-0 weights)."""
    from cpde_b200.expressions import glorot_like, pure, quadrature_inputs
    rng = np.random.default_rng(4)
    pts = rng.uniform(-1, 1, (points, 4))
    weights = rng.uniform(0, 1, points).astype(np.float32)
    t = pure(6, 'xyzw')
    x = quadrature_inputs(pts, t)
    layers = [4] + [512] * 6 + [1]
    linear = [1] + [0] * 6 + [1]
    sixth = [i for i, row in enumerate(t) if row[0] == 6]
    terms = [(0, i, -1) for i in sixth]
    coeffs = np.ones((len(terms), points), np.float32)
    return t, x, layers, linear, glorot_like(layers, seed=0), terms, coeffs, np.zeros((1, points), np.float32), weights


def config3_boundary_inputs(points=4096):
    """Config 3's boundary cost: equispaced points on the unit circle, weight
    2 pi / N each, integral of u^2 (value row only)."""
    from cpde_b200.expressions import Expression, quadrature_inputs, table
    phi = 2 * np.pi * np.arange(points) / points
    t = table([''], 'xy')
    x = quadrature_inputs(np.stack([np.cos(phi), np.sin(phi)], 1), t)
    expr = Expression('u**2', table=t, variables='xy', outputs='u', count=points)
    return t, x, expr, np.full(points, 2 * np.pi / points)


def train_request(net, costs, epochs, log_every, optimizer=0):
    """Op-8 payload (cuda/cpde_server.cu:365-371): fresh optimizer state,
    default steps, values reported every `log_every` epochs."""
    from cpde_b200.wire import Writer
    w = (Writer().put('Q', net).array(list(costs), 'u8').put('Q', epochs).put('i', optimizer).put('i', 1)
         .put('f', 0.0).put('i', 0).put('f', 0.0))
    for value in (0, log_every, 0, 0, 0):
        w.put('i', value)
    return w.string('').put('i', 0).bytes()


def _max_over_ranks(dist, value):
    if dist is None:
        return value
    import torch
    m = torch.tensor([value], device='cuda')
    dist.all_reduce(m, op=dist.ReduceOp.MAX)
    return float(m.item())


def config3_training(engine, dist, epochs=500, log_every=100, reference_device=None):
    """Config 3 as specified: `epochs` RPROP epochs (op 8: forward, both
    integral costs, weight gradients, validation and the update, one host
    synchronisation per epoch like the reference) of the interior residual
    (262,144 points in the disk) and the boundary term (4,096 circle points),
    2 -> 64^3 -> 1 sigmoid. With N ranks the points of both costs are split
    over them (strong scaling). Device time of the whole run on the engine's
    stream, max over ranks; the objective every `log_every` epochs. With
    `reference_device`, the reference CUDA server trains the same problem on
    that GPU (wall clock of its op 8)."""
    import torch
    from cpde_b200.wire import Reader
    t, x, layers, weights, expr, qw = config3_inputs()
    tb, xb, eb, qb = config3_boundary_inputs()
    net = engine.network(layers, weights)
    data, bdata = engine.data(x, t), engine.data(xb, tb)
    interior = engine.integral(net, data, len(qw), np.asarray(expr.nodes, np.int32), np.asarray(expr.constants),
                               expr.field_array(), qw)
    boundary = engine.integral(net, bdata, len(qb), np.asarray(eb.nodes, np.int32), np.asarray(eb.constants),
                               eb.field_array(), qb)
    engine.train(train_request(net, [interior, boundary], 3, 0))  # warm-up: compile, allocate
    engine.set_weights(net, weights)
    stream = torch.cuda.ExternalStream(engine.stream())
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start.record(stream)
    events = engine.train(train_request(net, [interior, boundary], epochs, log_every))
    stop.record(stream)
    torch.cuda.synchronize()
    ms = _max_over_ranks(dist, start.elapsed_time(stop) / epochs)
    curve = []
    for kind, payload in events:
        if kind == 2:
            r = Reader(payload)
            epoch, _, after, values = r.get('Q'), r.get('Q'), r.get('i'), r.array('f8')
            curve.append([int(epoch), float(values.sum())])
    for kind, h in ((2, interior), (2, boundary), (0, data), (0, bdata), (1, net)):
        engine.release(kind, h)
    world = dist.get_world_size() if dist is not None else 1
    out = dict(workload='config 3: 500 RPROP epochs (op 8) of the interior (262,144 disk points, '
                        '(u_xx+u_yy+1)^2) and boundary (4,096 circle points, u^2) integrals, 2->64^3->1 sigmoid',
               scaling='strong', n_gpus=world, epochs=epochs, ms_per_epoch=ms,
               points_derivs_per_s=(len(qw) * len(t) + len(qb) * len(tb)) / (ms / 1e3), objective_curve=curve,
               timer='CUDA events on the engine stream around the whole op-8 run, max over ranks')
    exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cuda_server'
    if reference_device is not None and exe.exists():
        from cpde_b200.client import Data, Network, Session
        env = dict(os.environ)
        env.pop('NVIDIA_TF32_OVERRIDE', None)
        try:
            with Session(exe, device=reference_device, env=env) as s:
                rnet = Network(s, layers, weights=weights)
                rc = [rnet.integral(Data(s, x, t), expr, weights=qw), rnet.integral(Data(s, xb, tb), eb, weights=qb)]
                rnet.train(rc, 3, optimizer='rprop', reset=True, log_every=0)
                rnet.set_weights(weights)
                t0 = time.perf_counter()
                result = rnet.train(rc, epochs, optimizer='rprop', reset=True, log_every=log_every)
                wall = (time.perf_counter() - t0) * 1e3 / epochs
            rcurve = [[int(ev['epoch']), float(np.sum(ev['values']))] for ev in result['events'] if ev['kind'] == 2]
            out.update(reference_cuda_ms_per_epoch=wall, reference_objective_curve=rcurve,
                       speedup_vs_reference_cuda=wall / ms,
                       reference_how='oracle/_ref/cpde_ref_cuda_server, op 8 through the wire protocol, host wall '
                                     'clock of the whole run (it synchronises every epoch)')
        except Exception as exc:
            out['reference_error'] = f'{type(exc).__name__}: {exc}'
    return out


def orders_sweep(engine, dist, points_per_gpu, steps=5, warmup=2, reference_device=None):
    """ms per fixed-weight epoch of the config-2 network (2 -> 128^4 -> 1
    sigmoid, matching against sin(2 pi x) e^-y) at orders 0..6, with
    `points_per_gpu` points per rank (weak scaling), device time, max over
    ranks; with `reference_device`, op-90 epochs of the reference CUDA
    server on the same workload and GPU."""
    import torch
    world = dist.get_world_size() if dist is not None else 1
    stream = torch.cuda.ExternalStream(engine.stream())
    rows = []
    for order in range(7):
        t, x, targets, weights = workload(points_per_gpu * world, order=order)
        R = len(t)
        net = engine.network(LAYERS, weights)
        data, tgt = engine.data(x, t), engine.data(targets, t)
        cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
        for _ in range(warmup):
            engine.epoch(net, [cost])
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        start.record(stream)
        for _ in range(steps):
            engine.epoch(net, [cost])
        stop.record(stream)
        torch.cuda.synchronize()
        ms = _max_over_ranks(dist, start.elapsed_time(stop) / steps)
        entry = dict(order=order, rows=R, points=points_per_gpu * world, ms=ms,
                     points_derivs_per_s=points_per_gpu * world * R / (ms / 1e3))
        for kind, h in ((2, cost), (0, tgt), (0, data), (1, net)):
            engine.release(kind, h)
        exe = ROOT / 'oracle' / '_ref' / 'cpde_ref_cuda_server'
        if reference_device is not None and exe.exists():
            from cpde_b200.client import Data, Network, Session
            env = dict(os.environ)
            env.pop('NVIDIA_TF32_OVERRIDE', None)
            with Session(exe, device=reference_device, env=env) as s:
                rnet = Network(s, LAYERS, weights=weights)
                rc = rnet.matching(Data(s, x, t), Data(s, targets, t), np.ones((1, R), np.float32))
                _, rdev, _, _ = rnet.benchmark(rc, warm=1, iterations=2, batches=1)
            entry.update(reference_cuda_ms=float(np.median(rdev)), speedup_vs_reference_cuda=float(np.median(rdev)) / ms)
        rows.append(entry)
    return dict(workload=f'2->128^4->1 sigmoid, all mixed derivatives through the order, {points_per_gpu} points '
                         'per GPU (weak scaling), fixed-weight epochs, device time, max over ranks',
                orders=rows)


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
                cpu_baseline=dict(value=base['value'], unit=UNIT, cores=base['cores'], kind='reference',
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

    clocks = Clocks(local)
    time.sleep(0.5)  # the sampler is running before the warm-up
    for _ in range(args.warmup):
        engine.epoch(net, [cost])
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_all()
    wall0 = time.time()
    start.record(stream)
    for _ in range(args.steps):
        engine.epoch(net, [cost])
    stop.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    clock = clocks.stop((wall0, wall1))
    ms = start.elapsed_time(stop) / args.steps
    # per-kernel CUDA-event times (launch counts, shares, rooflines) from a
    # second pass of the same steps: the events recorded around every launch
    # are kept out of the timed region above
    sync_all()
    engine.timing(True)
    engine.timing_report()
    for _ in range(args.steps):
        engine.epoch(net, [cost])
    torch.cuda.synchronize()
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

    for h, kind in ((cost, 2), (tgt, 0), (inp, 0), (net, 1)):
        engine.release(kind, h)
    legs = {}
    if not args.no_scaling_legs:
        ref_dev = local if world == 1 and not args.no_reference_cuda else None
        legs['orders_weak'] = orders_sweep(engine, dist, args.points, reference_device=ref_dev)
        legs['config3_training'] = config3_training(engine, dist, reference_device=ref_dev)

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
                    gemm_gflop_per_step=(fwd + dgrad + wgrad) / 1e9, loss=loss, **legs)
        if world == 1 and not args.no_cpu_baseline:
            line['cpu_baseline'] = cpu_baseline()
        if world == 1 and not args.no_reference_cuda:
            line['published_workload'] = published_workload(local, engine)
            engine.close()
            ref = same_gpu_comparison(local, config2_workload(args.points), warm=1, iterations=3, batches=3)
            if 'reference_cuda_ms' in ref:
                ref['speedup_of_value'] = ref['reference_cuda_ms'] / ms
            line['reference_cuda_same_gpu'] = ref
            line['parity'] = ref.get('parity')
            line['config3_integral'] = same_gpu_comparison(local, config3_workload(), warm=3, iterations=10,
                                                           batches=3, kernels=True)
            # the same at tier 4: exact-FP32 FFMA layers (the automatic tier runs this
            # 64-wide order-2 network on the 3xTF32 tensor cores)
            line['config3_integral_ffma'] = same_gpu_comparison(local, config3_workload(), warm=3, iterations=10,
                                                                 batches=3, kernels=True, tier=4)
            # a schema outside the generated fast-tier ones (generic tier)
            line['generic_tier'] = same_gpu_comparison(local, generic_workload(), warm=2, iterations=5, batches=3,
                                                       kernels=True)
            if not args.no_large_configs:
                peaks, source = measured_peaks()
                for key, make, ref_points in (('config4', config4_workload, 262144),
                                              ('config5', config5_workload, 262144)):
                    w = make()
                    entry = same_gpu_comparison(local, w, warm=1, iterations=1, batches=1,
                                                reference_points=ref_points, kernels=True)
                    entry['tensor_roofline'] = tensor_roofline(w, entry['ms'], peaks, source)
                    line[key] = entry
                    del w
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
    p.add_argument('--reference-points', type=int, default=512)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-reference-cuda', action='store_true')
    p.add_argument('--tier', type=int, default=0,
                   help='0 automatic, 1 generic, 2 tensor cores, 3 point-tile epochs, 4 exact-FP32 FFMA')
    p.add_argument('--no-large-configs', action='store_true', help='skip the config-4 and config-5 legs')
    p.add_argument('--no-scaling-legs', action='store_true',
                   help='skip the order sweep and the config-3 training run (both run at every N)')
    p.add_argument('--profile-workload', choices=sorted(WORKLOADS),
                   help='only run --warmup + --steps plain epochs of one workload on GPU 0 (a short, '
                        'self-contained command to profile) and print its ms per epoch')
    p.add_argument('--epoch-times', action='store_true',
                   help='with --profile-workload: also time every epoch (CUDA events between epochs) and print '
                        'the means of consecutive groups of 10, which show the GPU settling at its power cap')
    args = p.parse_args()
    if args.profile_workload:
        profile_workload(args)
    elif args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


WORKLOADS = {'config2': lambda points: config2_workload(points or POINTS),
             'generic': lambda points: generic_workload(points or POINTS),
             'config3': lambda points: config3_workload(points or 262144),
             'config4': lambda points: config4_workload(points or 1048576),
             'config5': lambda points: config5_workload(points or 4194304)}


def profile_workload(args):
    """Plain fixed-weight epochs of one workload (the same engine calls as the
    bench's timed loop) with device timing, nothing else: the command that
    the kernel profiles under profiles/ are taken from. --points overrides
    the workload's point count (its default otherwise)."""
    import torch
    from cpde_b200 import native
    w = WORKLOADS[args.profile_workload](args.points if args.points != POINTS else 0)
    with native.Engine(0) as e:
        e.set_tier(args.tier)
        net, data, cost = w.own(e)
        for _ in range(args.warmup):
            e.epoch(net, [cost])
        stream = torch.cuda.ExternalStream(e.stream())
        events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1 if args.epoch_times else 2)]
        torch.cuda.synchronize()
        events[0].record(stream)
        for i in range(args.steps):
            e.epoch(net, [cost])
            if args.epoch_times:
                events[i + 1].record(stream)
        events[-1].record(stream)
        torch.cuda.synchronize()
        loss, _ = e.epoch_result(net, sum(np.asarray(x).size for x in w.weights))
    line = dict(workload=w.name, points=w.points, tier=args.tier, steps=args.steps,
                ms_per_epoch=events[0].elapsed_time(events[-1]) / max(1, args.steps), loss=loss)
    if args.epoch_times:
        ms = [events[i].elapsed_time(events[i + 1]) for i in range(args.steps)]
        line['ms_per_epoch_by_10'] = [round(float(np.mean(ms[i:i + 10])), 3) for i in range(0, args.steps, 10)]
    print(json.dumps(line))


if __name__ == '__main__':
    main()
