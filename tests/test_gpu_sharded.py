"""Point-sharded engine groups on two GPUs (NCCL) against one engine holding
all samples. Needs at least two B200s; skipped otherwise.

Each rank runs in its own spawned process with an engine from
cpde_engine_create_sharded; rank 0 also runs an unsharded engine on the same
inputs. Tolerances: losses and per-layer normwise weight-gradient errors below
1e-5 (orders <= 3; the sums only change order), evaluation outputs gathered by
download identical to the unsharded ones, and RPROP weights after five epochs
bitwise identical across ranks.
"""
import numpy as np
import pytest

from cpde_b200 import codegen
from cpde_b200.client import sum_graph
from cpde_b200.expressions import quadrature_inputs
from cpde_b200.wire import Writer

pytestmark = pytest.mark.gpu

torch = pytest.importorskip('torch')


def _inputs():
    rng = np.random.default_rng(11)
    rows = codegen.SCHEMAS[3][1]  # full 2D order 3
    table = np.array([(sum(r), *r) for r in rows], np.int32)
    layers, linear = [2, 128, 128, 128, 1], [1, 0, 0, 0, 1]
    P = 3001  # odd: the shards differ by one sample
    x = quadrature_inputs(rng.uniform(-1, 1, (P, 2)), table)
    weights = [(rng.normal(size=h * (w + 1)) / np.sqrt(w)).astype(np.float32)
               for w, h in zip(layers[:-1], layers[1:])]
    target = rng.normal(size=(len(table), 1, P)).astype(np.float32)
    return table, layers, linear, x, weights, target


def _train_body(net, costs, epochs):
    # op-8 request: RPROP, fresh state, default steps, no logging/evaluation/saves
    w = (Writer().put('Q', net).array(costs, 'u8').put('Q', epochs).put('i', 0)
         .put('i', 1).put('f', 0.0).put('i', 0).put('f', 0.0))
    for value in (0, 1, 0, 0, 0):
        w.put('i', value)
    return w.string('').put('i', 0).bytes()


def _run(engine):
    from cpde_b200.native import EngineError
    table, layers, linear, x, weights, target = _inputs()
    R = len(table)
    out = {}
    net = engine.network(layers, weights, linear)
    data = engine.data(x, table)
    out['outputs'] = engine.download(engine.evaluate(net, data, chunk=500))
    tgt = engine.data(target, table)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32),
                           chunk=700)
    out['value'], out['grads'] = engine.graph_evaluate(net, [cost], sum_graph(1))
    engine.train(_train_body(net, [cost], 5))
    out['weights'] = [layer['buffers'][0] for layer in engine.state(net)[1]]
    bad = target.copy()
    bad[2, 0, 2900] = np.nan  # in rank 1's shard
    tgt2 = engine.data(bad, table)
    cost2 = engine.matching(net, data, tgt2, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
    try:
        engine.train(_train_body(net, [cost2], 1))
        out['error'] = None
    except EngineError as e:
        out['error'] = str(e)
    return out


def _rank(rank, world, uid, queue):
    from cpde_b200 import native
    torch.cuda.set_device(rank)
    with native.Engine(rank, rank, world, uid) as e:
        result = _run(e)
    reference = None
    if rank == 0:
        with native.Engine(0) as e:
            reference = _run(e)
    queue.put((rank, result, reference))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs two GPUs')
def test_two_gpu_group_matches_one_engine():
    import torch.multiprocessing as mp
    from cpde_b200 import native
    uid = native.sharding_id()
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, result, reference = queue.get(timeout=600)
        results[rank] = result
        if reference is not None:
            results['single'] = reference
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    single = results['single']
    for rank in (0, 1):
        r = results[rank]
        assert np.array_equal(r['outputs'], single['outputs'])
        assert abs(r['value'] - single['value']) <= 1e-5 * abs(single['value'])
        for a, b in zip(r['grads'], single['grads']):
            assert np.linalg.norm(np.asarray(a) - b) <= 1e-5 * np.linalg.norm(b)
        assert r['error'] is not None and r['error'] == single['error']
    for a, b in zip(results[0]['weights'], results[1]['weights']):
        assert np.array_equal(a, b)
    for a, b in zip(results[0]['weights'], single['weights']):
        assert np.allclose(a, b, rtol=1e-4, atol=1e-5)
