"""The multi-GPU path (P2P all-gather, dispatch and combine over NVSwitch,
replicated device planner) on 2, 4 and 8 GPUs (as many as the box has): one
process per GPU runs OffloadRuntime.execute; the oracle emulates the same
ranks in one process.  Cache decisions bit-exact on every rank, outputs
within the BF16 tolerance.  Failure detection at 2 GPUs: a rank that leaves
out its dispatch or combine flag stores (a host-side omission) makes the
peers' bounded waits run out; every rank then reports FERRYB_ETIMEOUT and
its output rows are NaN.  Skipped where the GPUs are missing."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import expert_ops as ref_ops
from oracle.layer import OracleRuntime
from tests.tolerance import assert_bf16_close

pytestmark = pytest.mark.gpu

# shape (layers, experts, topk, hidden, intermediate), tokens per rank,
# capacities as a function of the world size, steps
CASES = {
    'small': ((3, 32, 4, 256, 128), 12, lambda w: [min(16, 96 // w)] * w, 9),
    'qwen3': ((2, 128, 8, 2048, 768), 64, lambda w: [210 // w + (r < 210 % w) for r in range(w)], 6),
}
WORLDS = (2, 4, 8)


def _need(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')


def _spec(shape):
    from ferry_b200.model import ModelSpec
    layers, E, K, H, I = shape
    return ModelSpec('qwen3_moe', tuple(range(layers)), E, K, H, I)


def _world_inputs(spec, step, rank, T):
    from ferry_b200.workload import zipf_bias
    g = torch.Generator().manual_seed(7)
    gates = [(torch.randn(spec.experts, spec.hidden, generator=g) * 0.02).to(torch.bfloat16)
             for _ in range(spec.layers)]
    biases = [zipf_bias(spec.experts, 1.1, g) for _ in range(spec.layers)]
    gx = torch.Generator().manual_seed(100 * step + rank)
    x = torch.randn(T, spec.hidden, generator=gx).to(torch.bfloat16)
    layer = step % spec.layers
    sel, w, _ = ref_ops.route_qwen3(x, gates[layer], spec.topk, True, biases[layer])
    return layer, x, sel, w


def _worker(rank, world, port, case, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import cpu_pool
    torch.cuda.set_device(rank)
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    shape, T, caps_of, steps = CASES[case]
    caps = caps_of(world)
    spec = _spec(shape)
    pool = cpu_pool(spec, spec.layers, 0).pin_memory()
    rt = OffloadRuntime(spec, pool, caps, 'ferry', Topology.uniform(world, spec.experts))
    outs = []
    for step in range(steps):
        layer, x, sel, w = _world_inputs(spec, step, rank, T)
        got = rt.execute(layer, x.cuda(), sel.cuda(), w.cuda(), None)
        outs.append(got.cpu())
    torch.cuda.synchronize()
    torch.save({'outs': outs, 'slots': rt.controller.slots, 'owner': rt.controller.owner,
                'fetches': rt.fetches_per_rank, 'dispatch_bytes': rt.dispatch_bytes},
               os.path.join(out_dir, f'rank{rank}.pt'))
    dist.barrier()
    rt.close()
    dist.destroy_process_group()


@pytest.mark.parametrize('world', WORLDS)
@pytest.mark.parametrize('case', list(CASES))
def test_multi_gpu_execute_matches_oracle(case, world):
    _need(world)
    shape, T, caps_of, steps = CASES[case]
    caps = caps_of(world)
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_worker, args=(world, 29700 + 10 * world + len(case), case, tmp), nprocs=world)
        res = [torch.load(os.path.join(tmp, f'rank{r}.pt'), weights_only=False) for r in range(world)]
    spec = _spec(shape)
    from ferry_b200.workload import cpu_pool
    from oracle import planner as op
    pool = cpu_pool(spec, spec.layers, 0)
    masks = np.asarray([1 << r for r in range(world)], np.int64)
    lut = op.build_lut(spec.experts, world, masks, np.ones(world))
    orc = OracleRuntime(spec, pool, caps, 'ferry', masks, np.ones(world), lut)
    for step in range(steps):
        per = [_world_inputs(spec, step, r, T) for r in range(world)]
        want, _, _ = orc.execute(per[0][0], [p[1] for p in per], [p[2] for p in per], [p[3] for p in per])
        for r in range(world):
            assert_bf16_close(res[r]['outs'][step], want[r], f'{case} step {step} rank {r}')
    for r in range(world):
        np.testing.assert_array_equal(res[r]['slots'], orc.ctl.slots)
        np.testing.assert_array_equal(res[r]['owner'], orc.ctl.owner)
        np.testing.assert_array_equal(res[r]['fetches'], orc.fetches_per_rank)
    assert res[0]['dispatch_bytes'] > 0


def _gather_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from ferry_b200.metadata import RouteGather
    torch.cuda.set_device(rank)
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    res = {}
    for score in ('frequency', 'probability'):
        rg = RouteGather(8, 128, 128, score)
        for step, tokens in enumerate((64, 64, 5, 64)):  # parity halves alternate; sizes change
            g = torch.Generator().manual_seed(1000 * step + rank)
            sel = torch.stack([torch.randperm(128, generator=g)[:8] for _ in range(tokens)])
            probs = torch.softmax(torch.randn(tokens, 128, generator=g), -1)
            res[(score, step)] = rg.collect(sel.cuda(), probs.cuda())
        rg.close()
    torch.save(res, os.path.join(out_dir, f'g{rank}.pt'))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize('world', WORLDS)
def test_multi_gpu_route_gather_p2p(world):
    """RouteGather.collect over P2P stores into the peers' symmetric buffers:
    every rank receives the reference's gathered view (ids rank-major,
    origins, history rows of each rank's last tail tokens)."""
    _need(world)
    from oracle import metadata as om
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_gather_worker, args=(world, 29760 + world, tmp), nprocs=world)
        res = [torch.load(os.path.join(tmp, f'g{r}.pt'), weights_only=False) for r in range(world)]
    for score in ('frequency', 'probability'):
        for step, tokens in enumerate((64, 64, 5, 64)):
            sels, probs = [], []
            for r in range(world):
                g = torch.Generator().manual_seed(1000 * step + r)
                sels.append(torch.stack([torch.randperm(128, generator=g)[:8] for _ in range(tokens)]).numpy())
                probs.append(torch.softmax(torch.randn(tokens, 128, generator=g), -1).numpy())
            ids, origins = om.gather_ids(sels)
            tail = om.history_tail(tokens, 128, world)
            rows = (om.frequency_rows(ids, world, tokens, 128, 128) if score == 'frequency'
                    else om.probability_rows([p[-tail:] for p in probs]))
            for r in range(world):
                got_ids, got_origins, got_rows = res[r][(score, step)]
                np.testing.assert_array_equal(got_ids, ids)
                np.testing.assert_array_equal(got_origins, origins)
                np.testing.assert_array_equal(got_rows, rows)


def _fault_worker(rank, world, port, hook, out_dir):
    """Two ranks run one good layer, then a layer in which rank 1 leaves out
    its flag stores (`hook`); every wait on them is bounded at 0.3 s."""
    import torch.distributed as dist
    from datetime import timedelta
    from ferry_b200 import _lib
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import cpu_pool
    os.environ['NCCL_NVLS_ENABLE'] = '0'
    torch.cuda.set_device(rank)
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    shape, T, caps_of, _ = CASES['small']
    spec = _spec(shape)
    pool = cpu_pool(spec, spec.layers, 0).pin_memory()
    rt = OffloadRuntime(spec, pool, caps_of(world), 'ferry', Topology.uniform(world, spec.experts))
    res = {}
    layer, x, sel, w = _world_inputs(spec, 0, rank, T)
    good = rt.execute(layer, x.cuda(), sel.cuda(), w.cuda(), None)
    rt.check()
    res['good_finite'] = bool(torch.isfinite(good).all().item())
    rt.set_fault_hooks(T, hook if rank == 1 else 0, wait_ns=300_000_000)
    dist.barrier()  # both ranks leave the good layer before the faulty one starts
    layer, x, sel, w = _world_inputs(spec, 1, rank, T)
    bad = rt.execute(layer, x.cuda(), sel.cuda(), w.cuda(), None)
    try:
        rt.check()
        res['error'] = None
    except _lib.FerrybError as exc:
        res['error'] = str(exc)
    torch.cuda.synchronize()
    res['bad_all_nan'] = bool(torch.isnan(bad.float()).all().item())
    try:
        rt.close()
    except _lib.FerrybError:
        pass
    torch.save(res, os.path.join(out_dir, f'f{rank}.pt'))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize('hook', ['dispatch', 'combine'])
def test_two_gpu_missing_peer_flags_time_out(hook):
    """A rank that leaves out its dispatch (or combine) flag stores: the
    permute (or final-scatter) waits of both ranks run out after 0.3 s, each
    rank's check() raises FerrybError naming the layer, and each rank's output
    for that layer is NaN rather than a sum that silently misses the peer."""
    _need(2)
    from ferry_b200 import _lib
    bit = _lib.HOOK_NO_DISPATCH_SIGNAL if hook == 'dispatch' else _lib.HOOK_NO_COMBINE_SIGNAL
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_fault_worker, args=(2, 29790 + bit, bit, tmp), nprocs=2)
        res = [torch.load(os.path.join(tmp, f'f{r}.pt'), weights_only=False) for r in range(2)]
    for r in range(2):
        assert res[r]['good_finite'], f'rank {r}: the good layer is not finite'
        assert res[r]['error'] and 'MoE layer' in res[r]['error'] and 'peer' in res[r]['error'], res[r]
        assert res[r]['bad_all_nan'], f'rank {r}: the failed layer is not NaN'
