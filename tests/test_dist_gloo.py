"""Multi-process CPU tests of the N > 1 path over gloo (no GPU).

The benchmark's config 0: a DeepSeek-V2-Lite-shaped MoE layer (hidden 2048, 64
experts top-6, intermediate 1408) run by 4 gloo ranks with 16 tokens each for
8 consecutive steps, through the reference's distributed flow restated in
oracle/dist_layer.py; every rank's output must match what the single-process
emulation (oracle/layer.py) computes for that rank within the BF16 tolerance
(CPU GEMM rounding depends on the thread count), and every rank must reach
identical cache decisions.  A world-size-2 run checks the same at a smaller
shape, plus the symmetric-buffer handle exchange of ferry_b200.symm.
"""
import os
import tempfile

import numpy as np
import torch
import torch.multiprocessing as mp

from oracle import expert_ops as ops
from oracle import planner as op
from oracle.layer import OracleRuntime
from tests.tolerance import assert_bf16_close


class _Spec:
    def __init__(self, layers, experts, topk, hidden, inter):
        self.layers, self.experts, self.topk = layers, experts, topk
        self.hidden, self.intermediate = hidden, inter
        self.expert_elements = 3 * hidden * inter


def _setup(spec, seed, world):
    g = torch.Generator().manual_seed(seed)
    pool = (torch.randn(spec.layers * spec.experts, spec.expert_elements, generator=g) * 0.02).to(torch.bfloat16)
    gates = [(torch.randn(spec.experts, spec.hidden, generator=g) * 0.02).to(torch.bfloat16)
             for _ in range(spec.layers)]
    from ferry_b200.workload import zipf_bias
    biases = [zipf_bias(spec.experts, 1.1, g) for _ in range(spec.layers)]
    return pool, gates, biases


def _inputs(spec, step, rank, T, gates, biases):
    g = torch.Generator().manual_seed(1000 * step + rank)
    x = torch.randn(T, spec.hidden, generator=g).to(torch.bfloat16)
    layer = step % spec.layers
    sel, w, _ = ops.route_deepseek(x, gates[layer].float(), spec.topk, 1.0, biases[layer])
    return layer, x, sel, w


def _worker(rank, world, port, shape, caps, steps, T, out_dir):
    import torch.distributed as dist
    from oracle.dist_layer import DistOracleRuntime
    torch.set_num_threads(2)
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    spec = _Spec(*shape)
    pool, gates, biases = _setup(spec, 0, world)
    masks = np.asarray([1 << r for r in range(world)], np.int64)
    lut = op.build_lut(spec.experts, world, masks, np.ones(world))
    rt = DistOracleRuntime(spec, pool, caps, 'ferry', masks, np.ones(world), lut)
    outs = []
    for step in range(steps):
        layer, x, sel, w = _inputs(spec, step, rank, T, gates, biases)
        y, _ = rt.execute(layer, x, sel, w)
        outs.append(y)
    torch.save({'outs': outs, 'slots': rt.ctl.slots, 'owner': rt.ctl.owner},
               os.path.join(out_dir, f'rank{rank}.pt'))
    dist.barrier()
    dist.destroy_process_group()


def _run(world, shape, caps, steps, T, port):
    spec = _Spec(*shape)
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_worker, args=(world, port, shape, caps, steps, T, tmp), nprocs=world)
        res = [torch.load(os.path.join(tmp, f'rank{r}.pt'), weights_only=False) for r in range(world)]
    pool, gates, biases = _setup(spec, 0, world)
    masks = np.asarray([1 << r for r in range(world)], np.int64)
    lut = op.build_lut(spec.experts, world, masks, np.ones(world))
    orc = OracleRuntime(spec, pool, caps, 'ferry', masks, np.ones(world), lut)
    for step in range(steps):
        per = [_inputs(spec, step, r, T, gates, biases) for r in range(world)]
        want, _, _ = orc.execute(per[0][0], [p[1] for p in per], [p[2] for p in per], [p[3] for p in per])
        for r in range(world):  # CPU GEMMs differ in rounding with the thread count
            assert_bf16_close(res[r]['outs'][step], want[r], f'step {step} rank {r}')
    for r in range(world):
        np.testing.assert_array_equal(res[r]['slots'], orc.ctl.slots)
        np.testing.assert_array_equal(res[r]['owner'], orc.ctl.owner)


def test_config0_world4_gloo():
    """The benchmark's config 0: DSV2-Lite layer, 4 gloo ranks x 16 tokens, 8 steps,
    global 30 % cache of a 2-layer slice (38 slots -> 10/10/9/9)."""
    _run(4, (2, 64, 6, 2048, 1408), [10, 10, 9, 9], 8, 16, 29651)


def test_world2_gloo_small():
    _run(2, (2, 16, 4, 128, 64), [6, 5], 6, 8, 29652)


def _symm_worker(rank, world, port, out_dir):
    """The IPC-handle exchange of ferry_b200.symm over gloo, with the CUDA
    calls replaced by stand-ins (no GPU here)."""
    import ctypes
    import torch.distributed as dist
    from ferry_b200 import symm
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    opened = []

    def fake_call(name, *args):
        if name == 'ferryb_symm_alloc':
            args[1]._obj.value = 0x1000 * (rank + 1)
            if args[2] is not None:
                for i in range(64):
                    args[2][i] = (rank * 7 + i) & 0xff
        elif name == 'ferryb_symm_open':
            handle = bytes(args[0])
            args[1]._obj.value = 0x100000 + handle[0]
            opened.append(handle[0])
        return 0

    symm.call = fake_call
    buf = symm.SymmetricBuffer(4096, rank, world)
    bases = list(buf.bases)
    buf._opened = []
    buf.local = None
    torch.save({'bases': bases, 'opened': opened}, os.path.join(out_dir, f's{rank}.pt'))
    dist.barrier()
    dist.destroy_process_group()


def test_symmetric_handle_exchange_world2():
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_symm_worker, args=(2, 29653, tmp), nprocs=2)
        res = [torch.load(os.path.join(tmp, f's{r}.pt')) for r in range(2)]
    # rank r keeps its own address and maps the peer's handle (first byte = peer * 7)
    assert res[0]['bases'][0] == 0x1000 and res[1]['bases'][1] == 0x2000
    assert res[0]['opened'] == [7] and res[1]['opened'] == [0]
    assert res[0]['bases'][1] == 0x100000 + 7 and res[1]['bases'][0] == 0x100000


def _pool_worker(rank, world, port, out_dir):
    """SharedPinnedPool over gloo with cudaHostRegister replaced (no GPU here):
    every rank maps the same pages the first rank filled."""
    import torch.distributed as dist
    from ferry_b200 import pool as pool_mod
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    pool_mod.SharedPinnedPool._register = lambda self: None

    def fill(t):
        t.copy_(torch.arange(t.numel(), dtype=torch.float32).reshape(t.shape).to(torch.bfloat16))

    sp = pool_mod.SharedPinnedPool(6, 40, fill=fill)
    first = sp.tensor.clone()
    dist.barrier()
    if rank == world - 1:
        sp.tensor[5, 39] = 7.0  # a write by one rank is seen by all
    dist.barrier()
    torch.save({'first': first, 'after': sp.tensor.clone()}, os.path.join(out_dir, f'p{rank}.pt'))
    dist.barrier()
    sp.close()
    dist.destroy_process_group()


def test_shared_pinned_pool_world3():
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_pool_worker, args=(3, 29654, tmp), nprocs=3)
        res = [torch.load(os.path.join(tmp, f'p{r}.pt')) for r in range(3)]
    want = torch.arange(240, dtype=torch.float32).reshape(6, 40).to(torch.bfloat16)
    for r in range(3):
        assert torch.equal(res[r]['first'], want)
        assert float(res[r]['after'][5, 39]) == 7.0


def _transport_worker(rank, world, port, out_dir):
    """ferry_b200.transport.Transport over gloo with the oracle's CPU ops
    standing in for the kernels: with identity experts, dispatch then combine
    returns each token times its number of routes."""
    import torch.distributed as dist
    from ferry_b200.transport import Transport
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    T, H, K, E = 12, 64, 4, 16
    g = torch.Generator().manual_seed(77)
    sels, xs = [], []
    for r in range(world):
        sels.append(torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]))
        xs.append((torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16))
    ids = torch.cat(sels).numpy()
    owner = np.arange(E) % world
    dest = owner[ids]
    send_idx, send_ids, send_counts, recv_counts, starts, rows, cols = op.build_layout(ids, dest, T, rank, E)
    groups = [(int(e), torch.from_numpy(rows[starts[e]:starts[e + 1]]), torch.from_numpy(cols[starts[e]:starts[e + 1]]), 0)
              for e in np.flatnonzero(starts[1:] > starts[:-1])]
    layout = dict(send_idx=torch.from_numpy(send_idx), send_ids=torch.from_numpy(send_ids),
                  send_counts=send_counts.tolist(), recv_counts=recv_counts.tolist(), groups=groups)
    class _CpuOps:  # the oracle's ops under the reference's signatures (expert_ops.cpp:144-157)
        pack_dispatch = staticmethod(ops.pack_dispatch)
        unpack_dispatch = staticmethod(ops.unpack_dispatch)
        scatter_returned = staticmethod(ops.scatter_returned)

        @staticmethod
        def reduce_partials(parts, rows, received, hidden, like):
            return ops.reduce_partials(parts, rows, received, hidden)
    tr = Transport(_CpuOps, K, E)
    w = torch.ones(T, K).to(torch.bfloat16)
    xr, wr = tr.dispatch(xs[rank], sels[rank], w, layout)
    parts = [xr.index_select(0, grp[1]) for grp in groups]  # identity experts
    out = tr.combine(xs[rank], parts, layout)
    torch.save({'out': out, 'x': xs[rank], 'db': tr.dispatch_bytes, 'cb': tr.combine_bytes,
                'send': send_counts, 'recv': recv_counts}, os.path.join(out_dir, f't{rank}.pt'))
    dist.barrier()
    dist.destroy_process_group()


def test_transport_compat_world2_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_transport_worker, args=(2, 29655, tmp), nprocs=2)
        res = [torch.load(os.path.join(tmp, f't{r}.pt'), weights_only=False) for r in range(2)]
    K, H = 4, 64
    for r, d in enumerate(res):
        assert_bf16_close(d['out'], (d['x'].float() * K).to(torch.bfloat16), f'rank {r}')
        send, recv = d['send'], d['recv']
        assert d['db'] == (int(send.sum()) - int(send[r])) * (2 * H + 3 * K)
        assert d['cb'] == (int(recv.sum()) - int(recv[r])) * H * 2


def _topology_worker(rank, world, port, out_dir):
    """topology_for_run('auto') over gloo ranks with the GPU copy profile
    replaced by a stand-in that reports fixed per-subset bandwidths."""
    import json
    import torch.distributed as dist
    from ferry_b200 import profile_h2d, quota
    from ferry_b200.build_quota_lut import topology_for_run
    from ferry_b200.model import QWEN3_30B_A3B, spec_from_config
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    quota.build_lut = lambda *a: op.build_lut(*a)

    def fake_profile(rank_, world_, target, source, copies=16, repeats=2, group=None):
        import itertools
        doms = []
        for n in range(1, world_ + 1):
            for s in itertools.combinations(range(world_), n):
                per = [50.0 / (1 + 0.5 * (len(s) - 1))] * len(s)  # links shared as more ranks copy
                doms.append(dict(gpus=list(s), mask=sum(1 << g for g in s), gib_per_s=sum(per),
                                 per_gpu_gib_per_s=per))
        return doms
    profile_h2d.profile_ranks = fake_profile
    spec = spec_from_config(QWEN3_30B_A3B)
    topo, note = topology_for_run('auto', spec, rank, world, pool_row=torch.zeros(16, dtype=torch.bfloat16))
    with open(os.path.join(out_dir, f'{rank}.json'), 'w') as f:
        json.dump(dict(masks=topo.masks.tolist(), lut=topo.lut.tolist(), note=note), f)
    dist.destroy_process_group()


def test_auto_topology_world3_gloo():
    """Every rank gets rank 0's table, over all 7 rank subsets, and it is the
    oracle's build_lut of that profile."""
    import json
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_topology_worker, args=(3, 29656, tmp), nprocs=3)
        res = [json.load(open(os.path.join(tmp, f'{r}.json'))) for r in range(3)]
    assert res[0] == res[1] == res[2]
    masks = res[0]['masks']
    assert masks == [1, 2, 4, 3, 5, 6, 7] and res[0]['note'].startswith('auto: profiled 7 rank subsets')
    gib = [50.0 / (1 + 0.5 * (bin(m).count('1') - 1)) * bin(m).count('1') for m in masks]
    want = op.build_lut(128, 3, np.asarray(masks, np.int64), np.asarray([1.0 / g for g in gib]))
    assert np.array_equal(np.asarray(res[0]['lut']), want)
