"""The packet, reduction and copy ops against the reference's own compiled
extension (oracle/_ref, built from ferry/csrc/expert_ops.{cpp,cu}) on the
same GPU and the same inputs:

* pack_dispatch / unpack_dispatch (ferry/csrc/expert_ops.cpp:50-73):
  bit-exact, at packet strides 2H + 3k of every alignment;
* reduce_partials / scatter_returned (:76-92): the reference sums in float32
  with index_add_, one kernel per group and atomics inside a kernel.  Where
  every destination row receives at most one value per kernel (the executor's
  layouts: an expert sees a packet once; or at most two values, which any
  order adds alike) the result is bit-exact; with three or more values per
  row in one kernel the reference's own order is not fixed, and the results
  agree within one bf16 rounding step;
* H2DEngine (:97-142): the same cache bytes and copy counts after fetch /
  wait_host, and a copy into a slot waits for the compute marked with
  mark_used.

The oracle's CPU restatement (oracle/expert_ops.py, the checker of the fused
executor) is pinned to the reference here as well.  Skipped where
oracle/_ref was not built."""
import numpy as np
import pytest
import torch

from oracle import expert_ops as orc_ops
from oracle.build_ref import load_ref

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


@pytest.fixture(scope='module')
def ref():
    mod = load_ref()
    if mod is None:
        pytest.skip('reference extension not built (oracle/build_ref.py)')
    return mod


def _packets(T, H, K, E, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g).to(torch.bfloat16)
    idx = torch.randperm(T, generator=g)[:max(1, T // 2)].sort().values
    ids = torch.full((idx.numel(), K), -1, dtype=torch.int64)
    for i, t in enumerate(idx.tolist()):
        keep = sel[t][torch.randperm(K, generator=g)[:1 + i % K]].sort().values
        ids[i, :keep.numel()] = keep
    return x, sel, w, idx, ids


@pytest.mark.parametrize('H,K,E', [(2048, 8, 128), (2048, 6, 64), (256, 4, 16), (256, 3, 16)])
def test_pack_unpack_match_reference(ref, H, K, E):
    from ferry_b200 import expert_ops as ops
    x, sel, w, idx, ids = _packets(48, H, K, E, seed=3 * H + K)
    args = (x.to(DEV), sel.to(DEV), w.to(DEV), idx.to(DEV), ids.to(DEV), E)
    want = ref.pack_dispatch(*args)
    got = ops.pack_dispatch(*args)
    assert got.shape == want.shape and torch.equal(got, want)
    assert torch.equal(orc_ops.pack_dispatch(x, sel, w, idx, ids, E), want.cpu())
    wx, ww = ref.unpack_dispatch(want, H, K)
    gx, gw = ops.unpack_dispatch(got, H, K)
    assert torch.equal(gx, wx) and torch.equal(gw, ww)
    ox, ow = orc_ops.unpack_dispatch(want.cpu(), H, K)
    assert torch.equal(ox, wx.cpu()) and torch.equal(ow, ww.cpu())


def _layout_groups(received, n_groups, H, seed):
    """Groups as an executor layout makes them: each group's rows distinct."""
    g = torch.Generator().manual_seed(seed)
    parts, rows = [], []
    for i in range(n_groups):
        n = int(torch.randint(1, max(2, received), (1,), generator=g))
        rows.append(torch.randperm(received, generator=g)[:n].sort().values)
        parts.append((torch.randn(n, H, generator=g) * 0.1).to(torch.bfloat16))
    return parts, rows


@pytest.mark.parametrize('received,groups,H', [(64, 45, 2048), (37, 8, 2048), (5, 3, 256)])
def test_reduce_partials_matches_reference(ref, received, groups, H):
    from ferry_b200 import expert_ops as ops
    parts, rows = _layout_groups(received, groups, H, seed=received + groups)
    like = torch.empty(1, H, dtype=torch.bfloat16, device=DEV)
    dparts, drows = [p.to(DEV) for p in parts], [r.to(DEV) for r in rows]
    want = ref.reduce_partials(dparts, drows, received, H, like)
    got = ops.reduce_partials(dparts, drows, received, H, like)
    assert torch.equal(got, want)
    assert torch.equal(orc_ops.reduce_partials(parts, rows, received, H), want.cpu())


def _ulp_close(got, want):
    """|got - want| <= one bf16 rounding step of max(|got|, |want|) per element."""
    g, w = got.float().cpu(), want.float().cpu()
    step = torch.maximum(g.abs(), w.abs()) * 2.0 ** -7 + 1e-30
    return bool(((g - w).abs() <= step).all())


def test_reduce_partials_repeated_rows(ref):
    """Rows repeated inside one group: the reference's atomics have no fixed
    order, so the sums agree within one bf16 rounding step."""
    from ferry_b200 import expert_ops as ops
    g = torch.Generator().manual_seed(5)
    received, H = 16, 256
    rows = [torch.randint(0, received, (n,), generator=g) for n in (40, 3, 17)]
    parts = [torch.randn(r.numel(), H, generator=g).to(torch.bfloat16) for r in rows]
    like = torch.empty(1, H, dtype=torch.bfloat16, device=DEV)
    dparts, drows = [p.to(DEV) for p in parts], [r.to(DEV) for r in rows]
    want = ref.reduce_partials(dparts, drows, received, H, like)
    got = ops.reduce_partials(dparts, drows, received, H, like)
    assert _ulp_close(got, want)


@pytest.mark.parametrize('tokens,per_token,H', [(64, 2, 2048), (9, 1, 256), (32, 4, 2048)])
def test_scatter_returned_matches_reference(ref, tokens, per_token, H):
    """Each token receives `per_token` returned partials (one per peer it sent
    a packet to): bit-exact up to two per token, within one bf16 rounding step
    above (the reference's atomics add them in no fixed order)."""
    from ferry_b200 import expert_ops as ops
    g = torch.Generator().manual_seed(tokens * per_token)
    send_idx = torch.cat([torch.randperm(tokens, generator=g) for _ in range(per_token)])
    returned = (torch.randn(send_idx.numel(), H, generator=g) * 0.2).to(torch.bfloat16)
    want = ref.scatter_returned(returned.to(DEV), send_idx.to(DEV), tokens)
    got = ops.scatter_returned(returned.to(DEV), send_idx.to(DEV), tokens)
    orc = orc_ops.scatter_returned(returned, send_idx, tokens)
    if per_token <= 2:
        assert torch.equal(got, want) and torch.equal(orc, want.cpu())
    else:
        assert _ulp_close(got, want) and _ulp_close(orc, want)


def test_scatter_returned_empty(ref):
    from ferry_b200 import expert_ops as ops
    ret = torch.empty(0, 256, dtype=torch.bfloat16, device=DEV)
    idx = torch.empty(0, dtype=torch.int64, device=DEV)
    assert torch.equal(ops.scatter_returned(ret, idx, 7), ref.scatter_returned(ret, idx, 7))


def test_h2d_engine_matches_reference(ref):
    """fetch + wait_host fill the same cache bytes and count the same copies;
    a fetch into a slot that mark_used protects lands after the marked read."""
    from ferry_b200.expert_ops import H2DEngine
    g = torch.Generator().manual_seed(0)
    rows, width, slots = 12, 3 * 256 * 128, 6
    pool = torch.randn(rows, width, generator=g).to(torch.bfloat16).pin_memory()
    caches = [torch.zeros(slots, width, dtype=torch.bfloat16, device=DEV) for _ in range(2)]
    engines = [ref.H2DEngine(caches[0], pool), H2DEngine(caches[1], pool)]
    plan = [([0, 3, 5], [7, 2, 11]), ([1, 3], [4, 9]), ([0, 2, 4], [1, 0, 6])]
    for sl, keys in plan:
        for e in engines:
            e.fetch(sl, keys)
            e.wait_host(sl)
        assert torch.equal(caches[0], caches[1])
    assert engines[0].copies == engines[1].copies == sum(len(s) for s, _ in plan)
    # last-use ordering: a read of slot 2 queued behind ~ms of other work on
    # the compute stream, marked with mark_used, then a fetch into slot 2: the
    # read must still see the old row
    for cache, e in zip(caches, engines):
        torch.cuda.synchronize()
        old = cache[2].clone()
        a = torch.randn(4096, 4096, device=DEV)
        b = torch.empty_like(a)
        for _ in range(20):
            torch.mm(a, a, out=b)
            a, b = b, a
        snap = cache[2].clone()
        e.mark_used([2])
        e.fetch([2], [10])
        e.synchronize()
        torch.cuda.synchronize()
        assert torch.equal(snap, old)
        assert torch.equal(cache[2].cpu(), pool[10])
    engines[1].close()


def test_transport_world1_matches_reference_composition(ref):
    """Transport.dispatch/combine (one rank) against the reference's ops
    composed as ferry/transport.py composes them."""
    from ferry_b200.layout import device_layout
    from ferry_b200.transport import Transport
    g = torch.Generator().manual_seed(21)
    T, H, K, E = 64, 2048, 8, 128
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    sel = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g).to(torch.bfloat16).to(DEV)
    dest = np.zeros((T, K), np.int64)
    layout = device_layout(sel.numpy(), dest, T, 0, E, np.arange(E))
    tr = Transport(None, K, E)
    xr, wr = tr.dispatch(x, sel.to(DEV), w, layout)
    payload = ref.pack_dispatch(x, sel.to(DEV), w, layout['send_idx'], layout['send_ids'], E)
    want_x, want_w = ref.unpack_dispatch(payload, H, K)
    assert torch.equal(xr, want_x) and torch.equal(wr, want_w)
    parts = [(torch.randn(len(grp[1]), H, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
             for grp in layout['groups']]
    out = tr.combine(x, parts, layout)
    partial = ref.reduce_partials(parts, [grp[1] for grp in layout['groups']], xr.shape[0], H, x)
    want = ref.scatter_returned(partial, layout['send_idx'], T)
    assert torch.equal(out, want)


def _ref_runtime_worker(rank, world, port, out_dir):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from ferry_b200.model import ModelSpec
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import cpu_pool, zipf_bias
    from oracle.ref_runtime import RefGpuRuntime
    os.environ['NCCL_NVLS_ENABLE'] = '0'
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, device_id=torch.device('cuda', rank),
                            timeout=timedelta(seconds=60))
    spec = ModelSpec('qwen3_moe', (0, 1), 64, 8, 2048, 768)
    caps = [100]
    pool = cpu_pool(spec, spec.layers, 0).pin_memory()
    topo = Topology.uniform(1, spec.experts)
    ref = RefGpuRuntime(spec, pool, caps, 'ferry', topo.masks, topo.seconds, topo.lut)
    rt = OffloadRuntime(spec, pool, caps, 'ferry', topo)
    g = torch.Generator().manual_seed(3)
    gates = [(torch.randn(spec.experts, spec.hidden, generator=g) * 0.02).to(torch.bfloat16).cuda()
             for _ in range(2)]
    biases = [zipf_bias(spec.experts, 1.1, g).cuda() for _ in range(2)]
    errs, same = [], True
    for step in range(6):
        layer = step % 2
        x = torch.randn(32, spec.hidden, generator=g).to(torch.bfloat16).cuda()
        sel, w = ref.route(x, gates[layer], biases[layer])
        want = ref.execute(layer, x, sel, w)
        got = rt.execute(layer, x, sel, w, None)
        torch.cuda.synchronize()
        errs.append(((got.float() - want.float()).abs().max().item(), want.float().abs().max().item()))
        same = same and np.array_equal(rt.controller.slots, ref.ctl.slots)
    rt.close()
    ref.close()
    torch.save({'errs': errs, 'same': same, 'copies': (ref.h2d.copies, rt.h2d.copies)},
               os.path.join(out_dir, 'ref.pt'))
    dist.destroy_process_group()


def test_reference_runtime_composition_matches(ref):
    """The composed reference runtime (oracle/ref_runtime.py, the comparator of
    bench.py --impl reference-gpu) against this runtime on the same routed
    layers (one rank, NCCL collectives of one rank): the same cache decisions
    and copy counts, outputs within the BF16 tolerance."""
    import os
    import tempfile

    import torch.multiprocessing as mp
    from tests.tolerance import ABS_TOL, REL_TOL
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_ref_runtime_worker, args=(1, 29831, tmp), nprocs=1)
        res = torch.load(os.path.join(tmp, 'ref.pt'), weights_only=False)
    assert res['same'], 'cache decisions differ'
    assert res['copies'][0] == res['copies'][1]
    for err, scale in res['errs']:
        assert err <= ABS_TOL and err <= REL_TOL * scale, (err, scale)
