"""The routing-metadata and transport classes for callers composing the
reference's own flow (ferry_b200.metadata, ferry_b200.transport) against the
reference goldens (tests/golden, generated from ferry/metadata.py) and the
CPU oracle.  One GPU; the 4-rank all-gather is emulated as 4 symmetric
buffers on one GPU whose gather kernels all complete before any wait runs."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import expert_ops as ref_ops
from oracle import metadata as om
from tests.goldens import load
from tests.tolerance import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def test_gate_history_golden():
    from ferry_b200.metadata import GateHistory
    d = load('history')
    h = GateHistory(int(d['layers']), int(d['experts']), int(d['window']), device=DEV)
    for i in range(int(d['n'])):
        layer = int(d[f'c{i}_layer'])
        h.update(layer, d[f'c{i}_rows'])
        np.testing.assert_array_equal(h.scores(layer), d[f'c{i}_scores'], err_msg=f'case {i}')


@pytest.mark.parametrize('score', ['frequency', 'probability'])
def test_route_gather_world1(score):
    from ferry_b200.metadata import RouteGather
    g = torch.Generator().manual_seed(4)
    rg = RouteGather(6, 64, 128, score, device=DEV)
    for tokens in (16, 3, 200):
        sel = torch.stack([torch.randperm(64, generator=g)[:6] for _ in range(tokens)])
        probs = torch.softmax(torch.randn(tokens, 64, generator=g), -1)
        ids, origins, rows = rg.collect(sel.to(DEV), probs.to(DEV))
        want_ids, want_origins = om.gather_ids([sel.numpy()])
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(origins, want_origins)
        if score == 'frequency':
            want = om.frequency_rows(want_ids, 1, tokens, 128, 64)
        else:
            want = om.probability_rows([probs.numpy()[-om.history_tail(tokens, 128, 1):]])
        assert rows.dtype == want.dtype
        np.testing.assert_array_equal(rows, want)
    rg.close()


def test_symm_allgather_four_ranks_golden():
    """The P2P all-gather kernel over 4 buffers (ranks emulated on one GPU)
    reproduces the all_gather_into_tensor of the reference's RouteGather."""
    from ferry_b200 import _lib
    from ferry_b200.metadata import _device_bytes
    d = load('route_gather_frequency')
    world = int(d['world'])
    stream = _lib.stream_ptr(DEV)
    for step in range(4):
        sels = [d[f'r{r}_s{step}_sel'] for r in range(world)]
        tokens, topk = sels[0].shape
        stride = (tokens * topk + 15) // 16 * 16
        flags_at = world * stride
        nbytes = (flags_at + 8 * world + 255) // 256 * 256
        bufs = []
        for r in range(world):
            p = ctypes.c_void_p()
            _lib.call('ferryb_symm_alloc', nbytes, ctypes.byref(p), None)
            bufs.append(p.value)
        peers = torch.tensor(bufs, dtype=torch.int64, device=DEV)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        sends = []
        for r in range(world):
            send = torch.zeros(stride, dtype=torch.uint8, device=DEV)
            send[:tokens * topk].copy_(torch.as_tensor(sels[r].astype(np.uint8).reshape(-1)))
            sends.append(send)
            _lib.call('ferryb_symm_allgather', _lib.ptr(peers), world, r, 0, _lib.ptr(send), stride,
                      flags_at, ctypes.c_uint64(step + 1), stream)
        for r in range(world):
            _lib.call('ferryb_symm_wait', ctypes.c_void_p(bufs[r]), flags_at, world,
                      ctypes.c_uint64(step + 1), _lib.ptr(err), stream)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        for r in range(world):
            raw = _device_bytes(bufs[r], world * stride, DEV).cpu().numpy().reshape(world, stride)
            ids = raw[:, :tokens * topk].reshape(world * tokens, topk).astype(np.int64)
            np.testing.assert_array_equal(ids, d[f'r{r}_s{step}_ids'], err_msg=f'step {step} rank {r}')
        for b in bufs:
            _lib.call('ferryb_symm_free', ctypes.c_void_p(b))


def test_transport_world1_matches_oracle():
    """Transport.dispatch/combine with the device layout on one rank: every
    packet stays local, so dispatch = unpack(pack()) and combine =
    scatter(reduce()) of the oracle's expert_ops."""
    from ferry_b200.layout import device_layout
    from ferry_b200.transport import Transport
    g = torch.Generator().manual_seed(9)
    T, H, K, E = 24, 256, 4, 16
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g).to(torch.bfloat16)
    dest = np.zeros((T, K), np.int64)
    layout = device_layout(sel.numpy(), dest, T, 0, E, np.arange(E))
    tr = Transport(None, K, E)
    xr, wr = tr.dispatch(x.to(DEV), sel.to(DEV), w.to(DEV), layout)
    payload = ref_ops.pack_dispatch(x, sel, w, layout['send_idx'].cpu(), layout['send_ids'].cpu(), E)
    want_x, want_w = ref_ops.unpack_dispatch(payload, H, K)
    assert torch.equal(xr.cpu(), want_x) and torch.equal(wr.cpu(), want_w)
    parts = [(torch.randn(len(grp[1]), H, generator=g) * 0.1).to(torch.bfloat16) for grp in layout['groups']]
    out = tr.combine(x.to(DEV), [p.to(DEV) for p in parts], layout)
    partial = ref_ops.reduce_partials(parts, [grp[1].cpu() for grp in layout['groups']], xr.shape[0], H)
    want = ref_ops.scatter_returned(partial, layout['send_idx'].cpu(), T)
    assert_bf16_close(out.cpu(), want, 'combine')
    assert tr.dispatch_bytes == 0 and tr.combine_bytes == 0
