"""Argument checks of the Python entry points, with no GPU.

The C ABI receives bare pointers, so every buffer length a kernel relies on is
checked on the host before the call (the reference's TORCH_CHECKs,
ferry/csrc/expert_ops.cpp:20-34, plus the lengths its numba loops assume,
ferry/policy.py:25-127).  Here the CUDA-facing helpers are replaced by
recorders: valid arguments must reach the library call unchanged, invalid ones
must raise FerrybError (a RuntimeError) before it.
"""
import numpy as np
import pytest
import torch

from ferry_b200 import _lib, expert_ops, layout, policy, runtime
from ferry_b200._lib import FerrybError, check_tensor
from ferry_b200.model import ModelSpec

BF16 = torch.bfloat16


@pytest.fixture
def calls(monkeypatch):
    """Replace the library calls and stream lookups with a recorder."""
    seen = []

    def record(name, *args):
        seen.append(name)
        return 0
    for mod in (expert_ops, policy):
        monkeypatch.setattr(mod, 'call', record)
        monkeypatch.setattr(mod, 'stream_ptr', lambda *a: None)
    monkeypatch.setattr(expert_ops, 'require_cuda', lambda *t: None)
    monkeypatch.setattr(policy, '_dev', lambda device=None: torch.device('cpu'))
    return seen


def test_check_tensor():
    t = torch.zeros(4, 3, dtype=BF16)
    check_tensor(t, 't', (4, None), BF16, contiguous=True)
    for shape, dtype in (((4,), None), ((3, 3), None), ((4, 3), torch.float32)):
        with pytest.raises(FerrybError):
            check_tensor(t, 't', shape, dtype)
    with pytest.raises(FerrybError, match='contiguous'):
        check_tensor(t.t(), 't', (3, 4), contiguous=True)
    with pytest.raises(FerrybError, match='required'):
        check_tensor(None, 't', (1,))
    assert issubclass(FerrybError, RuntimeError)


def test_pack_unpack_checks(calls):
    T, H, K, E, n = 6, 16, 4, 8, 5
    hid = torch.zeros(T, H, dtype=BF16)
    sel = torch.zeros(T, K, dtype=torch.int64)
    w = torch.zeros(T, K, dtype=BF16)
    idx, ids = torch.zeros(n, dtype=torch.int64), torch.zeros(n, K, dtype=torch.int64)
    payload = expert_ops.pack_dispatch(hid, sel, w, idx, ids, E)
    assert payload.shape == (n, 2 * H + 3 * K) and calls == ['ferryb_pack_dispatch']
    bad = [(hid, sel[:, :2], w, idx, ids), (hid, sel, w[:, :2], idx, ids), (hid[:3], sel, w, idx, ids),
           (hid, sel, w, idx, ids[:2]), (hid, sel, w.float(), idx, ids)]
    for args in bad:
        with pytest.raises(FerrybError):
            expert_ops.pack_dispatch(*args, E)
    x, wr = expert_ops.unpack_dispatch(payload, H, K)
    assert x.shape == (n, H) and wr.shape == (n, K)
    for raw in (payload[:, :-1], payload.view(torch.int8), payload.reshape(-1)):
        with pytest.raises(FerrybError):
            expert_ops.unpack_dispatch(raw, H, K)
    assert calls == ['ferryb_pack_dispatch', 'ferryb_unpack_dispatch']


def test_reduce_scatter_checks(calls):
    H = 16
    like = torch.zeros(4, H, dtype=BF16)
    parts = [torch.zeros(3, H, dtype=BF16), torch.zeros(2, H, dtype=BF16)]
    rows = [torch.tensor([0, 1, 2]), torch.tensor([1, 3])]
    out = expert_ops.reduce_partials(parts, rows, 4, H, like)
    assert out.shape == (4, H) and calls == ['ferryb_reduce_partials']
    for p, r in (([parts[0]], rows), ([parts[0][:, :8], parts[1]], rows),
                 ([parts[0], parts[1][:1]], rows)):
        with pytest.raises(FerrybError):
            expert_ops.reduce_partials(p, r, 4, H, like)
    ret = torch.zeros(5, H, dtype=BF16)
    out = expert_ops.scatter_returned(ret, torch.zeros(5, dtype=torch.int64), 3)
    assert out.shape == (3, H) and calls[-1] == 'ferryb_scatter_returned'
    with pytest.raises(FerrybError):
        expert_ops.scatter_returned(ret, torch.zeros(4, dtype=torch.int64), 3)


def test_policy_step_checks(calls):
    E, R, L = 8, 2, 3
    sel = np.zeros((6, 2), np.int64)
    policy._demand(sel, np.zeros(6, np.int64), E, R)
    with pytest.raises(FerrybError):
        policy._demand(sel, np.zeros(5, np.int64), E, R)

    slots = np.full((R, 4), -1, np.int64)
    policy._admission_capacity(slots, [4, 3], 1, np.zeros(E, np.uint8), E)
    for s, caps, act in ((slots, [5, 3], np.zeros(E)), (slots[:1], [4, 3], np.zeros(E)),
                         (slots, [4, 3], np.zeros(E - 1))):
        with pytest.raises(FerrybError):
            policy._admission_capacity(s, caps, 1, act, E)

    demand = np.zeros((E, R), np.int64)
    owner = np.full(L * E, -1, np.int64)
    policy.load_balanced_assignment(demand, [1, 2], owner, 2, np.array([1, 1]), 200)
    for misses, own, quota in (([1, E], owner, [1, 1]), ([1], owner[:2 * E], [1, 1]),
                               ([1], owner, [1, 1, 1])):
        with pytest.raises(FerrybError):
            policy.load_balanced_assignment(demand, misses, own, 2, np.array(quota), 200)

    last, scores = np.zeros(L * E, np.int64), np.zeros((L, E), np.float32)
    slots[0, :2] = [3, L * E - 1]
    policy._choose_slot(0, 1, np.zeros(E), slots, [4, 3], last, scores, E)
    bad_slots = slots.copy()
    bad_slots[0, 1] = L * E
    for args in ((2, slots, last), (0, bad_slots, last), (0, slots, last[:-1])):
        with pytest.raises(FerrybError):
            policy._choose_slot(args[0], 1, np.zeros(E), args[1], [4, 3], args[2], scores, E)

    policy.layer_slots(np.zeros(4, np.int64), 4, 0, E)
    with pytest.raises(FerrybError):
        policy.layer_slots(np.zeros(3, np.int64), 4, 0, E)
    assert calls.count('ferryb_choose_slot') == 1 and calls.count('ferryb_layer_slots') == 1


def test_layout_shape_checks():
    layout._check_shapes((8, 2), (8, 2), 4)
    for sel, dest, n in (((8, 2), (8, 3), 4), ((8, 2), (8, 2), 3), ((8,), (8,), 4), ((8, 2), (8, 2), 0)):
        with pytest.raises(FerrybError):
            layout._check_shapes(sel, dest, n)


def _cpu_runtime(spec, score='frequency'):
    """An OffloadRuntime shell with only the fields its input checks read."""
    rt = runtime.OffloadRuntime.__new__(runtime.OffloadRuntime)
    rt.spec, rt.device, rt.eviction_score = spec, torch.device('cpu'), score
    return rt


class _Reached(Exception):
    pass


def test_runtime_input_checks(monkeypatch):
    spec = ModelSpec('qwen3_moe', (0, 1), 8, 2, 16, 8)
    rt = _cpu_runtime(spec, 'probability')

    def reached(tokens):
        raise _Reached(tokens)
    monkeypatch.setattr(rt, '_executor', reached, raising=False)
    T = 5
    x = torch.zeros(T, 16, dtype=BF16)
    sel, w = torch.zeros(T, 2, dtype=torch.int64), torch.zeros(T, 2, dtype=torch.float32)
    pt = torch.zeros(3, 8)
    with pytest.raises(_Reached):
        rt.execute(0, x, sel, w, pt)
    for args in ((x.float(), sel, w, pt), (x[:, :8], sel, w, pt), (x, sel[:, :1], w, pt),
                 (x, sel, w[:4], pt), (x, sel, w, pt[:, :4])):
        with pytest.raises(FerrybError):
            rt.execute(0, *args)
    gate, bias = torch.zeros(8, 16, dtype=BF16), torch.zeros(8)
    s_out, w_out = torch.zeros(T, 2, dtype=torch.int64), torch.zeros(T, 2, dtype=BF16)
    with pytest.raises(_Reached):
        rt.forward(0, x, gate, bias, s_out, w_out)
    with pytest.raises(_Reached):
        rt.forward(0, x.t().contiguous().t(), gate, None)  # a strided hidden is made contiguous
    for args in ((x, gate.float(), bias), (x, gate[:4], bias), (x, gate, bias.to(BF16)),
                 (x, gate, bias, s_out[:, :1]), (x, gate, bias, s_out, w_out.float()),
                 (x, gate.t().contiguous().t(), bias)):
        with pytest.raises(FerrybError):
            rt.forward(0, *args)


def test_runtime_rejects_other_device(monkeypatch):
    spec = ModelSpec('qwen3_moe', (0,), 8, 2, 16, 8)
    rt = _cpu_runtime(spec)
    rt.device = torch.device('cuda', 0)  # tensors below live on the CPU
    with pytest.raises(FerrybError, match='is on cpu'):
        rt.execute(0, torch.zeros(2, 16, dtype=BF16), torch.zeros(2, 2, dtype=torch.int64),
                   torch.zeros(2, 2, dtype=BF16), None)


def test_errors_carry_library_message():
    lib = _lib.lib()
    cfg = _lib.LayerConfig()  # all zero: rejected by the size query
    assert lib.ferryb_layer_workspace_bytes(cfg) < 0
    assert lib.ferryb_last_error()


def test_golden_inputs_pass_the_checks(calls):
    """Every argument set the GPU parity tests take from the reference's
    goldens gets through the checks to the library call."""
    from oracle import planner as op
    from tests.goldens import PLAN_CASES, PlanCase, load
    d = load('assignment')
    for i in range(int(d['n'])):
        policy.load_balanced_assignment(d[f'c{i}_demand'], d[f'c{i}_misses'], d[f'c{i}_owner'],
                                        int(d[f'c{i}_layer']), d[f'c{i}_quota'], int(d[f'c{i}_bps']))
    d = load('choose_slot')
    for i in range(int(d['n'])):
        policy._choose_slot(int(d[f'c{i}_rank']), int(d[f'c{i}_layer']), d[f'c{i}_active'],
                            d[f'c{i}_slots'], d[f'c{i}_caps'], d[f'c{i}_last'], d[f'c{i}_scores'],
                            int(d[f'c{i}_experts']))
    assert calls.count('ferryb_choose_slot') == int(d['n'])
    from ferry_b200.quota import Topology
    for name in PLAN_CASES:
        c = PlanCase(name)
        ctl = policy.Controller(policy._Spec(c.layers, c.experts, c.topk), c.caps, c.policy,
                                Topology.from_arrays(c.masks, c.seconds, c.lut), c.bps, c.salt,
                                window=c.window)
        s = c.step(0)
        ctl.plan(s['event'], s['layer'], s['selected'], c.origins(), s['scores'])
        policy._demand(s['selected'], c.origins(), c.experts, c.world)
        active = op.demand(s['selected'], c.origins(), c.experts, c.world).sum(1) > 0
        slots = np.full((c.world, int(max(c.caps))), -1, np.int64)
        policy._admission_capacity(slots, c.caps, s['layer'], active, c.experts)
        for r in range(c.world):
            policy.layer_slots(slots[r], c.caps[r], s['layer'], c.experts)
            layout._check_shapes(s['selected'].shape, s['selected'].shape, c.tokens)
    assert calls.count('ferryb_plan_layer') == len(PLAN_CASES)
