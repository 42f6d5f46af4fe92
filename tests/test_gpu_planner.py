"""Kernel 2 (device planner) and the device layout against the reference's
own outputs (tests/golden/, from the reference's numba code).  Bit-exact:
fetch lists, destinations, counts, cache state, gate scores, layouts."""
import numpy as np
import pytest
import torch

from oracle import planner as op
from tests.goldens import PLAN_CASES, PlanCase, load

pytestmark = pytest.mark.gpu


def _controller(c):
    from ferry_b200.policy import Controller, _Spec
    from ferry_b200.quota import Topology
    topo = Topology.from_arrays(c.masks, c.seconds, c.lut)
    score = 'probability' if c.step(0)['rows'].size else 'frequency'
    return Controller(_Spec(c.layers, c.experts, c.topk), c.caps, c.policy, topo, c.bps, c.salt,
                      window=c.window, score=score)


@pytest.mark.parametrize('name', PLAN_CASES)
def test_plan_with_host_scores(name):
    """Controller.plan(event, layer, selected, origins, gate_scores) as the reference calls it."""
    from ferry_b200.layout import build_layout
    from ferry_b200.policy import layer_slots
    c = PlanCase(name)
    ctl = _controller(c)
    for i in range(c.steps):
        s = c.step(i)
        if not s['ok']:
            with pytest.raises(AssertionError):
                ctl.plan(s['event'], s['layer'], s['selected'], c.origins(), s['scores'])
            break
        f, d, n = ctl.plan(s['event'], s['layer'], s['selected'], c.origins(), s['scores'])
        np.testing.assert_array_equal(f, s['fetches'], err_msg=f'{name} step {i} fetches')
        np.testing.assert_array_equal(d, s['dest'], err_msg=f'{name} step {i} destinations')
        np.testing.assert_array_equal(n, s['counts'], err_msg=f'{name} step {i} counts')
        if 'slots' in s:
            np.testing.assert_array_equal(ctl.slots, s['slots'], err_msg=f'{name} step {i} slots')
            np.testing.assert_array_equal(ctl.owner, s['owner'], err_msg=f'{name} step {i} owner')
            np.testing.assert_array_equal(ctl.last, s['last'], err_msg=f'{name} step {i} last')
        if i % 3 == 0 or i == c.steps - 1:  # layouts: every few steps keeps the test quick
            slots = ctl.slots
            for r in range(c.world):
                lay = build_layout(s['selected'], d, c.tokens, r, c.experts)
                exp = s['layout'][r]
                for got, key in zip(lay, ('send_idx', 'send_ids', 'send_counts', 'recv_counts',
                                          'starts', 'rows', 'cols')):
                    np.testing.assert_array_equal(got, exp[key], err_msg=f'{name} {i} r{r} {key}')
                np.testing.assert_array_equal(layer_slots(slots[r], c.caps[r], s['layer'], c.experts),
                                              exp['layer_slots'])


@pytest.mark.parametrize('name', [n for n in PLAN_CASES if n not in ('overflow', 'cfg0_caps5554')])
def test_plan_with_device_history(name):
    """The fused path: GateHistory update and scores computed on the device."""
    c = PlanCase(name)
    ctl = _controller(c)
    dev = ctl.device
    for i in range(c.steps):
        s = c.step(i)
        if not s['ok']:
            break
        ids = torch.as_tensor(s['selected'].astype(np.uint8), device=dev)
        dest = torch.empty(ids.shape, dtype=torch.int32, device=dev)
        prob = torch.as_tensor(s['rows'], device=dev) if s['rows'].size else None
        ctl._err.zero_()
        ctl.plan_device(s['event'], s['layer'], ids, dest, tokens_per_rank=c.tokens, prob_rows=prob)
        torch.cuda.synchronize()
        assert int(ctl._err.item()) == 0
        np.testing.assert_array_equal(ctl.scores[s['layer']], s['scores'], err_msg=f'{name} {i} scores')
        n = int(ctl._n_fetches.item())
        np.testing.assert_array_equal(ctl._fetches[:n].cpu().numpy(), s['fetches'], err_msg=f'{name} {i}')
        np.testing.assert_array_equal(dest.cpu().numpy(), s['dest'], err_msg=f'{name} {i} dest')


def test_greedy_quota_and_build_lut():
    from ferry_b200 import quota
    d = load('quota')
    for i in range(int(d['n'])):
        args = (int(d[f'c{i}_m']), d[f'c{i}_cap'], d[f'c{i}_masks'], d[f'c{i}_seconds'])
        if int(d[f'c{i}_ok']):
            np.testing.assert_array_equal(quota.greedy_quota(*args), d[f'c{i}_quota'], err_msg=f'case {i}')
        else:
            with pytest.raises(AssertionError):
                quota.greedy_quota(*args)
    for key in d.files:
        if key.startswith('lut') and not key.endswith(('_masks', '_seconds')):
            world = d[key].shape[1]
            np.testing.assert_array_equal(
                quota.build_lut(64, world, d[key + '_masks'], d[key + '_seconds']), d[key], err_msg=key)


def test_load_balanced_assignment():
    from ferry_b200.policy import load_balanced_assignment
    d = load('assignment')
    for i in range(int(d['n'])):
        got = load_balanced_assignment(d[f'c{i}_demand'], d[f'c{i}_misses'], d[f'c{i}_owner'],
                                       int(d[f'c{i}_layer']), d[f'c{i}_quota'], int(d[f'c{i}_bps']))
        np.testing.assert_array_equal(got, d[f'c{i}_ans'], err_msg=f'case {i}')


def test_choose_slot():
    from ferry_b200.policy import _choose_slot
    d = load('choose_slot')
    for i in range(int(d['n'])):
        got = _choose_slot(int(d[f'c{i}_rank']), int(d[f'c{i}_layer']), d[f'c{i}_active'],
                           d[f'c{i}_slots'], d[f'c{i}_caps'], d[f'c{i}_last'], d[f'c{i}_scores'],
                           int(d[f'c{i}_experts']))
        assert got == int(d[f'c{i}_slot']), f'case {i}'


def test_demand_and_admission_capacity():
    from oracle import planner as op
    from ferry_b200.policy import _admission_capacity, _demand
    c = PlanCase('qwen_r4')
    s = c.step(0)
    np.testing.assert_array_equal(_demand(s['selected'], c.origins(), c.experts, c.world),
                                  op.demand(s['selected'], c.origins(), c.experts, c.world))
    s5 = c.step(5)
    active = op.demand(s5['selected'], c.origins(), c.experts, c.world).sum(1) > 0
    np.testing.assert_array_equal(
        _admission_capacity(s['slots'], c.caps, s5['layer'], active, c.experts),
        op.admission_capacity(s['slots'], c.caps, s5['layer'], active, c.experts))


@pytest.mark.parametrize('world,tokens,experts,topk', [(1, 2500, 16, 4), (4, 700, 128, 8), (8, 300, 64, 6)])
def test_layout_multi_chunk_random(world, tokens, experts, topk):
    """The layout kernel past one 1,024-token chunk (prefill-sized layers),
    random destinations (including tokens with no route to some ranks),
    bit-exact against the oracle's build_layout for every rank."""
    from ferry_b200.layout import build_layout
    rng = np.random.default_rng(world * 1000 + tokens)
    n = world * tokens
    sel = np.stack([rng.choice(experts, topk, replace=False) for _ in range(n)]).astype(np.int64)
    owner = rng.integers(0, world, experts)
    dest = owner[sel]
    for r in range(world):
        got = build_layout(sel, dest, tokens, r, experts)
        want = op.build_layout(sel, dest, tokens, r, experts)
        for g, w, name in zip(got, want, ['send_idx', 'send_ids', 'send_counts', 'recv_counts',
                                          'starts', 'rows', 'cols']):
            np.testing.assert_array_equal(g, w, err_msg=f'{name} rank {r}')


@pytest.mark.parametrize('world,tokens,experts,topk', [(4, 700, 128, 8), (8, 300, 64, 6), (2, 1500, 32, 4)])
def test_fused_layout_outputs(world, tokens, experts, topk):
    """The fused executor's extra layout outputs: peer_row (receive row of each
    local token at every peer), recv_token and csr_pos, against numpy, for
    every rank, past one 1,024-token chunk."""
    from ferry_b200 import _lib
    from ferry_b200.layout import LayoutBuffers
    rng = np.random.default_rng(world + tokens)
    n = world * tokens
    sel = np.stack([rng.choice(experts, topk, replace=False) for _ in range(n)]).astype(np.int64)
    dest = rng.integers(0, world, (n, topk))
    ids_t = torch.as_tensor(sel.astype(np.uint8), device='cuda')
    dest_t = torch.as_tensor(dest.astype(np.int32), device='cuda')
    slot_of = torch.arange(experts, dtype=torch.int32, device='cuda')
    sends = np.stack([(dest == p).any(1) for p in range(world)])  # [world, n]
    for r in range(world):
        buf = LayoutBuffers(world, tokens, topk, experts, r, torch.device('cuda'), fused=True)
        buf.run(ids_t, dest_t, layer_slot=slot_of)
        torch.cuda.synchronize()
        _lib.check_device_error(buf.err, 'layout')
        want_pr = np.full((tokens, world), -1)
        for p in range(world):
            before = np.cumsum(sends[p]) - sends[p]
            g = r * tokens + np.arange(tokens)
            want_pr[:, p] = np.where(sends[p][g], before[g], -1)
        np.testing.assert_array_equal(buf.peer_row.cpu().numpy(), want_pr, err_msg=f'peer_row rank {r}')
        recv = np.flatnonzero(sends[r])
        n_recv = int(buf.n_recv.item())
        assert n_recv == recv.size
        np.testing.assert_array_equal(buf.recv_token[:n_recv].cpu().numpy(), recv)
        total = int(buf.starts[-1].item())
        rows, cols = buf.rows[:total].cpu().numpy(), buf.cols[:total].cpu().numpy()
        want_cp = np.full((n_recv, topk), -1)
        want_cp[rows, cols] = np.arange(total)
        np.testing.assert_array_equal(buf.csr_pos[:n_recv].cpu().numpy(), want_cp, err_msg=f'csr_pos rank {r}')


@pytest.mark.parametrize('world,caps_per_rank,layers,experts,topk,tokens', [
    (1, 300, 6, 64, 6, 48), (2, 90, 5, 64, 4, 40), (4, 40, 4, 128, 8, 24),
    # 2048 and 4096 slot records: two and four saved entries per thread
    (1, 1500, 32, 64, 6, 48), (2, 1100, 24, 128, 8, 32)])
def test_saved_victim_order_matches_full_sort(world, caps_per_rank, layers, experts, topk, tokens):
    """The incrementally maintained victim order against a controller that
    sorts every slot at every plan (its saved order cleared before each call):
    identical fetch lists, destinations and cache state over many layers,
    with Zipf-skewed routing, the device GateHistory and layers revisited out
    of order (including the same layer twice in a row)."""
    from ferry_b200.policy import Controller, _Spec
    from ferry_b200.quota import Topology
    rng = np.random.default_rng(world * 100 + layers)
    caps = [caps_per_rank] * world
    topo = Topology.uniform(world, experts)
    spec = _Spec(layers, experts, topk)
    inc = Controller(spec, caps, 'ferry', topo)
    full = Controller(spec, caps, 'ferry', topo)
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    order = [l % layers for l in range(3 * layers)] + list(rng.integers(0, layers, 3 * layers))
    order[5] = order[4]
    n = world * tokens
    for event, layer in enumerate(order):
        perm = rng.permutation(experts)
        sel = np.stack([perm[rng.choice(experts, topk, replace=False, p=p)] for _ in range(n)])
        ids = torch.as_tensor(sel.astype(np.uint8), device='cuda')
        full._order_meta.zero_()
        outs = []
        for ctl in (inc, full):
            dest = torch.empty(ids.shape, dtype=torch.int32, device='cuda')
            ctl.plan_device(event, layer, ids, dest, tokens_per_rank=tokens)
            torch.cuda.synchronize()
            assert int(ctl._err.item()) == 0
            m = int(ctl._n_fetches.item())
            outs.append((ctl._fetches[:m].cpu().numpy(), dest.cpu().numpy()))
        np.testing.assert_array_equal(outs[0][0], outs[1][0], err_msg=f'event {event} fetches')
        np.testing.assert_array_equal(outs[0][1], outs[1][1], err_msg=f'event {event} dest')
        np.testing.assert_array_equal(inc.slots, full.slots, err_msg=f'event {event} slots')
    assert int(inc._order_meta[0].item()) == 1
