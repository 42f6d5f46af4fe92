"""The CPU oracle against the reference's own outputs (tests/golden/, made by
running the reference's numba/numpy code).  Bit-exact throughout."""
import numpy as np
import pytest

from oracle import metadata as om
from oracle import planner as op
from tests.goldens import PLAN_CASES, PlanCase, load


def test_mt19937_matches_numba_randint():
    d = load('mt19937')
    for i in range(int(d['n'])):
        seed, n = int(d[f'c{i}_seed']), int(d[f'c{i}_n'])
        got = op.mt_randint_draws(seed, n, len(d[f'c{i}_draws']))
        np.testing.assert_array_equal(got, d[f'c{i}_draws'], err_msg=f'seed={seed} n={n}')


def test_greedy_quota_and_lut():
    d = load('quota')
    for i in range(int(d['n'])):
        args = (int(d[f'c{i}_m']), d[f'c{i}_cap'], d[f'c{i}_masks'], d[f'c{i}_seconds'])
        if int(d[f'c{i}_ok']):
            np.testing.assert_array_equal(op.greedy_quota(*args), d[f'c{i}_quota'], err_msg=f'case {i}')
        else:
            with pytest.raises(op.OracleAssertion):
                op.greedy_quota(*args)
    for key in d.files:
        if key.startswith('lut') and not key.endswith(('_masks', '_seconds')):
            masks, seconds = d[key + '_masks'], d[key + '_seconds']
            world = d[key].shape[1]
            np.testing.assert_array_equal(op.build_lut(64, world, masks, seconds), d[key], err_msg=key)


def test_load_balanced_assignment():
    d = load('assignment')
    for i in range(int(d['n'])):
        got = op.load_balanced_assignment(d[f'c{i}_demand'], d[f'c{i}_misses'], d[f'c{i}_owner'],
                                          int(d[f'c{i}_layer']), d[f'c{i}_quota'], int(d[f'c{i}_bps']))
        np.testing.assert_array_equal(got, d[f'c{i}_ans'], err_msg=f'case {i}')


def test_choose_slot():
    d = load('choose_slot')
    for i in range(int(d['n'])):
        got = op.choose_slot(int(d[f'c{i}_rank']), int(d[f'c{i}_layer']), d[f'c{i}_active'],
                             d[f'c{i}_slots'], d[f'c{i}_caps'], d[f'c{i}_last'], d[f'c{i}_scores'],
                             int(d[f'c{i}_experts']))
        assert got == int(d[f'c{i}_slot']), f'case {i}'


def test_gate_history():
    d = load('history')
    h = om.GateHistory(int(d['layers']), int(d['experts']), int(d['window']))
    for i in range(int(d['n'])):
        layer = int(d[f'c{i}_layer'])
        h.update(layer, d[f'c{i}_rows'])
        np.testing.assert_array_equal(h.scores(layer), d[f'c{i}_scores'], err_msg=f'case {i}')


@pytest.mark.parametrize('score', ['frequency', 'probability'])
def test_route_gather_rows(score):
    d = load(f'route_gather_{score}')
    world = int(d['world'])
    for step in range(4):
        sels = [d[f'r{r}_s{step}_sel'] for r in range(world)]
        ids, origins = om.gather_ids(sels)
        tokens = sels[0].shape[0]
        if score == 'frequency':
            rows = om.frequency_rows(ids, world, tokens, 128, 64)
        else:
            tail = om.history_tail(tokens, 128, world)
            rows = om.probability_rows([d[f'r{r}_s{step}_probs'][-tail:] for r in range(world)])
        for r in range(world):  # every rank receives the same gathered view
            np.testing.assert_array_equal(ids, d[f'r{r}_s{step}_ids'])
            np.testing.assert_array_equal(origins, d[f'r{r}_s{step}_origins'])
            np.testing.assert_array_equal(rows, d[f'r{r}_s{step}_rows'])


@pytest.mark.parametrize('name', PLAN_CASES)
def test_plan_sequence(name):
    c = PlanCase(name)
    ctl = op.Controller(c.layers, c.experts, c.caps, c.policy, c.masks, c.seconds, c.lut,
                        c.bps, c.salt)
    hist = om.GateHistory(c.layers, c.experts, c.window)
    tail = om.history_tail(c.tokens, c.window, c.world)
    for i in range(c.steps):
        s = c.step(i)
        sel = s['selected']
        if s['rows'].size:
            rows = s['rows']
        else:
            rows = om.frequency_rows(sel, c.world, c.tokens, c.window, c.experts)
        hist.update(s['layer'], rows)
        gs = hist.scores(s['layer'])
        np.testing.assert_array_equal(gs, s['scores'], err_msg=f'{name} step {i} scores')
        if not s['ok']:
            with pytest.raises(op.OracleAssertion):
                ctl.plan(s['event'], s['layer'], sel, c.origins(), gs)
            break
        f, dest, counts = ctl.plan(s['event'], s['layer'], sel, c.origins(), gs)
        np.testing.assert_array_equal(f, s['fetches'], err_msg=f'{name} step {i} fetches')
        np.testing.assert_array_equal(dest, s['dest'], err_msg=f'{name} step {i} destinations')
        np.testing.assert_array_equal(counts, s['counts'], err_msg=f'{name} step {i} counts')
        if 'slots' in s:
            np.testing.assert_array_equal(ctl.slots, s['slots'])
            np.testing.assert_array_equal(ctl.owner, s['owner'])
            np.testing.assert_array_equal(ctl.last, s['last'])
        for r in range(c.world):
            lay = op.build_layout(sel, dest, c.tokens, r, c.experts)
            exp = s['layout'][r]
            for got, key in zip(lay, ('send_idx', 'send_ids', 'send_counts', 'recv_counts',
                                      'starts', 'rows', 'cols')):
                np.testing.assert_array_equal(got, exp[key], err_msg=f'{name} step {i} rank {r} {key}')
            np.testing.assert_array_equal(op.layer_slots(ctl.slots[r], c.caps[r], s['layer'], c.experts),
                                          exp['layer_slots'])
