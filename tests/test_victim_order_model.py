"""The saved-victim-order rule of the device planner, checked on the CPU
against the oracle's own state evolution (no GPU): between two plans, a slot
record (rank, class, score, last use, key) changes only if its slot's content
changed or its key belongs to a layer planned since the order was saved or
to the layer being planned.  Replaying the reference's recorded plan
sequences, an order kept by that rule -- re-keying only those records and
merging them into the rest -- must equal a full sort of every record at every
plan that evicts."""
import numpy as np
import pytest

from oracle import metadata as om
from oracle import planner as op
from tests.goldens import PLAN_CASES, PlanCase


def _records(ctl, c, layer, active, scores_l):
    """Eviction key of every slot at eviction time (this layer's scores already
    written), as the device planner forms it; -> {slot index: key tuple}."""
    E = c.experts
    maxcap = int(np.max(c.caps))
    scores = ctl.scores.copy()
    scores[layer] = scores_l
    recs = {}
    for r, cap in enumerate(c.caps):
        for i in range(int(cap)):
            idx = r * maxcap + i
            key = int(ctl.slots[r][i])
            if key < 0:
                recs[idx] = (r, 0, 0.0, 0, i)
            elif key // E == layer and active[key % E]:
                recs[idx] = (r, 2, 0.0, 0, key)
            else:
                recs[idx] = (r, 1, float(scores.reshape(-1)[key]), int(ctl.last[key]), key)
    return recs


@pytest.mark.parametrize('name', PLAN_CASES)
def test_incremental_order_equals_full_sort(name):
    c = PlanCase(name)
    ctl = op.Controller(c.layers, c.experts, c.caps, c.policy, c.masks, c.seconds, c.lut, c.bps, c.salt)
    hist = om.GateHistory(c.layers, c.experts, c.window)
    E = c.experts
    saved = None          # [(slot, key tuple)] in order
    changed = set()       # layers planned since the order was saved
    checked = 0
    for i in range(c.steps):
        s = c.step(i)
        if not s['ok']:
            break
        layer = s['layer']
        rows = s['rows'] if s['rows'].size else om.frequency_rows(s['selected'], c.world, c.tokens,
                                                                    c.window, E)
        hist.update(layer, rows)
        gs = hist.scores(layer)
        active = np.zeros(E, bool)
        active[np.unique(s['selected'])] = True
        recs = _records(ctl, c, layer, active, gs)
        full = sorted(recs.items(), key=lambda kv: kv[1])
        m = len(s['fetches'])
        if m > 0:
            if saved is None:
                saved = full
            else:
                clean, dirty = [], []
                for idx, old in saved:
                    r, i_local = divmod(idx, int(np.max(c.caps)))
                    key = int(ctl.slots[r][i_local])
                    old_key = -1 if old[1] == 0 else old[4]
                    kl = key // E if key >= 0 else -1
                    if key != old_key or (key >= 0 and (kl == layer or kl in changed)):
                        dirty.append((idx, recs[idx]))
                    else:
                        clean.append((idx, old))
                merged = sorted(clean + sorted(dirty, key=lambda kv: kv[1]), key=lambda kv: kv[1])
                assert [kv[0] for kv in merged if kv[1][1] < 2] == [kv[0] for kv in full if kv[1][1] < 2], \
                    f'{name} step {i}: the kept order differs from a full sort'
                assert merged == [(idx, recs[idx]) for idx, _ in merged], f'{name} step {i}: stale record'
                checked += 1
                saved = full
            changed = {layer}
        elif saved is not None:
            changed.add(layer)
        ctl.plan(s['event'], layer, s['selected'], c.origins(), gs)
    if checked == 0:
        pytest.skip('no two evicting plans in this sequence')
