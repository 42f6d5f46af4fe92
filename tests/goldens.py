"""Readers for the golden fixtures in tests/golden/ (produced by make_golden.py)."""
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / 'golden'

PLAN_CASES = sorted(p.stem[len('plan_'):] for p in GOLDEN.glob('plan_*.npz'))


def load(name):
    return np.load(GOLDEN / f'{name}.npz')


class PlanCase:
    """One recorded Controller.plan sequence of the reference."""

    def __init__(self, name):
        self.name = name
        d = load(f'plan_{name}')
        self.d = d
        for k in ('layers', 'experts', 'topk', 'world', 'tokens', 'policy', 'bps', 'salt',
                  'window', 'steps', 'state_every'):
            setattr(self, k, int(d[k]))
        self.caps = d['caps']
        self.masks, self.seconds, self.lut = d['masks'], d['seconds'], d['lut']

    def origins(self):
        return np.repeat(np.arange(self.world, dtype=np.int64), self.tokens)

    def step(self, i):
        d = self.d
        s = dict(layer=int(d[f's{i}_layer']), event=int(d[f's{i}_event']),
                 selected=d[f's{i}_selected'].astype(np.int64), scores=d[f's{i}_scores'],
                 rows=d[f's{i}_rows'], ok=bool(d[f's{i}_ok']))
        if s['ok']:
            s.update(fetches=d[f's{i}_fetches'], dest=d[f's{i}_dest'].astype(np.int64),
                     counts=d[f's{i}_counts'])
            if f's{i}_slots' in d.files:
                s.update(slots=d[f's{i}_slots'].astype(np.int64),
                         owner=d[f's{i}_owner'].astype(np.int64),
                         last=d[f's{i}_last'].astype(np.int64))
            s['layout'] = {r: dict(send_idx=d[f's{i}_r{r}_send_idx'], send_ids=d[f's{i}_r{r}_send_ids'],
                                   send_counts=d[f's{i}_r{r}_send_counts'],
                                   recv_counts=d[f's{i}_r{r}_recv_counts'],
                                   starts=d[f's{i}_r{r}_starts'], rows=d[f's{i}_r{r}_rows'],
                                   cols=d[f's{i}_r{r}_cols'],
                                   layer_slots=d[f's{i}_r{r}_layer_slots'])
                           for r in range(self.world)}
        return s
