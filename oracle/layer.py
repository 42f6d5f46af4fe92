"""One FERRY MoE layer over R emulated ranks, end to end on the CPU (test
infrastructure only; also the CPU baseline that bench.py times).

Follows OffloadRuntime.execute (ferry/runtime.py:64-89) with every rank's
work done in this process: RouteGather (ferry/metadata.py:67-83), GateHistory,
Controller.plan (oracle/ferry_oracle.c), build_layout, pack_dispatch, the
all-to-all (in-process), execute_experts, reduce_partials, the combine
all-to-all and scatter_returned (oracle/expert_ops.py).  The expert cache of
a rank holds pool[key mod pool_rows] for every key in its slots, which is
what the reference's H2D copies put there.
"""
import numpy as np
import torch

from . import expert_ops as ops
from . import metadata as md
from . import planner as op


class OracleRuntime:
    def __init__(self, spec, pool, capacities, policy, masks, seconds, lut, window=128,
                 balance_tol_bps=200, salt=1, score='frequency'):
        self.spec, self.pool = spec, pool
        self.world = len(capacities)
        self.capacities = list(capacities)
        self.window, self.score = window, score
        self.ctl = op.Controller(spec.layers, spec.experts, capacities, policy, masks, seconds,
                                 lut, balance_tol_bps, salt)
        self.hist = md.GateHistory(spec.layers, spec.experts, window)
        self.event = 0
        self.fetches_per_rank = np.zeros(self.world, np.int64)

    def execute(self, layer, hidden, selected, weights, probs_tail=None):
        """hidden/selected/weights: one [T, .] CPU tensor per rank.  Returns the
        per-rank outputs [T, H] bf16 and the plan (fetches, destinations)."""
        spec, R = self.spec, self.world
        T = hidden[0].shape[0]
        ids, origins = md.gather_ids([s.numpy() for s in selected])
        if self.score == 'probability':
            tail = md.history_tail(T, self.window, R)
            rows = md.probability_rows([p[-tail:].numpy() for p in probs_tail])
        else:
            rows = md.frequency_rows(ids, R, T, self.window, spec.experts)
        self.hist.update(layer, rows)
        fetches, dest, counts = self.ctl.plan(self.event, layer, ids, origins, self.hist.scores(layer))
        self.fetches_per_rank += counts
        self.event += 1
        H, K, E = spec.hidden, spec.topk, spec.experts
        prow = self.pool.shape[0]
        layouts = [op.build_layout(ids, dest, T, r, E) for r in range(R)]
        payloads = [ops.pack_dispatch(hidden[s], selected[s], weights[s],
                                      torch.from_numpy(layouts[s][0]), torch.from_numpy(layouts[s][1]), E)
                    for s in range(R)]
        # all-to-all: receiver p gets, from each source s in rank order, s's packets for p
        partial_of = {}
        for p in range(R):
            pieces = []
            for s in range(R):
                sc = layouts[s][2]
                a = int(sc[:p].sum())
                pieces.append(payloads[s][a:a + int(sc[p])])
            raw = torch.cat(pieces) if pieces else torch.zeros(0, 2 * H + 3 * K, dtype=torch.uint8)
            x, w = ops.unpack_dispatch(raw, H, K)
            _, _, _, recv_counts, starts, rws, cls = layouts[p]
            slot_of = op.layer_slots(self.ctl.slots[p], self.capacities[p], layer, E)
            parts, part_rows = [], []
            for e in np.flatnonzero(starts[1:] > starts[:-1]):
                slot = int(slot_of[e])
                assert slot >= 0
                key = int(self.ctl.slots[p][slot])
                r = torch.from_numpy(rws[starts[e]:starts[e + 1]])
                c = torch.from_numpy(cls[starts[e]:starts[e + 1]])
                cache = self.pool[key % prow].unsqueeze(0)
                parts += ops.execute_experts(cache, x, w, [0], [r], [c], H, spec.intermediate)
                part_rows.append(r)
            partial = ops.reduce_partials(parts, part_rows, x.shape[0], H)
            # rows of the partial from source s are the receive rows of s's packets
            rc = recv_counts
            for s in range(R):
                a = int(rc[:s].sum())
                partial_of[(p, s)] = partial[a:a + int(rc[s])]
        outs = []
        for s in range(R):
            returned = torch.cat([partial_of[(p, s)] for p in range(R)])
            outs.append(ops.scatter_returned(returned, torch.from_numpy(layouts[s][0]), T))
        return outs, fetches, dest
