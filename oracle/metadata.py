"""CPU restatement of ferry/metadata.py (test infrastructure only).

GateHistory (ferry/metadata.py:15-38) and the RouteGather gather/row rule
(ferry/metadata.py:55-83), over numpy without torch.distributed so the tests
can drive R emulated ranks in one process.
"""
import numpy as np


def history_tail(tokens, window, world):
    """ferry/metadata.py:57 -- history rows contributed per rank: min(T, ceil(W / R))."""
    return min(tokens, (window + world - 1) // world)


def gather_ids(selected_per_rank):
    """ferry/metadata.py:70-76 -- rank-major all-gather of uint8 expert ids.

    selected_per_rank: one [T, k] integer array per rank (ids < 256).
    Returns (expert_ids[R*T, k] int64, origins[R*T] int64)."""
    world = len(selected_per_rank)
    wire = np.concatenate([np.asarray(s).astype(np.uint8).ravel() for s in selected_per_rank])
    tokens, topk = np.asarray(selected_per_rank[0]).shape
    ids = wire.astype(np.int64).reshape(world * tokens, topk)
    origins = np.arange(world * tokens, dtype=np.int64) // tokens
    return ids, origins


def frequency_rows(expert_ids, world, tokens, window, experts):
    """ferry/metadata.py:80-82 -- 0/1 indicator rows (float64) of the last `tail`
    tokens of every rank, rank-major."""
    topk = expert_ids.shape[1]
    tail = history_tail(tokens, window, world)
    per_rank = expert_ids.reshape(world, tokens, topk)
    rows = np.zeros((world * tail, experts), np.float64)
    for r in range(world):
        for i in range(tail):
            rows[r * tail + i, per_rank[r, tokens - tail + i]] = 1.0
    return rows


def probability_rows(prob_tails):
    """ferry/metadata.py:72, :78 -- rank-major float32 router-probability tails."""
    return np.concatenate([np.asarray(p, np.float32) for p in prob_tails], 0)


class GateHistory:
    """ferry/metadata.py:15-38 -- per-layer ring of the W most recent history rows.

    A batch of n >= W rows replaces the ring with its last W rows (ring head 0);
    a shorter batch is appended at the head.  scores() is the float64 sum of
    the ring's W slots, taken slot 0 first and slot W-1 last (unfilled slots
    are zero), divided by max(1, count) and rounded once to float32."""

    def __init__(self, layers, experts, window=128):
        self.window = window
        self.ring = np.zeros((layers, window, experts), np.float64)
        self.count = np.zeros(layers, np.int64)
        self.head = np.zeros(layers, np.int64)

    def update(self, layer, rows):
        rows = np.asarray(rows, np.float64)
        w = self.window
        if rows.shape[0] >= w:
            self.ring[layer] = rows[rows.shape[0] - w:]
            self.count[layer], self.head[layer] = w, 0
            return
        for row in rows:
            self.ring[layer, self.head[layer]] = row
            self.head[layer] = (self.head[layer] + 1) % w
            self.count[layer] = min(w, self.count[layer] + 1)

    def scores(self, layer):
        acc = np.zeros(self.ring.shape[2], np.float64)
        for slot in range(self.window):
            acc = acc + self.ring[layer, slot]
        return (acc / max(1, int(self.count[layer]))).astype(np.float32)
