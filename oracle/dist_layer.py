"""One FERRY MoE layer as the reference runs it across processes, on the CPU
over gloo (test infrastructure only).

Follows ferry/runtime.py:64-89 with real collectives: every rank all-gathers
the uint8 ids (ferry/metadata.py:70-76), plans identically (oracle planner),
builds its own layout, all-to-alls its packets (ferry/transport.py:17-29),
runs its cached experts (weights read from the pool as the cache would hold
them), reduces per packet, all-to-alls the partials back and scatters them
(ferry/transport.py:31-38).  The benchmark's config 0 (a DeepSeek-V2-Lite
layer on CPU) runs this at world size 4.
"""
import numpy as np
import torch
import torch.distributed as dist

from . import expert_ops as ops
from . import metadata as md
from . import planner as op


class DistOracleRuntime:
    def __init__(self, spec, pool, capacities, policy, masks, seconds, lut, window=128,
                 balance_tol_bps=200, salt=1):
        self.spec, self.pool = spec, pool
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.capacities = list(capacities)
        self.window = window
        self.ctl = op.Controller(spec.layers, spec.experts, capacities, policy, masks, seconds, lut,
                                 balance_tol_bps, salt)
        self.hist = md.GateHistory(spec.layers, spec.experts, window)
        self.event = 0

    @staticmethod
    def _exchange(x, send, recv):
        y = torch.empty((sum(recv),) + tuple(x.shape[1:]), dtype=x.dtype)
        dist.all_to_all_single(y, x.contiguous(), output_split_sizes=recv, input_split_sizes=send)
        return y

    def execute(self, layer, hidden, selected, weights):
        spec, R, rank = self.spec, self.world, self.rank
        T, K, E, H = hidden.shape[0], spec.topk, spec.experts, spec.hidden
        send = selected.to(torch.uint8).reshape(-1).contiguous()
        recv = torch.empty(R * send.numel(), dtype=torch.uint8)
        dist.all_gather_into_tensor(recv, send)
        ids = recv.numpy().reshape(R * T, K).astype(np.int64)
        origins = np.repeat(np.arange(R, dtype=np.int64), T)
        self.hist.update(layer, md.frequency_rows(ids, R, T, self.window, E))
        fetches, dest, counts = self.ctl.plan(self.event, layer, ids, origins, self.hist.scores(layer))
        self.event += 1
        send_idx, send_ids, send_counts, recv_counts, starts, rows, cols = op.build_layout(
            ids, dest, T, rank, E)
        payload = ops.pack_dispatch(hidden, selected, weights, torch.from_numpy(send_idx),
                                    torch.from_numpy(send_ids), E)
        raw = self._exchange(payload, send_counts.tolist(), recv_counts.tolist())
        x, w = ops.unpack_dispatch(raw, H, K)
        slot_of = op.layer_slots(self.ctl.slots[rank], self.capacities[rank], layer, E)
        parts, part_rows = [], []
        for e in np.flatnonzero(starts[1:] > starts[:-1]):
            slot = int(slot_of[e])
            assert slot >= 0, 'expert scheduled on this rank is not cached here'
            key = int(self.ctl.slots[rank][slot])
            r = torch.from_numpy(rows[starts[e]:starts[e + 1]])
            c = torch.from_numpy(cols[starts[e]:starts[e + 1]])
            parts += ops.execute_experts(self.pool[key % self.pool.shape[0]].unsqueeze(0), x, w, [0],
                                         [r], [c], H, spec.intermediate)
            part_rows.append(r)
        partial = ops.reduce_partials(parts, part_rows, x.shape[0], H)
        returned = self._exchange(partial, recv_counts.tolist(), send_counts.tolist())
        return ops.scatter_returned(returned, torch.from_numpy(send_idx), T), fetches
