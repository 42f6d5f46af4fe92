"""The reference's GPU runtime, composed for timing (baseline infrastructure
only: bench.py --impl reference-gpu runs it; nothing in ferry_b200 imports it).

OffloadRuntime.execute (ferry/runtime.py:64-89) step by step, on this rank's
GPU, with the reference's own compiled ops from oracle/_ref (built from
ferry/csrc/expert_ops.{cpp,cu}: H2DEngine, pack_dispatch, unpack_dispatch,
execute_experts, reduce_partials, scatter_returned) and, for the numba parts
that cannot travel to the GPU box, the oracle's bit-exact C restatement of
Controller.plan and build_layout:

  RouteGather.collect (ferry/metadata.py:67-83): uint8 ids through NCCL
      all_gather_into_tensor, then a blocking copy to pinned host memory;
  GateHistory.update/scores (ferry/metadata.py:24-38);
  Controller.plan (ferry/policy.py:130-194, oracle/ferry_oracle.c);
  H2DEngine.fetch of this rank's misses (ferry/csrc/expert_ops.cpp:105-116);
  device_layout (ferry/layout.py:80-94): build_layout on the host, one
      blocking host-to-device copy of the index arrays;
  Transport.dispatch (ferry/transport.py:22-29): pack_dispatch, NCCL
      all_to_all_single, unpack_dispatch;
  H2DEngine.wait_host (serial execution: the GEMMs wait for every fetch);
  execute_experts (cuBLAS per expert), mark_used;
  Transport.combine (ferry/transport.py:31-38): reduce_partials, NCCL
      all_to_all_single, scatter_returned.

The MoE hook's router (ferry/model.py:137-148) runs in torch on the GPU.
"""
import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import metadata as md
from . import planner as op
from .build_ref import load_ref


class RefGpuRuntime:
    def __init__(self, spec, pool, capacities, policy, masks, seconds, lut, window=128,
                 balance_tol_bps=200, salt=1):
        self.ops = load_ref()
        if self.ops is None:
            raise RuntimeError('the reference extension is not built (oracle/build_ref.py)')
        self.spec, self.pool = spec, pool
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.capacities = list(capacities)
        self.cap = self.capacities[self.rank]
        self.window = window
        self.cache = torch.empty((self.cap, spec.expert_elements), dtype=torch.bfloat16, device='cuda')
        self.ctl = op.Controller(spec.layers, spec.experts, capacities, policy, masks, seconds, lut,
                                 balance_tol_bps, salt)
        self.hist = md.GateHistory(spec.layers, spec.experts, window)
        self.h2d = self.ops.H2DEngine(self.cache, pool)
        self.event = 0
        self.fetches_per_rank = np.zeros(self.world, np.int64)
        self._gather = {}

    def route(self, hidden, gate, bias=None):
        """_qwen3_forward's router: bf16 gate Linear, float32 softmax, top-k,
        renormalisation, bf16 weights (the synthetic popularity bias as the
        Linear's bias)."""
        logits = F.linear(hidden, gate, None if bias is None else bias.to(hidden.dtype))
        probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
        weights, selected = torch.topk(probs, self.spec.topk, dim=-1)
        weights = weights / weights.sum(-1, keepdim=True)
        return selected, weights.to(hidden.dtype)

    def _collect(self, selected):
        tokens = selected.shape[0]
        if tokens not in self._gather:
            n = tokens * self.spec.topk
            self._gather[tokens] = (torch.empty(n, dtype=torch.uint8, device='cuda'),
                                    torch.empty(self.world * n, dtype=torch.uint8, device='cuda'),
                                    torch.empty(self.world * n, dtype=torch.uint8, pin_memory=True))
        send, recv, host = self._gather[tokens]
        send.copy_(selected.to(torch.uint8).reshape(-1))
        dist.all_gather_into_tensor(recv, send)
        host.copy_(recv)  # blocking, as ferry/metadata.py:74
        ids = host.numpy().reshape(self.world * tokens, self.spec.topk).astype(np.int64)
        origins = np.repeat(np.arange(self.world, dtype=np.int64), tokens)
        return ids, origins

    @staticmethod
    def _exchange(x, send, recv):
        y = torch.empty((sum(recv),) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
        dist.all_to_all_single(y, x, output_split_sizes=recv, input_split_sizes=send)
        return y

    def execute(self, layer, hidden, selected, weights):
        spec, ops = self.spec, self.ops
        T, E, H = hidden.shape[0], spec.experts, spec.hidden
        ids, origins = self._collect(selected)
        self.hist.update(layer, md.frequency_rows(ids, self.world, T, self.window, E))
        fetches, dest, counts = self.ctl.plan(self.event, layer, ids, origins, self.hist.scores(layer))
        self.fetches_per_rank += counts
        mine = fetches[fetches[:, 0] == self.rank]
        fetch_slots = mine[:, 2].tolist()
        self.h2d.fetch(fetch_slots, mine[:, 1].tolist())
        slot_of = op.layer_slots(self.ctl.slots[self.rank], self.cap, layer, E)
        send_idx, send_ids, send_counts, recv_counts, starts, rows, cols = op.build_layout(
            ids, dest, T, self.rank, E)
        group_experts = np.flatnonzero(starts[1:] > starts[:-1])
        pieces = [send_idx, send_ids.reshape(-1)]
        for e in group_experts:
            pieces += [rows[starts[e]:starts[e + 1]], cols[starts[e]:starts[e + 1]]]
        storage = torch.from_numpy(np.concatenate(pieces)).to('cuda', non_blocking=False)
        views = storage.split([len(p) for p in pieces])
        d_send_idx, d_send_ids = views[0], views[1].view(-1, spec.topk)
        g_slots = [int(slot_of[e]) for e in group_experts]
        g_rows = [views[2 + 2 * i] for i in range(len(group_experts))]
        g_cols = [views[3 + 2 * i] for i in range(len(group_experts))]
        send, recv = send_counts.tolist(), recv_counts.tolist()
        payload = ops.pack_dispatch(hidden, selected, weights, d_send_idx, d_send_ids, E)
        x, w = ops.unpack_dispatch(self._exchange(payload, send, recv), H, spec.topk)
        self.h2d.wait_host(fetch_slots)
        parts = ops.execute_experts(self.cache, x, w, g_slots, g_rows, g_cols, H, spec.intermediate)
        self.h2d.mark_used(g_slots)
        self.event += 1
        partial = ops.reduce_partials(parts, g_rows, sum(recv), H, hidden)
        returned = self._exchange(partial, recv, send)
        return ops.scatter_returned(returned, d_send_idx, T)

    def close(self):
        self.h2d.synchronize()
