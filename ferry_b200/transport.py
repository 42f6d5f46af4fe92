"""Drop-in for ferry/transport.py: dispatch and combine for callers that
compose the reference's own layer flow.

Packets keep the reference's bf16 wire format ([hidden | per-expert routing
weights | expert ids] bytes, ferry/transport.py:22-29) and are packed,
unpacked, reduced and scattered by libferryb's kernels (ferry_b200.expert_ops);
the two exchanges are torch.distributed all_to_all_single calls with the
layout's split sizes, as in the reference.  The fused executor
(ferry_b200.runtime) replaces both exchanges with P2P stores into the peers'
symmetric buffers inside its dispatch and combine kernels.
"""
import torch
import torch.distributed as dist

from . import expert_ops as default_ops


class Transport:
    def __init__(self, ops=None, topk=None, experts=None, group=None):
        self.ops = ops if ops is not None else default_ops
        self.topk, self.experts, self.group = topk, experts, group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dispatch_bytes = self.combine_bytes = 0

    def _exchange(self, x, send, recv):
        send, recv = [int(v) for v in send], [int(v) for v in recv]
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return x.contiguous()
        y = torch.empty((sum(recv),) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
        dist.all_to_all_single(y, x.contiguous(), output_split_sizes=recv, input_split_sizes=send,
                               group=self.group)
        return y

    def dispatch(self, hidden, selected, weights, layout):
        """Packets to the ranks that own their experts; returns (x, w) of the
        packets this rank received."""
        payload = self.ops.pack_dispatch(hidden, selected, weights, layout['send_idx'],
                                         layout['send_ids'], self.experts)
        send, recv = layout['send_counts'], layout['recv_counts']
        raw = self._exchange(payload, send, recv)
        self.dispatch_bytes += (int(sum(send)) - int(send[self.rank])) * payload.shape[1]
        return self.ops.unpack_dispatch(raw, hidden.shape[1], self.topk)

    def combine(self, hidden, parts, layout):
        """One fp32-summed partial per received packet back to its source rank,
        summed there into the token's output."""
        recv, send = layout['recv_counts'], layout['send_counts']
        received = int(sum(recv))
        partial = self.ops.reduce_partials(parts, [g[1] for g in layout['groups']], received,
                                           hidden.shape[1], hidden)
        returned = self._exchange(partial, recv, send)
        self.combine_bytes += (received - int(recv[self.rank])) * hidden.shape[1] * 2
        return self.ops.scatter_returned(returned, layout['send_idx'], hidden.shape[0])
