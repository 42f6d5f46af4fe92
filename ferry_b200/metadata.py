"""Drop-in for ferry/metadata.py: RouteGather and GateHistory.

The fused executor (ferry_b200.runtime) does this work inside kernels 1 and
2; these classes serve callers that compose the reference's own flow
(RouteGather.collect -> GateHistory.update/scores -> Controller.plan).

RouteGather.collect all-gathers the uint8 expert ids (and, for the
probability score, the float32 router-probability tail) with P2P stores into
every rank's symmetric buffer plus a sequence flag per rank
(ferryb_symm_allgather / ferryb_symm_wait) instead of NCCL, then makes the
one device-to-host copy the reference makes (ferry/metadata.py:74).  Its
outputs are the reference's: expert_ids [R*T, k] int64, origins [R*T] int64
and the history rows [R*tail, E] float64 (frequency: one-hot of each rank's
last `tail` tokens, rank-major) or float32 (probability).

GateHistory keeps the ring on the GPU (ferryb_history_update / _scores):
update takes the rows RouteGather returns, scores returns float32 numpy.
"""
import ctypes

import numpy as np
import torch
import torch.distributed as dist

from ._lib import call, ptr, stream_ptr
from .symm import SymmetricBuffer


def _rank_world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


class _CudaBytes:
    """A raw device address range seen through __cuda_array_interface__ (no
    stream synchronisation implied: the caller orders it on its stream)."""

    def __init__(self, address, nbytes):
        self.__cuda_array_interface__ = {'shape': (nbytes,), 'typestr': '|u1',
                                         'data': (address, False), 'version': 3, 'stream': None}


def _device_bytes(address, nbytes, device):
    return torch.as_tensor(_CudaBytes(address, nbytes), device=device)


class GateHistory:
    """Per-layer mean of the history rows of the W most recent routed tokens
    (ferry/metadata.py:15-38), on the GPU."""

    def __init__(self, layers, experts, window=128, device=None):
        self.layers, self.experts, self.window = layers, experts, window
        self.device = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
        self._rows = torch.zeros((layers, window, experts), dtype=torch.float64, device=self.device)
        self._count = torch.zeros(layers, dtype=torch.int64, device=self.device)
        self._head = torch.zeros(layers, dtype=torch.int64, device=self.device)

    def update(self, layer, probs):
        p = torch.as_tensor(np.ascontiguousarray(probs, dtype=np.float64)).to(self.device)
        if p.ndim != 2 or p.shape[1] != self.experts:
            raise ValueError(f'history rows must be [n, {self.experts}]')
        call('ferryb_history_update', ptr(self._rows), ptr(self._count), ptr(self._head), self.layers,
             self.window, self.experts, int(layer), ptr(p), p.shape[0], stream_ptr(self.device))

    def scores(self, layer):
        out = torch.empty(self.experts, dtype=torch.float32, device=self.device)
        call('ferryb_history_scores', ptr(self._rows), ptr(self._count), self.layers, self.window,
             self.experts, int(layer), ptr(out), stream_ptr(self.device))
        return out.cpu().numpy()

    @property
    def rows(self):
        return self._rows.cpu().numpy()

    @property
    def count(self):
        return self._count.cpu().numpy()

    @property
    def head(self):
        return self._head.cpu().numpy()


class _Slots:
    """Buffers of one token count: a send staging row, the symmetric receive
    buffer (two halves alternating by call parity, each holding every rank's
    row and then one flag word per rank), pinned host memory."""

    def __init__(self, rg, tokens):
        self.tail = min(tokens, -(-rg.window // rg.world))
        self.ids = tokens * rg.topk
        self.size = self.ids + (self.tail * rg.experts * 4 if rg.score == 'probability' else 0)
        self.stride = (self.size + 15) // 16 * 16  # 16-byte rows for vector stores
        self.send = torch.zeros(self.stride, dtype=torch.uint8, device=rg.device)
        self.host = torch.empty(rg.world * self.stride, dtype=torch.uint8, pin_memory=True)
        self.origins = np.repeat(np.arange(rg.world, dtype=np.int64), tokens)
        self.flags_at = rg.world * self.stride
        self.half = (self.flags_at + 8 * rg.world + 255) // 256 * 256
        self.err = torch.zeros(1, dtype=torch.int32, device=rg.device)
        self.symm = None
        if rg.world > 1:
            self.symm = SymmetricBuffer(2 * self.half, rg.rank, rg.world, rg.group)
            self.peers = torch.tensor(self.symm.bases, dtype=torch.int64, device=rg.device)
            self.calls = 0

    def close(self):
        if self.symm is not None:
            self.symm.close()
            self.symm = None


class RouteGather:
    """Fixed-size all-gather of expert ids (and the router-probability tail) per
    rank (ferry/metadata.py:41-83).  Every rank must hold the same number of
    tokens in a forward pass."""

    def __init__(self, topk, experts, window, score='frequency', group=None, device=None):
        if score not in ('frequency', 'probability'):
            raise ValueError(score)
        self.topk, self.experts, self.window, self.score = topk, experts, window, score
        self.group = group
        self.rank, self.world = _rank_world(group)
        self.device = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
        self.buffers = {}

    def _slots(self, tokens):
        s = self.buffers.get(tokens)
        if s is None:
            s = self.buffers[tokens] = _Slots(self, tokens)
        return s

    def collect(self, selected, probs_tail):
        tokens = selected.shape[0]
        s = self._slots(tokens)
        s.send[:s.ids].copy_(selected.to(torch.uint8).reshape(-1))
        if self.score == 'probability':
            tail = probs_tail[-s.tail:].float().contiguous().view(torch.uint8).reshape(-1)
            s.send[s.ids:s.size].copy_(tail)
        stream = stream_ptr(self.device)
        if s.symm is None:
            s.host[:s.stride].copy_(s.send)
        else:
            s.calls += 1
            seq = s.calls
            base = (seq & 1) * s.half
            call('ferryb_symm_allgather', ptr(s.peers), self.world, self.rank, base, ptr(s.send),
                 s.stride, base + s.flags_at, ctypes.c_uint64(seq), stream)
            call('ferryb_symm_wait', ctypes.c_void_p(s.symm.local), base + s.flags_at, self.world,
                 ctypes.c_uint64(seq), ptr(s.err), stream)
            s.host.copy_(_device_bytes(s.symm.local + base, self.world * s.stride, self.device))
            if int(s.err.item()):
                raise RuntimeError('RouteGather: timed out waiting for a peer rank\'s routing ids')
        raw = s.host.numpy().reshape(self.world, s.stride)[:, :s.size]
        expert_ids = raw[:, :s.ids].reshape(self.world * tokens, self.topk).astype(np.int64)
        if self.score == 'probability':
            rows = raw[:, s.ids:].copy().view(np.float32).reshape(self.world * s.tail, self.experts)
        else:
            recent = expert_ids.reshape(self.world, tokens, self.topk)[:, tokens - s.tail:]
            rows = np.zeros((self.world * s.tail, self.experts), np.float64)
            np.put_along_axis(rows, recent.reshape(-1, self.topk), 1.0, axis=1)
        return expert_ids, s.origins, rows

    def close(self):
        for s in self.buffers.values():
            s.close()
        self.buffers = {}
