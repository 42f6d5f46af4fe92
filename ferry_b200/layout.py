"""Drop-in for ferry/layout.py: the expert-parallel layout on the GPU.

build_layout keeps the reference's signature (ferry/layout.py:12, numpy in,
numpy out) and device_layout its dict result (ferry/layout.py:78-94), without
the blocking host-to-device upload: the layout is computed by a CUDA kernel
from device-resident ids and destinations.  LayoutBuffers is the fused
runtime's preallocated form (no allocation per layer).
"""
import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import addr, call, stream_ptr


class LayoutBuffers:
    """Device buffers of one rank's layout for up to `tokens_per_rank` tokens."""

    def __init__(self, world, tokens_per_rank, topk, experts, rank, device, fused=True):
        self.world, self.T, self.topk, self.experts, self.rank = world, tokens_per_rank, topk, experts, rank
        n_tok = world * tokens_per_rank
        i64, i32 = torch.int64, torch.int32
        z = lambda *shape, dtype=i64: torch.zeros(shape, dtype=dtype, device=device)  # noqa: E731
        self.send_idx = z(max(1, tokens_per_rank * world))
        self.send_ids = z(max(1, tokens_per_rank * world), topk)
        self.send_counts = z(world)
        self.recv_counts = z(world)
        self.starts = z(experts + 1)
        self.rows = z(max(1, n_tok * topk))
        self.cols = z(max(1, n_tok * topk))
        self.n_send = z(1, dtype=i32)
        self.n_recv = z(1, dtype=i32)
        self.err = z(1, dtype=i32)
        self.fused = fused
        if fused:
            self.recv_token = z(max(1, n_tok), dtype=i32)
            self.csr_pos = z(max(1, n_tok), topk, dtype=i32)
            self.peer_row = z(max(1, tokens_per_rank), world, dtype=i32)
            self.groups = z(experts, 4, dtype=i32)  # GemmGroup {slot, start, count, expert}
            self.summary_dev = z(ctypes.sizeof(_lib.LayoutSummary), dtype=torch.uint8)
        else:
            self.recv_token = self.csr_pos = self.peer_row = self.groups = self.summary_dev = None

    def args(self, ids, dest, fetches=None, n_fetches=None, layer_slot=None):
        a = _lib.LayoutArgs()
        a.ids, a.dest = addr(ids), addr(dest)
        a.world, a.tokens_per_rank, a.topk, a.experts, a.rank = (
            self.world, self.T, self.topk, self.experts, self.rank)
        a.fetches, a.n_fetches, a.layer_slot = addr(fetches), addr(n_fetches), addr(layer_slot)
        for name in ('send_idx', 'send_ids', 'send_counts', 'recv_counts', 'starts', 'rows',
                     'cols', 'n_send', 'n_recv', 'recv_token', 'csr_pos', 'peer_row', 'groups',
                     'err'):
            setattr(a, name, addr(getattr(self, name)))
        a.summary = addr(self.summary_dev)
        return a

    def run(self, ids, dest, fetches=None, n_fetches=None, layer_slot=None, stream=None):
        a = self.args(ids, dest, fetches, n_fetches, layer_slot)
        self._args = a  # keep alive until the launch is enqueued
        call('ferryb_build_layout', ctypes.byref(a),
             stream if stream is not None else stream_ptr(ids.device))


def _device():
    return torch.device('cuda', torch.cuda.current_device())


def _check_shapes(sel_shape, dest_shape, n_local):
    """selected and destinations: the same [world * n_local, k] shape (the
    kernel reads both through bare pointers)."""
    if (len(sel_shape) != 2 or tuple(dest_shape) != tuple(sel_shape) or n_local <= 0
            or sel_shape[0] % n_local):
        raise _lib.FerrybError(f'selected {list(sel_shape)} and destinations {list(dest_shape)} must '
                               f'be equal [world * {n_local}, k] arrays')


def build_layout(selected, destinations, n_local, rank, experts):
    """ferry/layout.py:12-75 -> (send_idx, send_ids, send_counts, recv_counts,
    starts, rows, cols) as int64 numpy arrays."""
    dev = _device()
    sel = np.asarray(selected)
    _check_shapes(sel.shape, np.shape(destinations), n_local)
    world = sel.shape[0] // n_local
    topk = sel.shape[1]
    ids = torch.as_tensor(sel.astype(np.uint8), device=dev)
    dest = torch.as_tensor(np.asarray(destinations).astype(np.int32), device=dev)
    buf = LayoutBuffers(world, n_local, topk, experts, rank, dev, fused=False)
    buf.run(ids, dest)
    _lib.check_device_error(buf.err, 'build_layout')
    sent, total = int(buf.n_send.item()), None
    starts = buf.starts.cpu().numpy()
    total = int(starts[-1])
    return (buf.send_idx[:sent].cpu().numpy(), buf.send_ids[:sent].cpu().numpy(),
            buf.send_counts.cpu().numpy(), buf.recv_counts.cpu().numpy(), starts,
            buf.rows[:total].cpu().numpy(), buf.cols[:total].cpu().numpy())


def device_layout(selected, destinations, tokens_per_rank, rank, experts, slot_of):
    """ferry/layout.py:78-94: the same dict, with device index tensors."""
    dev = _device()
    sel = torch.as_tensor(np.asarray(selected).astype(np.uint8), device=dev) \
        if not torch.is_tensor(selected) else selected.to(dev, torch.uint8)
    dst = torch.as_tensor(np.asarray(destinations).astype(np.int32), device=dev) \
        if not torch.is_tensor(destinations) else destinations.to(dev, torch.int32)
    _check_shapes(tuple(sel.shape), tuple(dst.shape), tokens_per_rank)
    world = sel.shape[0] // tokens_per_rank
    topk = sel.shape[1]
    buf = LayoutBuffers(world, tokens_per_rank, topk, experts, rank, dev, fused=False)
    buf.run(sel, dst)
    _lib.check_device_error(buf.err, 'device_layout')
    starts = buf.starts.cpu().numpy()
    sent = int(buf.n_send.item())
    groups = []
    for e in np.flatnonzero(starts[1:] > starts[:-1]):
        slot = int(slot_of[e])
        assert slot >= 0, 'expert scheduled on this rank is not cached here'
        a, b = int(starts[e]), int(starts[e + 1])
        groups.append((int(e), buf.rows[a:b], buf.cols[a:b], slot))
    return dict(send_idx=buf.send_idx[:sent], send_ids=buf.send_ids[:sent],
                send_counts=buf.send_counts.cpu().tolist(), recv_counts=buf.recv_counts.cpu().tolist(),
                groups=groups)
