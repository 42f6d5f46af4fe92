"""Drop-in for the reference's native module ``ferry_expert_ops``
(ferry/csrc/expert_ops.cpp:144-157): same function names, argument meaning
and error behaviour (RuntimeError on bad input), backed by libferryb's sm_100a
kernels through the C ABI.  Outputs are allocated by the torch caching
allocator; inputs are borrowed.
"""
import ctypes

import torch

from . import _lib
from ._lib import call, ptr, require_cuda, stream_ptr

BF16 = torch.bfloat16


def _check(cond, msg):
    if not cond:
        raise _lib.FerrybError(msg)


def execute_experts(cache, input, routing_weights, slots, rows, cols, hidden, intermediate):
    """ferry/csrc/expert_ops.cpp:16-45.  Returns one [len(rows[i]), hidden] bf16
    tensor per group: (silu(x Wg^T) * (x Wu^T)) Wd^T * w[rows, cols]."""
    require_cuda(cache, input, routing_weights)
    _check(cache.dtype == BF16 and input.dtype == BF16 and routing_weights.dtype == BF16,
           'cache, input and routing_weights must be bf16')
    _check(cache.dim() == 2 and cache.is_contiguous() and cache.shape[1] == 3 * hidden * intermediate,
           'cache must be contiguous [slots, 3*hidden*intermediate]')
    _check(input.dim() == 2 and input.shape[1] == hidden, 'input must be [n, hidden]')
    _check(routing_weights.dim() == 2 and routing_weights.shape[0] == input.shape[0],
           'routing_weights must be [n, topk]')
    _check(len(slots) == len(rows) == len(cols), 'slots, rows and cols must have equal length')
    sizes = []
    for r, c in zip(rows, cols):
        _check(r.dtype == torch.long and c.shape == r.shape, 'rows/cols must be matching int64')
        sizes.append(int(r.numel()))
    total = sum(sizes)
    out = torch.empty((total, hidden), dtype=BF16, device=input.device)
    if total:
        input_c = input.contiguous()
        rw = routing_weights.contiguous()
        rows_c = torch.cat([r.reshape(-1) for r in rows]).to(input.device)
        cols_c = torch.cat([c.reshape(-1) for c in cols]).to(input.device)
        n_groups = len(slots)
        ws_bytes = _lib.lib().ferryb_execute_experts_workspace(total, n_groups, hidden, intermediate)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=input.device)
        call('ferryb_execute_experts', ptr(cache), cache.shape[0], ptr(input_c), input_c.shape[0],
             ptr(rw), rw.shape[1], _lib.host_i64(slots), _lib.host_i64(sizes), n_groups,
             ptr(rows_c), ptr(cols_c), hidden, intermediate, ptr(out), ptr(ws), ws_bytes,
             stream_ptr(input.device))
    return list(out.split(sizes)) if sizes else []


def pack_dispatch(hidden, selected, weights, send_idx, send_ids, experts):
    """ferry/csrc/expert_ops.cpp:50-66 -> uint8 [n, 2H + 3k] packets."""
    require_cuda(hidden, selected, weights, send_idx, send_ids)
    _check(hidden.dtype == BF16 and weights.dtype == BF16, 'hidden and weights must be bf16')
    _check(hidden.dim() == 2 and selected.dim() == 2 and send_idx.dim() == 1 and send_ids.dim() == 2,
           'hidden, selected and send_ids must be 2-D, send_idx 1-D')
    n, h, k = send_idx.shape[0], hidden.shape[1], send_ids.shape[1]
    _check(selected.shape == (hidden.shape[0], k) and weights.shape == selected.shape
           and send_ids.shape[0] == n, 'selected/weights must be [tokens, k], send_ids [n, k]')
    payload = torch.empty((n, 2 * h + 3 * k), dtype=torch.uint8, device=hidden.device)
    if n:
        hid = hidden.contiguous()
        sel = selected.contiguous().long()
        w = weights.contiguous()
        si, sids = send_idx.contiguous().long(), send_ids.contiguous().long()
        err = torch.zeros(1, dtype=torch.int32, device=hidden.device)
        call('ferryb_pack_dispatch', ptr(hid), hid.shape[0], h, ptr(sel), ptr(w), k, ptr(si),
             ptr(sids), n, experts, ptr(payload), ptr(err), stream_ptr(hidden.device))
        _lib.check_device_error(err, 'pack_dispatch')
    return payload


def unpack_dispatch(raw, hidden, topk):
    """ferry/csrc/expert_ops.cpp:68-73 -> (x [m, H] bf16, w [m, k] bf16)."""
    require_cuda(raw)
    _check(raw.dtype == torch.uint8 and raw.dim() == 2 and raw.shape[1] == 2 * hidden + 3 * topk,
           f'raw must be uint8 [m, 2*hidden + 3*topk = {2 * hidden + 3 * topk}]')
    m = raw.shape[0]
    x = torch.empty((m, hidden), dtype=BF16, device=raw.device)
    w = torch.empty((m, topk), dtype=BF16, device=raw.device)
    if m:
        r = raw.contiguous()
        call('ferryb_unpack_dispatch', ptr(r), m, hidden, topk, ptr(x), ptr(w), stream_ptr(raw.device))
    return x, w


def reduce_partials(parts, rows, received, hidden, like):
    """ferry/csrc/expert_ops.cpp:76-83: float32 sum of the groups' outputs per
    receive row (in group order), returned as bf16 [received, hidden]."""
    require_cuda(like, *parts)
    _check(len(parts) == len(rows), 'parts and rows must have equal length')
    for p, r in zip(parts, rows):
        _check(p.dim() == 2 and p.shape[1] == hidden and p.shape[0] == r.numel(),
               'each part must be [len(rows[i]), hidden]')
    if not parts:
        return torch.zeros((received, hidden), dtype=BF16, device=like.device)
    src = torch.cat([p.to(BF16) for p in parts])
    keys = torch.cat([r.reshape(-1) for r in rows]).to(like.device)
    if src.shape[0] == 0:
        return torch.zeros((received, hidden), dtype=BF16, device=like.device)
    out = torch.empty((received, hidden), dtype=BF16, device=like.device)
    ws_bytes = _lib.lib().ferryb_segment_sum_workspace(src.shape[0], received)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=like.device)
    call('ferryb_reduce_partials', ptr(src), ptr(keys.long()), src.shape[0], received, hidden,
         ptr(out), ptr(ws), ws_bytes, stream_ptr(like.device))
    return out


def scatter_returned(returned, send_idx, tokens):
    """ferry/csrc/expert_ops.cpp:86-92: float32 sum of returned partials per
    token (in packet order), bf16 [tokens, hidden]."""
    require_cuda(returned, send_idx)
    _check(returned.dim() == 2 and send_idx.numel() == returned.shape[0],
           'returned must be [n, hidden] with one send_idx per row')
    hidden = returned.shape[1]
    if returned.shape[0] == 0:
        return torch.zeros((tokens, hidden), dtype=returned.dtype, device=returned.device)
    out = torch.empty((tokens, hidden), dtype=BF16, device=returned.device)
    ret = returned.contiguous().to(BF16)
    idx = send_idx.contiguous().long()
    ws_bytes = _lib.lib().ferryb_segment_sum_workspace(ret.shape[0], tokens)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=returned.device)
    call('ferryb_scatter_returned', ptr(ret), ptr(idx), ret.shape[0], tokens, hidden, ptr(out),
         ptr(ws), ws_bytes, stream_ptr(returned.device))
    return out.to(returned.dtype)


class H2DEngine:
    """ferry/csrc/expert_ops.cpp:97-142: pinned-pool -> cache-slot copies on
    copy-engine streams, per-slot events, last-use ordering."""

    def __init__(self, cache, pool, n_streams=1):
        require_cuda(cache)
        _check(pool.is_pinned() and pool.shape[1] == cache.shape[1],
               'pool must be pinned with the cache row size')
        self.cache, self.pool = cache, pool
        h = ctypes.c_void_p()
        call('ferryb_h2d_create', ptr(cache), cache.shape[0], cache.shape[1] * cache.element_size(),
             ptr(pool), pool.shape[0], int(n_streams), ctypes.byref(h))
        self._h = h

    def _arr(self, values):
        return _lib.host_i64(values), len(values)

    def fetch(self, slots, keys):
        s, n = self._arr(slots)
        k, _ = self._arr(keys)
        call('ferryb_h2d_fetch', self._h, s, k, n)

    def wait_host(self, slots):
        s, n = self._arr(slots)
        call('ferryb_h2d_wait_host', self._h, s, n)

    def wait_device(self, slots):
        s, n = self._arr(slots)
        call('ferryb_h2d_wait_device', self._h, s, n, stream_ptr(self.cache.device))

    def mark_used(self, slots):
        s, n = self._arr(slots)
        call('ferryb_h2d_mark_used', self._h, s, n, stream_ptr(self.cache.device))

    def synchronize(self):
        call('ferryb_h2d_synchronize', self._h)

    @property
    def copies(self):
        return int(_lib.lib().ferryb_h2d_copies(self._h))

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            _lib.lib().ferryb_h2d_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
