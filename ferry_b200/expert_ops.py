"""Drop-in for the reference's native module ``ferry_expert_ops``
(ferry/csrc/expert_ops.cpp:144-157): same function names, argument meaning
and error behaviour (RuntimeError on bad input), backed by libferryb's sm_100a
kernels through the C ABI.  Outputs are allocated by the torch caching
allocator; inputs are borrowed.
"""
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
