"""The allocation-free routed-expert entry point (ferryb_execute_experts_noalloc).

Some callers cannot allocate device memory -- a host application that has
already given the whole GPU to its own memory pool, or a plugin reached through
a C binding without a device allocator.  For them the library keeps a fixed
4 MiB scratch array of its own.  This test calls that entry point through the
C ABI twice in a row (different inputs, so the second call runs on the first
call's leftovers in the shared array) and compares each result with the
workspace-based ferryb_execute_experts within the BF16 tolerance; it also
checks that an oversized call is refused with a clear error.  The file is named
to be collected last.
"""

import pytest
import torch

from ferry_b200 import _lib
from tests.tolerance import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = torch.device('cuda', 0)


def _inputs(seed, hidden, inter, slots, sizes, n_input, topk):
    g = torch.Generator().manual_seed(seed)
    cache = (torch.randn(slots, 3 * hidden * inter, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    x = torch.randn(n_input, hidden, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.rand(n_input, topk, generator=g).to(torch.bfloat16).to(DEV)
    slot_ids = [int(torch.randint(0, slots, (1,), generator=g)) for _ in sizes]
    rows = torch.cat([torch.randint(0, n_input, (n,), generator=g) for n in sizes]).to(DEV)
    cols = torch.cat([torch.randint(0, topk, (n,), generator=g) for n in sizes]).to(DEV)
    return cache, x, w, slot_ids, rows, cols


def _with_workspace(cache, x, w, slot_ids, sizes, rows, cols, hidden, inter):
    lib = _lib.lib()
    total = sum(sizes)
    out = torch.empty((total, hidden), dtype=torch.bfloat16, device=DEV)
    ws_bytes = lib.ferryb_execute_experts_workspace(total, len(sizes), hidden, inter)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    _lib.call('ferryb_execute_experts', _lib.ptr(cache), cache.shape[0], _lib.ptr(x), x.shape[0],
              _lib.ptr(w), w.shape[1], _lib.host_i64(slot_ids), _lib.host_i64(sizes), len(sizes),
              _lib.ptr(rows), _lib.ptr(cols), hidden, inter, _lib.ptr(out), _lib.ptr(ws), ws_bytes,
              _lib.stream_ptr(DEV))
    return out


def _no_alloc(cache, x, w, slot_ids, sizes, rows, cols, hidden, inter):
    total = sum(sizes)
    out = torch.empty((total, hidden), dtype=torch.bfloat16, device=DEV)
    _lib.call('ferryb_execute_experts_noalloc', _lib.ptr(cache), cache.shape[0], _lib.ptr(x),
              x.shape[0], _lib.ptr(w), w.shape[1], _lib.host_i64(slot_ids), _lib.host_i64(sizes),
              len(sizes), _lib.ptr(rows), _lib.ptr(cols), hidden, inter, _lib.ptr(out),
              _lib.stream_ptr(DEV))
    return out


CALLS = [
    # hidden, inter, slots, group sizes, tokens, topk  (a Qwen3-shaped decode call)
    (2048, 768, 4, [3, 17, 1, 64, 9], 64, 8),
    (2048, 768, 3, [40, 2, 5], 48, 8),
]


def test_noalloc_matches_workspace_entry_point_twice():
    torch.cuda.set_device(DEV)
    for i, (hidden, inter, slots, sizes, n_input, topk) in enumerate(CALLS):
        cache, x, w, slot_ids, rows, cols = _inputs(100 + i, hidden, inter, slots, sizes, n_input, topk)
        want = _with_workspace(cache, x, w, slot_ids, sizes, rows, cols, hidden, inter)
        got = _no_alloc(cache, x, w, slot_ids, sizes, rows, cols, hidden, inter)
        torch.cuda.synchronize()
        assert_bf16_close(got.cpu(), want.cpu(), f'call {i}')


def test_noalloc_refuses_calls_beyond_its_scratch():
    torch.cuda.set_device(DEV)
    limit = _lib.lib().ferryb_execute_experts_noalloc_limit()
    assert limit == 4 << 20
    hidden, inter, topk = 2048, 768, 8
    sizes = [2048]  # 2048 routes x (2048 + 768) bf16 ~ 11.5 MB > 4 MiB
    cache = torch.zeros((1, 3 * hidden * inter), dtype=torch.bfloat16, device=DEV)
    x = torch.zeros((16, hidden), dtype=torch.bfloat16, device=DEV)
    w = torch.zeros((16, topk), dtype=torch.bfloat16, device=DEV)
    rows = torch.zeros(2048, dtype=torch.int64, device=DEV)
    cols = torch.zeros(2048, dtype=torch.int64, device=DEV)
    with pytest.raises(_lib.FerrybError, match='scratch'):
        _no_alloc(cache, x, w, [0], sizes, rows, cols, hidden, inter)
