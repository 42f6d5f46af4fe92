"""Kernel 5 (tcgen05 grouped SwiGLU GEMM) against the CPU oracle of
ferry/csrc/expert_ops.cpp:16-45 and, where it was built, the reference's own
extension running on the same GPU."""
import pytest
import torch

from oracle import expert_ops as ref_ops
from oracle.build_ref import load_ref
from tests.tolerance import assert_bf16_close

pytestmark = pytest.mark.gpu


def _case(hidden, inter, slots, sizes, n_input, topk, seed):
    g = torch.Generator().manual_seed(seed)
    cache = (torch.randn(slots, 3 * hidden * inter, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(n_input, hidden, generator=g).to(torch.bfloat16)
    w = torch.rand(n_input, topk, generator=g).to(torch.bfloat16)
    slot_ids, rows, cols = [], [], []
    for i, n in enumerate(sizes):
        slot_ids.append(int(torch.randint(0, slots, (1,), generator=g)))
        r = torch.randperm(n_input, generator=g)[:n].sort().values if n <= n_input else \
            torch.randint(0, n_input, (n,), generator=g)
        rows.append(r.long())
        cols.append(torch.randint(0, topk, (n,), generator=g).long())
    return cache, x, w, slot_ids, rows, cols


CASES = [
    # hidden, inter, slots, group sizes, tokens, topk
    (256, 128, 3, [1, 5, 17, 3], 40, 4),
    (256, 256, 4, [16, 32, 64, 128, 130, 1, 0, 200], 256, 8),
    (2048, 768, 6, [1, 2, 3, 4, 9, 14, 33, 64], 64, 8),      # Qwen3 decode shape
    (2048, 1408, 3, [6, 1, 16, 11], 16, 6),                  # DeepSeek-V2-Lite shape
]


@pytest.mark.parametrize('case', CASES, ids=lambda c: f'H{c[0]}_I{c[1]}_n{sum(c[3])}')
def test_execute_experts_matches_oracle(case):
    from ferry_b200 import expert_ops
    hidden, inter, slots, sizes, n_input, topk = case
    cache, x, w, slot_ids, rows, cols = _case(hidden, inter, slots, sizes, n_input, topk, 7)
    want = ref_ops.execute_experts(cache, x, w, slot_ids, rows, cols, hidden, inter)
    dev = torch.device('cuda', 0)
    got = expert_ops.execute_experts(cache.to(dev), x.to(dev), w.to(dev), slot_ids,
                                     [r.to(dev) for r in rows], [c.to(dev) for c in cols],
                                     hidden, inter)
    torch.cuda.synchronize()
    assert len(got) == len(want)
    for i, (a, b) in enumerate(zip(got, want)):
        assert_bf16_close(a.cpu(), b, f'group {i} (n={sizes[i]})')


def test_execute_experts_matches_reference_extension():
    ref = load_ref()
    if ref is None:
        pytest.skip('reference extension not built (oracle/build_ref.py)')
    from ferry_b200 import expert_ops
    hidden, inter, slots, sizes, n_input, topk = CASES[2]
    cache, x, w, slot_ids, rows, cols = _case(hidden, inter, slots, sizes, n_input, topk, 11)
    dev = torch.device('cuda', 0)
    args = (cache.to(dev), x.to(dev), w.to(dev), slot_ids, [r.to(dev) for r in rows],
            [c.to(dev) for c in cols], hidden, inter)
    want = ref.execute_experts(*args)
    got = expert_ops.execute_experts(*args)
    for i, (a, b) in enumerate(zip(got, want)):
        assert_bf16_close(a, b, f'group {i}')
