"""The reference's packet and reduction ops (ferry/csrc/expert_ops.cpp:50-92:
pack_dispatch, unpack_dispatch, reduce_partials, scatter_returned) on the GPU
against the CPU oracle, bit-exact, at packet strides 2H + 3k of every
alignment (k = 8 Qwen3, 6 DeepSeek-V2, 4, 3), with -1-padded packets, empty
inputs and repeated destination rows."""
import pytest
import torch

from oracle import expert_ops as ref_ops

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def _packets(T, H, K, E, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g).to(torch.bfloat16)
    # packets: a random subset of tokens, each with a random subset of its ids, -1 padded
    idx = torch.randperm(T, generator=g)[:max(1, T // 2)].sort().values
    ids = torch.full((idx.numel(), K), -1, dtype=torch.int64)
    for i, t in enumerate(idx.tolist()):
        keep = sel[t][torch.randperm(K, generator=g)[:1 + i % K]].sort().values
        ids[i, :keep.numel()] = keep
    return x, sel, w, idx, ids


@pytest.mark.parametrize('H,K,E', [(2048, 8, 128), (2048, 6, 64), (256, 4, 16), (256, 3, 16)])
def test_pack_unpack_bit_exact(H, K, E):
    from ferry_b200 import expert_ops as ops
    x, sel, w, idx, ids = _packets(40, H, K, E, seed=H + K)
    want = ref_ops.pack_dispatch(x, sel, w, idx, ids, E)
    got = ops.pack_dispatch(x.to(DEV), sel.to(DEV), w.to(DEV), idx.to(DEV), ids.to(DEV), E)
    assert got.shape == want.shape and torch.equal(got.cpu(), want)
    gx, gw = ops.unpack_dispatch(got, H, K)
    wx, ww = ref_ops.unpack_dispatch(want, H, K)
    assert torch.equal(gx.cpu(), wx) and torch.equal(gw.cpu(), ww)
    # a packet view that starts at an odd row (base alignment follows the stride)
    gx1, gw1 = ops.unpack_dispatch(got[1:], H, K)
    assert torch.equal(gx1.cpu(), wx[1:]) and torch.equal(gw1.cpu(), ww[1:])


def test_pack_empty():
    from ferry_b200 import expert_ops as ops
    x, sel, w, _, _ = _packets(4, 256, 4, 16, seed=1)
    got = ops.pack_dispatch(x.to(DEV), sel.to(DEV), w.to(DEV), torch.zeros(0, dtype=torch.int64, device=DEV),
                            torch.zeros((0, 4), dtype=torch.int64, device=DEV), 16)
    assert got.shape == (0, 2 * 256 + 12)


@pytest.mark.parametrize('received,H', [(37, 2048), (5, 256), (0, 256)])
def test_reduce_and_scatter_bit_exact(received, H):
    from ferry_b200 import expert_ops as ops
    g = torch.Generator().manual_seed(received + H)
    parts, rows = [], []
    for n in (3, 11, 1, 20):
        if received == 0:
            break
        rows.append(torch.randint(0, received, (n,), generator=g))  # repeated rows allowed
        parts.append(torch.randn(n, H, generator=g).to(torch.bfloat16))
    want = ref_ops.reduce_partials(parts, rows, received, H)
    got = ops.reduce_partials([p.to(DEV) for p in parts], [r.to(DEV) for r in rows], received, H,
                              torch.empty(1, H, dtype=torch.bfloat16, device=DEV))
    assert torch.equal(got.cpu(), want)
    tokens = 9
    send_idx = torch.randint(0, tokens, (received,), generator=g)
    want_o = ref_ops.scatter_returned(want, send_idx, tokens)
    got_o = ops.scatter_returned(got, send_idx.to(DEV), tokens)
    assert torch.equal(got_o.cpu(), want_o)
