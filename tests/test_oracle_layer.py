"""The oracle's end-to-end layer (oracle/layer.py) is self-consistent: with R
emulated ranks every token's output equals sum_j w_j expert_j(x) computed
densely (BF16 tolerance), and the fetch counts follow the plan."""
import numpy as np
import pytest
import torch

from oracle import expert_ops as ops
from oracle.layer import OracleRuntime
from oracle import planner as op
from tests.tolerance import assert_bf16_close


class _Spec:
    def __init__(self, layers, experts, topk, hidden, inter):
        self.layers, self.experts, self.topk = layers, experts, topk
        self.hidden, self.intermediate = hidden, inter
        self.expert_elements = 3 * hidden * inter


@pytest.mark.parametrize('world', [1, 2, 3])
def test_oracle_layer_matches_dense(world):
    spec = _Spec(2, 16, 4, 64, 32)
    g = torch.Generator().manual_seed(world)
    pool = (torch.randn(spec.layers * spec.experts, spec.expert_elements, generator=g) * 0.05).to(torch.bfloat16)
    masks = np.asarray([1 << r for r in range(world)], np.int64)
    seconds = np.ones(world)
    lut = op.build_lut(spec.experts, world, masks, seconds)
    caps = [14] * world
    orc = OracleRuntime(spec, pool, caps, 'ferry', masks, seconds, lut)
    T = 6
    for step in range(4):
        layer = step % 2
        xs = [torch.randn(T, spec.hidden, generator=g).to(torch.bfloat16) for _ in range(world)]
        gate = (torch.randn(spec.experts, spec.hidden, generator=g) * 0.05).to(torch.bfloat16)
        routed = [ops.route_qwen3(x, gate, spec.topk) for x in xs]
        outs, fetches, dest = orc.execute(layer, xs, [r[0] for r in routed], [r[1] for r in routed])
        for r in range(world):
            sel, w, _ = routed[r]
            dense = torch.zeros(T, spec.hidden)
            for t in range(T):
                for j in range(spec.topk):
                    e = int(sel[t, j])
                    y = ops.expert_forward(xs[r][t:t + 1], pool[layer * spec.experts + e],
                                           spec.hidden, spec.intermediate)
                    dense[t] += (y.float() * w[t, j].float()).to(torch.bfloat16).float()[0]
            assert_bf16_close(outs[r], dense.to(torch.bfloat16), f'rank {r} step {step}')
