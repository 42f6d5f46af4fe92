"""The fused per-layer executor (kernels 1-5 chained by ferryb_layer_*) on one
GPU against the CPU oracle of the reference's OffloadRuntime.execute:
cache decisions bit-exact, layer outputs within the BF16 tolerance."""
import numpy as np
import pytest
import torch

from oracle import expert_ops as ref_ops
from oracle.layer import OracleRuntime
from tests.tolerance import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = torch.device('cuda', 0)


def _spec(layers, experts, topk, hidden, inter, kind='qwen3_moe'):
    from ferry_b200.model import ModelSpec
    return ModelSpec(kind, tuple(range(layers)), experts, topk, hidden, inter)


def _setup(spec, caps, seed=0, policy='ferry', score='frequency', sync_fetch=False):
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import cpu_pool, zipf_bias
    torch.manual_seed(seed)
    pool = cpu_pool(spec, spec.layers, seed).pin_memory()
    topo = Topology.uniform(len(caps), spec.experts)
    rt = OffloadRuntime(spec, pool, caps, policy, topo, eviction_score=score, sync_fetch=sync_fetch)
    orc = OracleRuntime(spec, pool, caps, policy, topo.masks, topo.seconds, topo.lut, score=score)
    g = torch.Generator().manual_seed(seed + 7)
    gates = [(torch.randn(spec.experts, spec.hidden, generator=g) * 0.02).to(torch.bfloat16)
             for _ in range(spec.layers)]
    biases = [zipf_bias(spec.experts, 1.1, g) for _ in range(spec.layers)]
    return rt, orc, gates, biases, g


CASES = [
    # layers, experts, topk, hidden, inter, tokens, capacity
    (3, 16, 4, 256, 128, 8, 10),
    (2, 128, 8, 2048, 768, 64, 180),     # Qwen3 layer shape, decode batch 64
    (2, 64, 6, 2048, 1408, 16, 60),      # DeepSeek-V2-Lite layer shape
]


@pytest.mark.parametrize('sync_fetch', [False, True], ids=['flags', 'sync_fetch'])
@pytest.mark.parametrize('case', CASES, ids=lambda c: f'E{c[1]}_k{c[2]}_H{c[3]}_T{c[5]}')
def test_execute_matches_oracle(case, sync_fetch):
    """Both fetch modes: readiness flags waited on by the GEMM (default) and
    sync_fetch (every copy waited for by the stream first; smoke() and
    profiler runs use it)."""
    layers, E, K, H, I, T, cap = case
    spec = _spec(layers, E, K, H, I)
    rt, orc, gates, biases, g = _setup(spec, [cap], sync_fetch=sync_fetch)
    for step in range(3 * layers):
        layer = step % layers
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        sel, w, _ = ref_ops.route_qwen3(x, gates[layer], K, True, biases[layer])
        want, fetches, dest = orc.execute(layer, [x], [sel], [w])
        got = rt.execute(layer, x.to(DEV), sel.to(DEV), w.to(DEV), None)
        torch.cuda.synchronize()
        assert_bf16_close(got.cpu(), want[0], f'step {step}')
        np.testing.assert_array_equal(rt.controller.slots, orc.ctl.slots, err_msg=f'step {step}')
        np.testing.assert_array_equal(rt.controller.owner, orc.ctl.owner)
        np.testing.assert_array_equal(rt.controller.last, orc.ctl.last)
    np.testing.assert_array_equal(rt.fetches_per_rank, orc.fetches_per_rank)
    assert rt.h2d.copies == int(orc.fetches_per_rank[0])
    rt.close()


def test_forward_router_and_layer():
    """Kernel 1 in the loop: routing against a torch GPU router, then the layer
    output against the oracle fed the kernel's own routing."""
    layers, E, K, H, I, T, cap = CASES[1]
    spec = _spec(layers, E, K, H, I)
    rt, orc, gates, biases, g = _setup(spec, [cap], seed=3)
    n_mismatch = 0
    for step in range(4):
        layer = step % layers
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        sel_out = torch.empty((T, K), dtype=torch.int64, device=DEV)
        w_out = torch.empty((T, K), dtype=torch.bfloat16, device=DEV)
        got = rt.forward(layer, x.to(DEV), gates[layer].to(DEV), biases[layer].to(DEV), sel_out, w_out)
        torch.cuda.synchronize()
        # torch reference of the hook's router on the same GPU (cuBLAS bf16 logits)
        logits = torch.nn.functional.linear(x.to(DEV), gates[layer].to(DEV),
                                            biases[layer].to(DEV).to(torch.bfloat16))
        probs = torch.softmax(logits.float(), -1)
        ref_w, ref_sel = torch.topk(probs, K, -1)
        ref_w = ref_w / ref_w.sum(-1, keepdim=True)
        # same expert sets except where probabilities tie within rounding
        for t in range(T):
            a, b = set(sel_out[t].tolist()), set(ref_sel[t].tolist())
            if a != b:
                n_mismatch += 1
                kth = probs[t].sort(descending=True).values
                assert (kth[K - 1] - kth[K]).abs().item() < 1e-3, f'token {t}: {a} vs {b}'
        same = (sel_out.sort(-1).values == ref_sel.sort(-1).values).all(-1)
        assert_bf16_close(w_out[same].float().sort(-1).values.cpu(),
                          ref_w[same].float().sort(-1).values.cpu(), 'router weights')
        want, _, _ = orc.execute(layer, [x], [sel_out.cpu()], [w_out.cpu()])
        assert_bf16_close(got.cpu(), want[0], f'forward step {step}')
        np.testing.assert_array_equal(rt.controller.slots, orc.ctl.slots)
    assert n_mismatch <= T  # near-ties only
    rt.close()


def test_reset_and_counters():
    layers, E, K, H, I, T, cap = CASES[0]
    spec = _spec(layers, E, K, H, I)
    rt, orc, gates, biases, g = _setup(spec, [cap], seed=5)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    sel, w, _ = ref_ops.route_qwen3(x, gates[0], K, True, biases[0])
    rt.execute(0, x.to(DEV), sel.to(DEV), w.to(DEV), None)
    assert rt.event == 1 and rt.h2d.copies > 0
    rt.reset()
    assert rt.event == 0 and rt.h2d.copies == 0
    assert (rt.controller.slots == -1).all()
    got = rt.execute(0, x.to(DEV), sel.to(DEV), w.to(DEV), None)
    want, _, _ = orc.execute(0, [x], [sel], [w])
    assert_bf16_close(got.cpu(), want[0], 'after reset')
    rt.close()


def test_forward_deepseek_shared_experts():
    """DeepSeek-V2-Lite MoE block through forward(): the greedy softmax router in
    kernel 1, routed experts, and the two shared experts (one 2816-wide MLP) run
    in the copies' shadow and added as transformers does (bf16 add); execute()
    leaves the shared expert out, as the reference's execute does."""
    from ferry_b200.model import ModelSpec, pack_expert
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import cpu_pool
    E, K, H, I, Is, T, cap, layers = 64, 6, 2048, 1408, 2816, 16, 60, 2
    spec = ModelSpec('deepseek_v2', tuple(range(layers)), E, K, H, I, Is)
    pool = cpu_pool(spec, layers, 11).pin_memory()
    g = torch.Generator().manual_seed(12)
    gates = [(torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16) for _ in range(layers)]
    shared = [[(torch.randn(*shp, generator=g) * 0.02).to(torch.bfloat16)
               for shp in ((Is, H), (Is, H), (H, Is))] for _ in range(layers)]
    rows = [pack_expert(*s).to(DEV) for s in shared]
    topo = Topology.uniform(1, E)
    rt = OffloadRuntime(spec, pool, [cap], 'ferry', topo, norm_topk_prob=False, shared_experts=rows)
    orc = OracleRuntime(spec, pool, [cap], 'ferry', topo.masks, topo.seconds, topo.lut)
    for step in range(4):
        layer = step % layers
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        sel_out = torch.empty((T, K), dtype=torch.int64, device=DEV)
        w_out = torch.empty((T, K), dtype=torch.bfloat16, device=DEV)
        got = rt.forward(layer, x.to(DEV), gates[layer].to(DEV), None, sel_out, w_out)
        torch.cuda.synchronize()
        routed, _, _ = orc.execute(layer, [x], [sel_out.cpu()], [w_out.cpu()])
        want = (routed[0].float() + ref_ops.shared_expert(x, *shared[layer]).float()).to(torch.bfloat16)
        assert_bf16_close(got.cpu(), want, f'forward+shared step {step}')
        np.testing.assert_array_equal(rt.controller.slots, orc.ctl.slots)
    # execute(): routed experts only
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    sel, w, _ = ref_ops.route_deepseek(x, gates[0].float(), K, 1.0, None)
    got = rt.execute(0, x.to(DEV), sel.to(DEV), w.to(DEV), None)
    torch.cuda.synchronize()
    want, _, _ = orc.execute(0, [x], [sel], [w])
    assert_bf16_close(got.cpu(), want[0], 'execute without shared')
    rt.close()


@pytest.mark.parametrize('policy,score', [('random', 'frequency'), ('ferry', 'probability')])
def test_execute_policies_and_scores(policy, score):
    """FERRY-Random (MT19937 draws, one rank) and the router-probability
    eviction score (probs_tail rows into the device history) through the full
    executor: decisions bit-exact, outputs within tolerance."""
    layers, E, K, H, I, T, cap = 3, 32, 4, 256, 128, 12, 20
    spec = _spec(layers, E, K, H, I)
    rt, orc, gates, biases, g = _setup(spec, [cap], seed=8, policy=policy, score=score)
    for step in range(3 * layers):
        layer = step % layers
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        sel, w, probs = ref_ops.route_qwen3(x, gates[layer], K, True, biases[layer])
        pt = probs if score == 'probability' else None
        want, _, _ = orc.execute(layer, [x], [sel], [w], [pt] if pt is not None else None)
        got = rt.execute(layer, x.to(DEV), sel.to(DEV), w.to(DEV), pt.to(DEV) if pt is not None else None)
        torch.cuda.synchronize()
        assert_bf16_close(got.cpu(), want[0], f'{policy}/{score} step {step}')
        np.testing.assert_array_equal(rt.controller.slots, orc.ctl.slots, err_msg=f'step {step}')
        np.testing.assert_array_equal(rt.controller.owner, orc.ctl.owner)
    np.testing.assert_array_equal(rt.fetches_per_rank, orc.fetches_per_rank)
    rt.close()


@pytest.mark.parametrize('E,K,T', [(256, 16, 1), (256, 8, 3), (16, 1, 5)])
def test_execute_edge_shapes(E, K, T):
    """Edge shapes: one token, the maximum of 256 experts (ids travel as
    uint8) and top-16, top-1."""
    layers, H, I = 2, 256, 128
    spec = _spec(layers, E, K, H, I)
    cap = min(layers * E, max(3 * K * T, E // 2))
    rt, orc, gates, biases, g = _setup(spec, [cap], seed=E + K + T)
    for step in range(4):
        layer = step % layers
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        sel, w, _ = ref_ops.route_qwen3(x, gates[layer], K, True, biases[layer])
        want, _, _ = orc.execute(layer, [x], [sel], [w])
        got = rt.execute(layer, x.to(DEV), sel.to(DEV), w.to(DEV), None)
        torch.cuda.synchronize()
        assert_bf16_close(got.cpu(), want[0], f'E{E} K{K} T{T} step {step}')
        np.testing.assert_array_equal(rt.controller.slots, orc.ctl.slots)
    rt.close()


def test_forward_probability_score():
    """The router in the loop with the probability eviction score: kernel 1
    writes each rank's router-probability tail into the history; the layer
    output matches the oracle fed the kernel's own routing (outputs do not
    depend on which experts were cached), and the cache stays consistent."""
    layers, E, K, H, I, T, cap = 2, 32, 4, 256, 128, 16, 24
    spec = _spec(layers, E, K, H, I)
    rt, orc, gates, biases, g = _setup(spec, [cap], seed=21, score='probability')
    for step in range(6):
        layer = step % layers
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        sel_out = torch.empty((T, K), dtype=torch.int64, device=DEV)
        w_out = torch.empty((T, K), dtype=torch.bfloat16, device=DEV)
        got = rt.forward(layer, x.to(DEV), gates[layer].to(DEV), biases[layer].to(DEV), sel_out, w_out)
        torch.cuda.synchronize()
        _, _, probs = ref_ops.route_qwen3(x, gates[layer], K, True, biases[layer])
        want, _, _ = orc.execute(layer, [x], [sel_out.cpu()], [w_out.cpu()], [probs])
        assert_bf16_close(got.cpu(), want[0], f'forward/probability step {step}')
        slots = rt.controller.slots[0]
        owner = rt.controller.owner
        held = slots[slots >= 0]
        assert len(set(held.tolist())) == held.size and (owner[held] == 0).all()
    rt.close()


def test_bench_configuration_matches_oracle():
    """The bench's own workload: the 48-layer Qwen3-30B-A3B MoE stack, 64 decode
    tokens, 1,843 cache slots (30 % global), Zipf(1.1) router bias, rho = 0.5
    hidden states, layer l routing x_l + out_(l-1), through forward() (router in
    kernel 1) for three decode steps.  The oracle is fed this runtime's routing
    and layer inputs, so that each of the 144 layers is compared on its own:
    cache decisions bit-exact, outputs within the BF16 tolerance.  The pool
    holds two layers' experts (key mod 256 rows, as bench.py --pool-layers 2)."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import SyntheticMoE
    spec = bench.qwen3_spec(48)
    T, caps = 64, spec.cache_slots(0.3, 1)
    assert caps == [1843]
    wl = SyntheticMoE(spec, seed=0, device=DEV, pool_layers=2)
    topo = Topology.uniform(1, spec.experts)
    rt = OffloadRuntime(spec, wl.pool, caps, 'ferry', topo)
    orc = OracleRuntime(spec, wl.pool, caps, 'ferry', topo.masks, topo.seconds, topo.lut)
    inputs = bench.make_inputs(spec, T, 1, [0], 3)[0]
    sel = torch.empty((T, spec.topk), dtype=torch.int64, device=DEV)
    w = torch.empty((T, spec.topk), dtype=torch.bfloat16, device=DEV)
    for step in range(3):
        prev = None
        for l in range(spec.layers):
            x = inputs[step][l].to(DEV)
            h = x if prev is None else x + prev
            prev = rt.forward(l, h, wl.gate[l], wl.bias[l], sel, w)
            want, _, _ = orc.execute(l, [h.cpu()], [sel.cpu()], [w.cpu()])
            assert_bf16_close(prev.cpu(), want[0], f'step {step} layer {l}')
        np.testing.assert_array_equal(rt.controller.slots, orc.ctl.slots, err_msg=f'step {step}')
        np.testing.assert_array_equal(rt.controller.owner, orc.ctl.owner)
        np.testing.assert_array_equal(rt.controller.last, orc.ctl.last)
    np.testing.assert_array_equal(rt.fetches_per_rank, orc.fetches_per_rank)
    rt.close()
