"""The full-model harness (transformers 5.5 models, MoE blocks hooked into
OffloadRuntime.forward) on tiny random models: prefill logits of the hooked
model against the same model running transformers' own expert modules with
the same weights (different bf16 rounding points, so a tolerance), then a
short greedy decode through the KV cache."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def _tiny(kind):
    from ferry_b200.model import DEEPSEEK_V2_LITE, QWEN3_30B_A3B
    if kind == 'qwen3':
        return dict(QWEN3_30B_A3B, num_hidden_layers=3, num_experts=16, num_experts_per_tok=4, hidden_size=256,
                    moe_intermediate_size=128, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=64, vocab_size=512)
    return dict(DEEPSEEK_V2_LITE, num_hidden_layers=3, n_routed_experts=16, num_experts_per_tok=4,
                hidden_size=256, moe_intermediate_size=128, intermediate_size=512, num_attention_heads=4,
                num_key_value_heads=4, kv_lora_rank=64, qk_rope_head_dim=32, qk_nope_head_dim=32,
                v_head_dim=32, vocab_size=512)


@pytest.mark.parametrize('kind', ['qwen3', 'deepseek'])
def test_hooked_model_matches_transformers_experts(kind):
    from ferry_b200.harness import (build_model, expert_pool_from_model, generate, install_hooks,
                                    shared_expert_rows)
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    cfg = _tiny(kind)
    model, spec = build_model(cfg, DEV, seed=3, keep_experts=True)
    # random-init gates give near-uniform routing; scale them up so top-k is decisive
    with torch.no_grad():
        for idx in spec.moe_layers:
            model.model.layers[idx].mlp.gate.weight.mul_(20.0)
    pool = expert_pool_from_model(model, spec)
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randint(0, cfg['vocab_size'], (2, 24), generator=g, device=DEV)
    with torch.no_grad():
        want = model(input_ids=x).logits.float()
    caps = spec.cache_slots(0.7, 1)  # every expert of a prefill layer fits (16 of 33 slots)
    rt = OffloadRuntime(spec, pool, caps, 'ferry', Topology.uniform(1, spec.experts),
                        norm_topk_prob=bool(cfg['norm_topk_prob']),
                        routed_scaling_factor=float(cfg.get('routed_scaling_factor', 1.0)),
                        shared_experts=shared_expert_rows(model, spec))
    install_hooks(model, spec, rt)
    with torch.no_grad():
        got = model(input_ids=x).logits.float()
    rel = (got - want).abs().max() / want.abs().max()
    agree = (got.argmax(-1) == want.argmax(-1)).float().mean()
    assert rel < 0.05, f'max |diff| / max |ref| = {rel:.4f}'
    assert agree > 0.9, f'argmax agreement {agree:.3f}'
    tokens, times = generate(model, x, 6)
    assert tokens.shape == (2, 6) and len(times) == 6 and times[-1] >= times[0] > 0
    assert rt.fetches_per_rank[0] > 0
    rt.close()


def _oracle_hooks(model, spec, cfg, orc, shared_rows):
    """The reference's MoE hooks (ferry/model.py:137-158) over the CPU oracle of
    OffloadRuntime.execute: the hook's router, the runtime, and (DeepSeek-V2)
    the shared expert added in bf16."""
    from oracle import expert_ops as ops
    H, I = spec.hidden, spec.shared_intermediate
    for layer, idx in enumerate(spec.moe_layers):
        mlp = model.model.layers[idx].mlp
        gate = mlp.gate.weight.detach().cpu()
        shared = None if shared_rows is None else shared_rows[layer].cpu()

        def forward(hidden_states, _layer=layer, _gate=gate, _shared=shared):
            shape = hidden_states.shape
            x = hidden_states.reshape(-1, shape[-1]).cpu()
            if spec.model_type == 'qwen3_moe':
                sel, w, _ = ops.route_qwen3(x, _gate, spec.topk, bool(cfg['norm_topk_prob']))
            else:
                sel, w, _ = ops.route_deepseek(x, _gate, spec.topk, float(cfg['routed_scaling_factor']))
            y = orc.execute(_layer, [x], [sel], [w])[0][0]
            if _shared is not None:  # transformers' DeepseekV2MLP, as the reference hook adds it
                s = ops.shared_expert(x, _shared[:I * H].view(I, H), _shared[I * H:2 * I * H].view(I, H),
                                      _shared[2 * I * H:].view(H, I))
                y = (y.float() + s.float()).to(torch.bfloat16)
            return y.to(hidden_states.device).view(shape)
        mlp.forward = forward


@pytest.mark.parametrize('kind', ['qwen3', 'deepseek'])
def test_hooked_model_final_hidden_states_match_reference_hooks(kind):
    """The whole model with its MoE blocks on this runtime against the same
    model with the reference's hooks over the CPU oracle of its runtime (same
    weights, same cache policy), on a prefill and three decode steps
    (teacher-forced tokens, KV cache).  Every decoder layer's output hidden
    states, up to the last one (the final hidden states the model's norm
    reads), are within the north star's BF16 tolerance: max abs <= 2e-2 and
    <= 1e-2 of max |ref|.  The final RMSNorm then scales the residual stream by
    1/rms (about 7x in these models), so one bf16 step of its output at values
    in [2, 8) is 0.016-0.031; its output is held to the relative bound
    (<= 1e-2 of max |ref|)."""
    from transformers import DynamicCache

    from ferry_b200.harness import build_model, expert_pool_from_model, install_hooks, shared_expert_rows
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from oracle.layer import OracleRuntime
    from tests.tolerance import REL_TOL, assert_bf16_close, bf16_report
    cfg = _tiny(kind)
    model, spec = build_model(cfg, DEV, seed=3, keep_experts=True)
    with torch.no_grad():
        for idx in spec.moe_layers:
            model.model.layers[idx].mlp.gate.weight.mul_(20.0)
    pool = expert_pool_from_model(model, spec)
    shared = shared_expert_rows(model, spec)
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randint(0, cfg['vocab_size'], (2, 24), generator=g, device=DEV)
    steps = torch.randint(0, cfg['vocab_size'], (3, 2, 1), generator=g, device=DEV)
    caps = spec.cache_slots(0.7, 1)
    topo = Topology.uniform(1, spec.experts)
    pre = {}
    model.model.norm.register_forward_hook(lambda m, i, o: pre.__setitem__('x', i[0].detach().clone()))

    def run():
        """Per forward: (decoder layer outputs ..., final hidden states before
        the norm, after the norm)."""
        cache = DynamicCache(config=model.config)
        outs = []
        with torch.no_grad():
            for i, ids in enumerate([x] + list(steps)):
                o = model.model(input_ids=ids, past_key_values=cache, use_cache=True,
                                output_hidden_states=True)
                outs.append(list(o.hidden_states[1:-1]) + [pre['x'], o.last_hidden_state])
        return outs

    rt = OffloadRuntime(spec, pool, caps, 'ferry', topo, norm_topk_prob=bool(cfg['norm_topk_prob']),
                        routed_scaling_factor=float(cfg.get('routed_scaling_factor', 1.0)),
                        shared_experts=shared)
    install_hooks(model, spec, rt)
    got = run()
    rt.close()
    orc = OracleRuntime(spec, pool, caps, 'ferry', topo.masks, topo.seconds, topo.lut)
    _oracle_hooks(model, spec, cfg, orc, shared)
    want = run()
    for i, (a, b) in enumerate(zip(got, want)):
        for j, (p, q) in enumerate(zip(a[:-1], b[:-1])):
            assert_bf16_close(p.float().cpu(), q.float().cpu(), f'{kind} forward {i}, hidden states {j}')
        err, scale = bf16_report(a[-1], b[-1])
        assert err <= REL_TOL * scale, f'{kind} forward {i}, after the final norm: {err:.3e} vs {scale:.3e}'
