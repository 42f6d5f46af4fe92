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
