"""The harness's checkpoint loader (the reference's load, ferry/model.py:
73-122) on tiny random checkpoints written here (no GPU): the routed experts
must land in the pool rows exactly as the model holds them and every dense
parameter in the model, from sharded per-expert files (the Hugging Face
layout) and from one file of transformers 5's fused expert parameters;
Qwen3-MoE and DeepSeek-V2 (a dense first layer, shared experts)."""
import json

import pytest
import torch

from ferry_b200.harness import build_model, expert_pool_from_model, hf_config, load_checkpoint
from ferry_b200.model import DEEPSEEK_V2_LITE, QWEN3_30B_A3B


def _tiny(kind):
    if kind == 'qwen3':
        return dict(QWEN3_30B_A3B, num_hidden_layers=2, num_experts=4, num_experts_per_tok=2,
                    hidden_size=64, moe_intermediate_size=32, intermediate_size=128,
                    num_attention_heads=4, num_key_value_heads=2, head_dim=16, vocab_size=96,
                    max_position_embeddings=128)
    return dict(DEEPSEEK_V2_LITE, num_hidden_layers=3, n_routed_experts=4, num_experts_per_tok=2,
                n_shared_experts=1, hidden_size=64, moe_intermediate_size=32, intermediate_size=128,
                num_attention_heads=4, num_key_value_heads=4, kv_lora_rank=16, qk_rope_head_dim=8,
                qk_nope_head_dim=8, v_head_dim=16, vocab_size=96, max_position_embeddings=128)


def _write(model, spec, cfg, path, fused, drop=None):
    """The model as a checkpoint directory; per-expert tensors in two shards
    plus an index, or everything in one file with the fused parameters."""
    from safetensors.torch import save_file
    hf_config(cfg).save_pretrained(path)
    sd = {k: v.contiguous().clone() for k, v in model.state_dict().items()}
    if not fused:
        I = spec.intermediate
        for idx in spec.moe_layers:
            pre = f'model.layers.{idx}.mlp.experts.'
            gu, dn = sd.pop(pre + 'gate_up_proj'), sd.pop(pre + 'down_proj')
            for e in range(spec.experts):
                sd[f'{pre}{e}.gate_proj.weight'] = gu[e, :I].clone()
                sd[f'{pre}{e}.up_proj.weight'] = gu[e, I:].clone()
                sd[f'{pre}{e}.down_proj.weight'] = dn[e].clone()
    if drop:
        del sd[drop]
    if fused:
        save_file(sd, str(path / 'model.safetensors'))
        return
    names = sorted(sd)
    shards = {'model-00001-of-00002.safetensors': names[::2], 'model-00002-of-00002.safetensors': names[1::2]}
    for f, ns in shards.items():
        save_file({n: sd[n] for n in ns}, str(path / f))
    (path / 'model.safetensors.index.json').write_text(json.dumps(
        {'metadata': {}, 'weight_map': {n: f for f, ns in shards.items() for n in ns}}))


@pytest.mark.parametrize('fused', [False, True])
@pytest.mark.parametrize('kind', ['qwen3', 'deepseek'])
def test_load_checkpoint_matches_model(tmp_path, kind, fused):
    cfg = _tiny(kind)
    model, spec = build_model(cfg, 'cpu', seed=5, keep_experts=True)
    _write(model, spec, cfg, tmp_path, fused)
    loaded, spec2, pool = load_checkpoint(tmp_path, device='cpu')
    assert spec2 == spec
    assert torch.equal(pool, expert_pool_from_model(model, spec))
    want = {n: p for n, p in model.named_parameters() if '.mlp.experts.' not in n}
    got = dict(loaded.named_parameters())
    assert set(got) == set(want)
    assert all(torch.equal(got[n], want[n]) for n in want)
    for idx in spec.moe_layers:
        assert loaded.model.layers[idx].mlp.experts is None
    # the loaded model computes what the original does with its dense weights
    # (rotary buffers rebuilt on the device)
    x = torch.randint(0, cfg['vocab_size'], (1, 5))
    emb_a = loaded.model.embed_tokens(x)
    emb_b = model.model.embed_tokens(x)
    assert torch.equal(emb_a, emb_b)
    rot = [m for _, m in loaded.named_modules() if hasattr(m, 'inv_freq')]
    assert rot and all(not m.inv_freq.is_meta for m in rot)


def test_load_checkpoint_rejects_missing_tensors(tmp_path):
    cfg = _tiny('qwen3')
    model, spec = build_model(cfg, 'cpu', seed=5, keep_experts=True)
    (tmp_path / 'a').mkdir()
    _write(model, spec, cfg, tmp_path / 'a', fused=False, drop='model.layers.1.mlp.experts.3.up_proj.weight')
    with pytest.raises(ValueError, match='incomplete.*MoE layer 1, expert 3'):
        load_checkpoint(tmp_path / 'a', device='cpu')
    (tmp_path / 'b').mkdir()
    _write(model, spec, cfg, tmp_path / 'b', fused=False, drop='model.layers.0.self_attn.o_proj.weight')
    with pytest.raises(ValueError, match='dense parameters are missing'):
        load_checkpoint(tmp_path / 'b', device='cpu')


def test_runtime_expert_ops_names():
    """ferry/runtime.py:26-31's expert_ops() returns a module with the
    extension's six names."""
    from ferry_b200.runtime import expert_ops
    ops = expert_ops()
    for name in ('execute_experts', 'pack_dispatch', 'unpack_dispatch', 'reduce_partials',
                 'scatter_returned', 'H2DEngine'):
        assert callable(getattr(ops, name)), name
