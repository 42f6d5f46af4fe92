"""Model geometry of the two MoE families FERRY serves (ferry/model.py:24-70).

ModelSpec and read_spec keep the reference's fields and rules (MoE layer
selection, expert row size, the global cache budget split).  QWEN3_30B_A3B
and DEEPSEEK_V2_LITE are the benchmark's two models (no checkpoint files
are available here; weights are random-initialised by ferry_b200.workload).
"""
import json
from dataclasses import dataclass
from pathlib import Path

import torch


@dataclass(frozen=True)
class ModelSpec:
    model_type: str
    moe_layers: tuple      # decoder-layer indices that hold routed experts
    experts: int           # routed experts per MoE layer
    topk: int
    hidden: int
    intermediate: int      # routed-expert intermediate size
    shared_intermediate: int = 0  # DeepSeek-V2 shared experts as one MLP (n_shared * moe_intermediate)

    @property
    def layers(self):
        return len(self.moe_layers)

    @property
    def expert_elements(self):
        return 3 * self.hidden * self.intermediate

    @property
    def expert_bytes(self):
        return 2 * self.expert_elements

    def cache_slots(self, cache_ratio, world):
        """Global budget floor(layers * experts * ratio) split evenly, lower ranks
        taking the remainder (ferry/model.py:45-48)."""
        total = int(self.layers * self.experts * cache_ratio)
        return [total // world + (r < total % world) for r in range(world)]


def spec_from_config(c):
    """ferry/model.py:51-70 on a config dict."""
    kind = c['model_type']
    n = c['num_hidden_layers']
    if kind == 'qwen3_moe':
        step = c.get('decoder_sparse_step', 1)
        dense = set(c.get('mlp_only_layers') or [])
        layers = tuple(i for i in range(n) if i not in dense and (i + 1) % step == 0)
        # transformers 5 writes the expert count as num_local_experts
        experts = c['num_experts'] if 'num_experts' in c else c['num_local_experts']
    elif kind == 'deepseek_v2':
        first = c['first_k_dense_replace']
        freq = c.get('moe_layer_freq', 1)
        layers = tuple(i for i in range(n) if i >= first and i % freq == 0)
        experts = c['n_routed_experts']
        if c.get('topk_method', 'greedy') != 'greedy':
            raise NotImplementedError('only greedy top-k routing is supported for DeepSeek-V2')
    else:
        raise NotImplementedError(f'unsupported model_type {kind}')
    shared = (c.get('n_shared_experts') or 0) * c['moe_intermediate_size'] if kind == 'deepseek_v2' else 0
    return ModelSpec(kind, layers, experts, c['num_experts_per_tok'], c['hidden_size'],
                     c['moe_intermediate_size'], shared)


def pack_expert(gate_w, up_w, down_w):
    """One expert (or shared-expert MLP) as a cache/pool row: [gate I x H | up
    I x H | down H x I] of the nn.Linear weights (ferry/model.py:88)."""
    return torch.cat([gate_w.reshape(-1), up_w.reshape(-1), down_w.reshape(-1)]).to(torch.bfloat16)


def read_spec(model_path):
    return spec_from_config(json.loads((Path(model_path) / 'config.json').read_text()))


# The benchmark's configs 1/3/4 (Qwen3-30B-A3B) and 0/2 (DeepSeek-V2-Lite).
# (public model configs; the full-model harness builds them with random weights)
QWEN3_30B_A3B = dict(model_type='qwen3_moe', num_hidden_layers=48, num_experts=128,
                     num_experts_per_tok=8, hidden_size=2048, moe_intermediate_size=768,
                     intermediate_size=6144, norm_topk_prob=True, decoder_sparse_step=1,
                     mlp_only_layers=[], num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                     vocab_size=151936, max_position_embeddings=262144, rms_norm_eps=1e-6,
                     rope_theta=10000000.0, hidden_act='silu', tie_word_embeddings=False)
DEEPSEEK_V2_LITE = dict(model_type='deepseek_v2', num_hidden_layers=27, n_routed_experts=64,
                        num_experts_per_tok=6, hidden_size=2048, moe_intermediate_size=1408,
                        intermediate_size=10944, first_k_dense_replace=1, moe_layer_freq=1,
                        n_shared_experts=2, routed_scaling_factor=1.0, topk_method='greedy',
                        norm_topk_prob=False, n_group=1, topk_group=1, kv_lora_rank=512,
                        q_lora_rank=None, qk_rope_head_dim=64, qk_nope_head_dim=128, v_head_dim=128,
                        num_attention_heads=16, num_key_value_heads=16, vocab_size=102400,
                        max_position_embeddings=163840, rms_norm_eps=1e-6, rope_theta=10000.0,
                        hidden_act='silu', tie_word_embeddings=False)
