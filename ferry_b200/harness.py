"""Full-model decode harness on transformers 5.5 with random-initialised
weights: the MoE blocks of a Qwen3-MoE or DeepSeek-V2 model run through
OffloadRuntime.forward (kernel 1 router, device planner, copy-engine expert
fetches, P2P dispatch/combine, tcgen05 grouped SwiGLU; DeepSeek-V2 shared
experts added in the combine), everything else is the model's own torch code.

It follows the reference's harness (ferry/model.py:73-158, scripts/run_cell.py
:48-76) with transformers 5.5 semantics: a MoE block's forward returns one
tensor, routed experts are one module of 3-D parameters (never materialised
here: they live in the pinned expert pool), and no checkpoint exists, so
parameters are N(0, 0.02) and norms 1.  One process per GPU: attention is
data-parallel (each rank decodes its own batch), experts expert-parallel.

Metrics (run_cell.py:150-154 semantics, CUDA events per rank, max over
ranks): TTFT = prefill + first token; TPOT = mean time per later token;
decode tokens/s = R * B * (new_tokens - 1) / (max_r last_r - max_r first_r).
"""
import time

import torch
import torch.distributed as dist

from .model import pack_expert, spec_from_config


def hf_config(cfg_dict, **overrides):
    """A transformers config object from a config dict (model.py's dicts)."""
    from transformers import DeepseekV2Config, Qwen3MoeConfig
    d = dict(cfg_dict, **overrides)
    cls = Qwen3MoeConfig if d['model_type'] == 'qwen3_moe' else DeepseekV2Config
    d.pop('model_type')
    return cls(**d)


def _rope_modules(model):
    return [(name, mod) for name, mod in model.named_modules() if hasattr(mod, 'inv_freq')]


def build_model(cfg_dict, device, seed=0, keep_experts=False, **overrides):
    """(model, spec): the model on `device`, without routed-expert parameters
    unless keep_experts (then transformers' own expert modules are kept, e.g.
    to compare against)."""
    from transformers import AutoModelForCausalLM
    cfg = hf_config(cfg_dict, **overrides)
    spec = spec_from_config(dict(cfg_dict, **overrides))
    with torch.device('meta'):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16)
    if not keep_experts:
        for idx in spec.moe_layers:
            model.model.layers[idx].mlp.experts = None  # routed experts live in the pinned pool
    model.to_empty(device=device)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if 'norm' in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=gen)
        for name, mod in _rope_modules(model):  # buffers were never computed on the meta device
            fresh = type(mod)(mod.config, device=device)
            for b in ('inv_freq', 'original_inv_freq'):
                if hasattr(fresh, b):
                    setattr(mod, b, getattr(fresh, b))
            mod.attention_scaling = fresh.attention_scaling
    model.eval()
    return model, spec


def expert_pool_from_model(model, spec):
    """The routed experts of a keep_experts model as a pinned pool [L*E, 3HI]
    in the row layout [gate | up | down] (ferry/model.py:86-105)."""
    I = spec.intermediate
    pool = torch.empty((spec.layers * spec.experts, spec.expert_elements), dtype=torch.bfloat16,
                       pin_memory=True)
    for layer, idx in enumerate(spec.moe_layers):
        ex = model.model.layers[idx].mlp.experts
        for e in range(spec.experts):
            gu = ex.gate_up_proj[e]
            pool[layer * spec.experts + e].copy_(pack_expert(gu[:I], gu[I:], ex.down_proj[e]))
    return pool


def shared_expert_rows(model, spec):
    """DeepSeek-V2 shared-expert MLPs as pool-layout rows, one per MoE layer."""
    rows = []
    for idx in spec.moe_layers:
        se = getattr(model.model.layers[idx].mlp, 'shared_experts', None)
        rows.append(None if se is None else pack_expert(se.gate_proj.weight, se.up_proj.weight,
                                                        se.down_proj.weight).contiguous())
    return rows if any(r is not None for r in rows) else None


def install_hooks(model, spec, runtime):
    """Route every MoE block through runtime.forward (router in kernel 1)."""
    for layer, idx in enumerate(spec.moe_layers):
        mlp = model.model.layers[idx].mlp
        gate = mlp.gate.weight

        def forward(hidden_states, _layer=layer, _gate=gate):
            shape = hidden_states.shape
            flat = hidden_states.reshape(-1, shape[-1]).contiguous()
            return runtime.forward(_layer, flat, _gate).view(shape)
        mlp.forward = forward


@torch.no_grad()
def generate(model, input_ids, new_tokens):
    """Greedy decode; returns (tokens [B, new_tokens], per-token event times in
    ms from the start, measured on this rank's stream)."""
    from transformers import DynamicCache
    start = torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(new_tokens)]
    cache = DynamicCache(config=model.config)
    start.record()
    out = model(input_ids=input_ids, past_key_values=cache, use_cache=True)
    nxt = out.logits[:, -1].argmax(-1, keepdim=True)
    marks[0].record()
    tokens = [nxt]
    for i in range(1, new_tokens):
        out = model(input_ids=nxt, past_key_values=out.past_key_values, use_cache=True)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        marks[i].record()
        tokens.append(nxt)
    marks[-1].synchronize()
    return torch.cat(tokens, 1), [start.elapsed_time(m) for m in marks]


def decode_metrics(times_ms, batch, world):
    """TTFT, TPOT and decode tokens/s, max over ranks."""
    t = torch.tensor(times_ms, dtype=torch.float64, device='cuda' if world > 1 else 'cpu')
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t = t.cpu().tolist()
    n = len(t)
    decode_s = (t[-1] - t[0]) / 1e3
    return {'ttft_ms': t[0], 'tpot_ms': (t[-1] - t[0]) / max(1, n - 1),
            'decode_tokens_per_s': world * batch * (n - 1) / decode_s if n > 1 and decode_s > 0 else None,
            'total_tokens_per_s': world * batch * n / (t[-1] / 1e3)}


def run(cfg_dict, *, batch, prompt_len, new_tokens, cache_ratio=0.3, seed=0, layers=None, warmup=1,
        rank=0, world=1, device=None, timing=False, policy='ferry', topology=None):
    """Build, hook and run one generation (after `warmup` untimed ones).
    topology: None/'uniform', 'auto' (profile the ranks' host links now) or a
    topology JSON path (ferry_b200.build_quota_lut.topology_for_run)."""
    from .build_quota_lut import topology_for_run
    from .runtime import OffloadRuntime
    from .workload import SyntheticMoE
    device = device or torch.device('cuda', torch.cuda.current_device())
    overrides = {'num_hidden_layers': layers} if layers else {}
    model, spec = build_model(cfg_dict, device, seed, **overrides)
    wl = SyntheticMoE(spec, seed=seed + 1, device=device, shared=world > 1)
    caps = spec.cache_slots(cache_ratio, world)
    topo, topo_note = topology_for_run(topology, spec, rank, world, pool_row=wl.pool[0], device=device)
    rt = OffloadRuntime(spec, wl.pool, caps, policy, topo,
                        norm_topk_prob=bool(cfg_dict.get('norm_topk_prob', True)),
                        routed_scaling_factor=float(cfg_dict.get('routed_scaling_factor', 1.0)),
                        shared_experts=shared_expert_rows(model, spec), timing=timing)
    install_hooks(model, spec, rt)
    vocab = cfg_dict['vocab_size']
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    prompts = torch.randint(0, vocab, (batch, prompt_len), generator=g, device=device)
    for _ in range(warmup):
        generate(model, prompts, min(new_tokens, 4))
        rt.reset()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tokens, times = generate(model, prompts, new_tokens)
    wall = time.perf_counter() - t0
    m = decode_metrics(times, batch, world)
    m.update(fetches_per_rank=rt.fetches_per_rank.tolist(),
             decode_fetches_per_rank=rt.decode_fetches_per_rank.tolist(), wall_s=wall, topology=topo_note)
    return model, rt, tokens, m
