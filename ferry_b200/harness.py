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
import json
import re
import time
from pathlib import Path

import torch
import torch.distributed as dist

from .model import pack_expert, read_spec, spec_from_config


def hf_config(cfg_dict, **overrides):
    """A transformers config object from a config dict (model.py's dicts)."""
    from transformers import DeepseekV2Config, Qwen3MoeConfig
    d = dict(cfg_dict, **overrides)
    cls = Qwen3MoeConfig if d['model_type'] == 'qwen3_moe' else DeepseekV2Config
    d.pop('model_type')
    return cls(**d)


def _rope_modules(model):
    return [(name, mod) for name, mod in model.named_modules() if hasattr(mod, 'inv_freq')]


def _fresh_rope(model, device):
    """Rotary buffers computed on `device` (a model built on the meta device
    never computed them)."""
    for _, mod in _rope_modules(model):
        fresh = type(mod)(mod.config, device=device)
        for b in ('inv_freq', 'original_inv_freq'):
            if hasattr(fresh, b):
                setattr(mod, b, getattr(fresh, b))
        mod.attention_scaling = fresh.attention_scaling


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
        _fresh_rope(model, device)
    model.eval()
    return model, spec


# Routed-expert tensors of a checkpoint: one 2-D weight per expert and
# projection (the Hugging Face layout), or transformers 5's fused 3-D
# parameters of a layer's experts.
_EXPERT_2D = re.compile(r'model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight')
_EXPERT_3D = re.compile(r'model\.layers\.(\d+)\.mlp\.experts\.(gate_up_proj|down_proj)')


def load_checkpoint(model_path, device='cuda'):
    """(model, spec, pool) from a local checkpoint directory (config.json and
    model.safetensors, or shards listed by model.safetensors.index.json): the
    reference's load (ferry/model.py:73-122).  Dense weights (attention,
    norms, routers, shared experts, embeddings) land on `device` in bf16; the
    routed experts go straight from the files into one host pool
    [layers * experts, 3 * H * I] bf16 in the row layout [gate | up | down]
    (pinned when CUDA is present), never into the model.  Raises ValueError
    if an expert projection or a dense parameter is missing, or a tensor has
    the wrong size."""
    from safetensors import safe_open
    from transformers import AutoConfig, AutoModelForCausalLM, GenerationConfig
    path = Path(model_path)
    spec = read_spec(path)
    cfg = AutoConfig.from_pretrained(path, local_files_only=True)
    with torch.device('meta'):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16)
    for idx in spec.moe_layers:
        model.model.layers[idx].mlp.experts = None  # routed experts live in the pool
    index = path / 'model.safetensors.index.json'
    if index.exists():
        weight_map = json.loads(index.read_text())['weight_map']
    else:
        with safe_open(str(path / 'model.safetensors'), framework='pt') as f:
            weight_map = {name: 'model.safetensors' for name in f.keys()}
    layer_of = {idx: i for i, idx in enumerate(spec.moe_layers)}
    E, H, I = spec.experts, spec.hidden, spec.intermediate
    hi = H * I
    part_at = {'gate_proj': 0, 'up_proj': hi, 'down_proj': 2 * hi}
    pool = torch.empty((spec.layers * E, spec.expert_elements), dtype=torch.bfloat16,
                       pin_memory=torch.cuda.is_available())
    have = torch.zeros((spec.layers * E, 3), dtype=torch.bool)
    dense = {}

    def put(layer_idx, e, part, w):
        if layer_idx not in layer_of or not 0 <= e < E:
            raise ValueError(f'routed expert {e} of layer {layer_idx} is not in the model')
        if w.numel() != hi:
            raise ValueError(f'layer {layer_idx} expert {e} {part}: {w.numel()} elements, want {hi}')
        key = layer_of[layer_idx] * E + e
        pool[key, part_at[part]:part_at[part] + hi].copy_(w.reshape(-1))
        have[key, ('gate_proj', 'up_proj', 'down_proj').index(part)] = True

    for shard in sorted(set(weight_map.values())):
        with safe_open(str(path / shard), framework='pt', device='cpu') as f:
            for name in sorted(n for n, s in weight_map.items() if s == shard):
                m2, m3 = _EXPERT_2D.fullmatch(name), _EXPERT_3D.fullmatch(name)
                if m2:
                    put(int(m2[1]), int(m2[2]), m2[3], f.get_tensor(name))
                elif m3:
                    w = f.get_tensor(name)  # gate_up [E, 2I, H] or down [E, H, I]
                    for e in range(w.shape[0]):
                        if m3[2] == 'gate_up_proj':
                            put(int(m3[1]), e, 'gate_proj', w[e, :I])
                            put(int(m3[1]), e, 'up_proj', w[e, I:])
                        else:
                            put(int(m3[1]), e, 'down_proj', w[e])
                else:
                    dense[name] = f.get_tensor(name).to(torch.bfloat16)
    if not bool(have.all()):
        key = int((~have.all(dim=1)).nonzero()[0])
        raise ValueError(f'routed-expert weights are incomplete (first missing: MoE layer '
                         f'{key // E}, expert {key % E})')
    result = model.load_state_dict(dense, strict=False, assign=True)
    model.tie_weights()
    missing = [n for n, p in model.named_parameters() if p.is_meta]
    if missing:
        raise ValueError(f'{len(missing)} dense parameters are missing, e.g. {missing[0]}')
    if result.unexpected_keys:
        raise ValueError(f'unexpected tensors in the checkpoint, e.g. {result.unexpected_keys[0]}')
    with torch.no_grad():
        _fresh_rope(model, device)  # the only buffers a checkpoint does not carry
    left = [n for n, b in model.named_buffers() if b.is_meta]
    if left:
        raise ValueError(f'buffer {left[0]} has no value')
    model.to(device)
    if (path / 'generation_config.json').exists():
        model.generation_config = GenerationConfig.from_pretrained(path, local_files_only=True)
    model.eval()
    return model, spec, pool


def expert_pool_from_model(model, spec):
    """The routed experts of a keep_experts model as a host pool [L*E, 3HI]
    (pinned when CUDA is present) in the row layout [gate | up | down]
    (ferry/model.py:86-105)."""
    I = spec.intermediate
    pool = torch.empty((spec.layers * spec.experts, spec.expert_elements), dtype=torch.bfloat16,
                       pin_memory=torch.cuda.is_available())
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


def install_hooks(model, spec, runtime, history_window=None):
    """Route every MoE block through runtime.forward (router in kernel 1).
    history_window is accepted for the reference's signature
    (ferry/model.py:125); the runtime keeps its own window."""
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
        rank=0, world=1, device=None, timing=False, policy='ferry', topology=None, checkpoint=None):
    """Build, hook and run one generation (after `warmup` untimed ones).
    topology: None/'uniform', 'auto' (profile the ranks' host links now) or a
    topology JSON path (ferry_b200.build_quota_lut.topology_for_run).
    checkpoint: a local checkpoint directory (load_checkpoint) whose weights
    and config replace the random model of cfg_dict; each rank then holds its
    own pinned pool, as the reference's does."""
    from .build_quota_lut import topology_for_run
    from .runtime import OffloadRuntime
    from .workload import SyntheticMoE
    device = device or torch.device('cuda', torch.cuda.current_device())
    wl = None  # owns a shared pool's mapping: kept alive while the runtime runs
    if checkpoint is not None:
        model, spec, pool = load_checkpoint(checkpoint, device)
        cfg_dict = dict(model.config.to_dict(), model_type=spec.model_type)
    else:
        overrides = {'num_hidden_layers': layers} if layers else {}
        model, spec = build_model(cfg_dict, device, seed, **overrides)
        wl = SyntheticMoE(spec, seed=seed + 1, device=device, shared=world > 1)
        pool = wl.pool
    caps = spec.cache_slots(cache_ratio, world)
    topo, topo_note = topology_for_run(topology, spec, rank, world, pool_row=pool[0], device=device)
    rt = OffloadRuntime(spec, pool, caps, policy, topo,
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
    rt.pool_owner = wl  # the pool stays mapped as long as the runtime exists
    return model, rt, tokens, m
