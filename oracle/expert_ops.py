"""torch-CPU restatement of ferry_expert_ops and of the MoE-hook routers
(test infrastructure only).

The reference ops (ferry/csrc/expert_ops.cpp, expert_ops.cu) TORCH_CHECK that
their inputs are CUDA tensors, so they have no CPU path; these functions
follow their ATen op order and bf16 rounding points on CPU tensors.  GEMMs
accumulate in float32 and round once to bf16, as cuBLAS's bf16 GEMM does (the
summation order differs, which is why expert outputs are compared within the
BF16 tolerance, not bit-exactly).
"""
import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


def _mm_bf16(a, b_t):
    """bf16 GEMM a @ b_t.T with float32 accumulation and one rounding to bf16."""
    return (a.float() @ b_t.float().t()).to(BF16)


def silu_mul(gate, up):
    """ferry/csrc/expert_ops.cu:6-14 -- bf16(g / (1 + exp(-g)) * u), float32 math."""
    g, u = gate.float(), up.float()
    return ((g / (1.0 + torch.exp(-g))) * u).to(BF16)


def expert_views(row, hidden, intermediate):
    """ferry/model.py:86-88 and expert_ops.cpp:35-38 -- [gate I x H | up I x H | down H x I]."""
    part = hidden * intermediate
    return (row[:part].view(intermediate, hidden), row[part:2 * part].view(intermediate, hidden),
            row[2 * part:3 * part].view(hidden, intermediate))


def expert_forward(x, row, hidden, intermediate):
    """One routed expert without the routing weight (expert_ops.cpp:39-41)."""
    gate, up, down = expert_views(row, hidden, intermediate)
    return _mm_bf16(silu_mul(_mm_bf16(x, gate), _mm_bf16(x, up)), down)


def execute_experts(cache, inputs, routing_weights, slots, rows, cols, hidden, intermediate):
    """ferry/csrc/expert_ops.cpp:16-45 -- list of [n_e, H] bf16, one per group."""
    outputs = []
    for slot, r, c in zip(slots, rows, cols):
        r, c = r.long(), c.long()
        y = expert_forward(inputs.index_select(0, r), cache[slot], hidden, intermediate)
        outputs.append((y.float() * routing_weights[r, c].float().unsqueeze(1)).to(BF16))
    return outputs


def pack_dispatch(hidden, selected, weights, send_idx, send_ids, experts):
    """ferry/csrc/expert_ops.cpp:50-66 -- packet bytes [hidden | k bf16 weights | k u8 ids]."""
    n, h, k = send_idx.shape[0], hidden.shape[1], send_ids.shape[1]
    dense = torch.zeros(hidden.shape[0], experts, dtype=torch.float32)
    dense.scatter_add_(1, selected.long(), weights.float())
    dense = dense.to(BF16)
    valid = send_ids >= 0
    packet_w = dense[send_idx.long().unsqueeze(1), send_ids.long().clamp_min(0)] * valid
    payload = torch.empty(n, 2 * h + 3 * k, dtype=torch.uint8)
    payload[:, :2 * h] = hidden.index_select(0, send_idx.long()).contiguous().view(torch.uint8)
    payload[:, 2 * h:2 * h + 2 * k] = packet_w.to(BF16).contiguous().view(torch.uint8)
    payload[:, 2 * h + 2 * k:] = send_ids.to(torch.uint8)
    return payload


def unpack_dispatch(raw, hidden, topk):
    """ferry/csrc/expert_ops.cpp:68-73."""
    m = raw.shape[0]
    x = raw[:, :2 * hidden].contiguous().view(BF16).view(m, hidden)
    w = raw[:, 2 * hidden:2 * hidden + 2 * topk].contiguous().view(BF16).view(m, topk)
    return x, w


def reduce_partials(parts, rows, received, hidden):
    """ferry/csrc/expert_ops.cpp:76-83 -- float32 index_add_ per group, then bf16."""
    partial = torch.zeros(received, hidden, dtype=torch.float32)
    for p, r in zip(parts, rows):
        partial.index_add_(0, r.long(), p.float())
    return partial.to(BF16)


def scatter_returned(returned, send_idx, tokens):
    """ferry/csrc/expert_ops.cpp:86-92 -- float32 index_add_ per token, then bf16."""
    out = torch.zeros(tokens, returned.shape[1], dtype=torch.float32)
    if returned.shape[0]:
        out.index_add_(0, send_idx.long(), returned.float())
    return out.to(returned.dtype)


def route_qwen3(hidden, gate_weight, topk, norm_topk_prob=True, bias=None):
    """ferry/model.py:137-148 (_qwen3_forward): bf16 router GEMM, float32 softmax,
    top-k, renormalisation, bf16 weights.  `bias` (float32 [E]) is the synthetic
    popularity bias, added inside the GEMM before the bf16 rounding (a Linear
    with bias).  Returns (selected int64, weights bf16, probs float32)."""
    acc = hidden.float() @ gate_weight.float().t()
    if bias is not None:
        acc = acc + bias.float()
    logits = acc.to(BF16)
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    w, sel = torch.topk(probs, topk, dim=-1)
    if norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    return sel, w.to(BF16), probs


def route_deepseek(hidden, gate_weight, topk, scaling=1.0, bias=None):
    """transformers DeepseekV2Moe.route_tokens_to_experts (greedy) as the reference
    hook consumes it (ferry/model.py:151-158): float32 logits and softmax, top-k,
    no renormalisation, times routed_scaling_factor, bf16 weights."""
    logits = F.linear(hidden.float(), gate_weight.float())
    if bias is not None:
        logits = logits + bias.float()
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    w, sel = torch.topk(probs, topk, dim=-1)
    return sel, (w * scaling).to(BF16), probs


def shared_expert(x, gate_w, up_w, down_w):
    """transformers DeepseekV2MLP with bf16 Linears: down(silu(gate(x)) * up(x)),
    each Linear and each elementwise op rounding to bf16."""
    g = _mm_bf16(x, gate_w)
    u = _mm_bf16(x, up_w)
    a = (F.silu(g.float()).to(BF16).float() * u.float()).to(BF16)
    return _mm_bf16(a, down_w)
