"""Seeded synthetic workloads with the shapes of the benchmark's configs.

No checkpoints or datasets are available, so (as the configs prescribe):
  * weights are random-init N(0, 0.02) in bf16: router gates [E, H] per MoE
    layer and the routed experts, packed into a pinned host pool with one row
    per (MoE layer, expert) = [gate I x H | up I x H | down H x I]
    (ferry/model.py:86-105);
  * a Zipf(s) popularity bias b_e = log p_e, p_e ~ rank_e^-s over a seeded
    permutation of the experts, is added to each layer's router logits;
  * decode hidden states are N(0, 1) with step-to-step correlation rho:
    h_{s+1} = rho h_s + sqrt(1 - rho^2) N(0, 1).
`pool_layers` < layers makes the pool hold fewer layers' experts; the H2D
engine then reads row (key mod pool rows), i.e. later layers reuse the first
layers' weights (a host-memory saving for multi-GPU runs; the bytes moved are
the same).
"""
import math

import torch


def zipf_bias(experts, s, generator):
    perm = torch.randperm(experts, generator=generator)
    p = 1.0 / (torch.arange(1, experts + 1, dtype=torch.float64) ** s)
    p = p / p.sum()
    bias = torch.empty(experts, dtype=torch.float32)
    bias[perm] = torch.log(p).float()
    return bias


class SyntheticMoE:
    def __init__(self, spec, *, seed=0, zipf_s=1.1, rho=0.5, device='cuda', pool_layers=None,
                 build_pool=True, shared=False, group=None):
        """shared: one pool per node in shared pinned memory (ferry_b200.pool),
        filled by the group's first rank, instead of one pinned pool per rank."""
        self.spec, self.rho, self.device = spec, rho, torch.device(device)
        E, H, L = spec.experts, spec.hidden, spec.layers
        g = torch.Generator().manual_seed(seed)
        self.gate = [(torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(self.device)
                     for _ in range(L)]
        self.bias = [zipf_bias(E, zipf_s, g).to(self.device) for _ in range(L)]
        self.pool_layers = L if pool_layers is None else max(1, min(L, pool_layers))
        self.shared_pool = None
        self.pool = None
        if build_pool:
            rows = self.pool_layers * spec.experts
            if shared:
                from .pool import SharedPinnedPool
                self.shared_pool = SharedPinnedPool(rows, spec.expert_elements,
                                                    fill=lambda t: self._fill(t, seed + 1), group=group)
                self.pool = self.shared_pool.tensor
            else:
                self.pool = torch.empty((rows, spec.expert_elements), dtype=torch.bfloat16,
                                        pin_memory=torch.cuda.is_available())
                self._fill(self.pool, seed + 1)

    def _fill(self, pool, seed):
        """N(0, 0.02) bf16 rows drawn on the GPU from a seeded generator."""
        spec = self.spec
        rows = pool.shape[0]
        gen = torch.Generator(device=self.device).manual_seed(seed)
        chunk = max(1, (1 << 30) // (spec.expert_elements * 2))
        for r0 in range(0, rows, chunk):
            n = min(chunk, rows - r0)
            block = torch.randn((n, spec.expert_elements), generator=gen, device=self.device,
                                dtype=torch.float32).mul_(0.02).to(torch.bfloat16)
            pool[r0:r0 + n].copy_(block)
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
        return pool

    def hidden_stream(self, tokens, seed=0, world=1, rank=0):
        """Per MoE layer, an endless ρ-correlated sequence of [tokens, H] states."""
        return HiddenStream(self.spec, tokens, self.rho, seed * 1000 + rank, self.device)


class HiddenStream:
    """Drawn on the CPU from a seeded generator (so every arm of the bench, GPU
    or CPU, sees the same states) and handed out on `device`."""

    def __init__(self, spec, tokens, rho, seed, device):
        self.gen = torch.Generator().manual_seed(seed)
        self.device = torch.device(device)
        self.rho, self.c = rho, math.sqrt(1 - rho * rho)
        self.state = [torch.randn((tokens, spec.hidden), generator=self.gen)
                      for _ in range(spec.layers)]

    def next(self, layer):
        """The layer's hidden states for the next decode step (bf16)."""
        h = self.state[layer]
        out = h.to(torch.bfloat16)
        self.state[layer] = h.mul(self.rho).add_(torch.randn(h.shape, generator=self.gen), alpha=self.c)
        return out.to(self.device)


def cpu_pool(spec, layers, seed=0):
    """A small pool on the CPU for tests (N(0, 0.02) bf16)."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(layers * spec.experts, spec.expert_elements, generator=g) * 0.02).to(torch.bfloat16)
