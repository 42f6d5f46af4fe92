"""Offline host-to-device bandwidth profile of the visible GPUs (the
reference's scripts/profile_h2d.py, same JSON output).

For every non-empty subset of the visible GPUs, each GPU of the subset copies
expert-sized rows from its own pinned host buffer into HBM on a copy-engine
stream, all GPUs at once (their streams are held by a short device spin until
every copy is enqueued).  The per-GPU effective bandwidth and the subset's
aggregate are recorded: singletons give each GPU's own link, larger subsets
expose shared PCIe switches, NUMA nodes and host-memory limits.  On an
8-GPU B200 HGX node that is 255 subsets.

  python -m ferry_b200.profile_h2d --model qwen3 --output topology/b200_profile.json
  python -m ferry_b200.build_quota_lut --profile topology/b200_profile.json \\
      --model qwen3 --output topology/b200_qwen3.json
"""
import argparse
import itertools
import json
import os
import statistics
from pathlib import Path

import torch

from .model import DEEPSEEK_V2_LITE, QWEN3_30B_A3B, read_spec, spec_from_config

MODELS = {'qwen3': QWEN3_30B_A3B, 'deepseek': DEEPSEEK_V2_LITE}


def model_spec(model=None, model_path=None):
    if model_path:
        return read_spec(model_path)
    return spec_from_config(MODELS[model])


class Rig:
    """Per GPU: a pinned source row, a small ring of HBM targets, a stream."""

    def __init__(self, gpus, elements, ring=4):
        self.sources, self.targets, self.streams = {}, {}, {}
        for g in gpus:
            with torch.cuda.device(g):
                self.sources[g] = torch.randn(elements, dtype=torch.bfloat16).pin_memory()
                self.targets[g] = [torch.empty(elements, dtype=torch.bfloat16, device=g)
                                   for _ in range(ring)]
                self.streams[g] = torch.cuda.Stream(device=g)
        self.nbytes = elements * 2

    def measure(self, subset, copies, spin_cycles):
        """GiB/s per GPU of `copies` back-to-back row copies, all GPUs of the
        subset copying at the same time."""
        starts, ends = {}, {}
        for g in subset:
            with torch.cuda.device(g), torch.cuda.stream(self.streams[g]):
                if spin_cycles:
                    torch.cuda._sleep(spin_cycles)  # hold until every GPU is enqueued
                starts[g] = torch.cuda.Event(enable_timing=True)
                ends[g] = torch.cuda.Event(enable_timing=True)
                starts[g].record(self.streams[g])
        for i in range(copies):
            for g in subset:
                with torch.cuda.device(g), torch.cuda.stream(self.streams[g]):
                    self.targets[g][i % len(self.targets[g])].copy_(self.sources[g], non_blocking=True)
        for g in subset:
            with torch.cuda.device(g):
                ends[g].record(self.streams[g])
        for g in subset:
            ends[g].synchronize()
        return {g: copies * self.nbytes / (starts[g].elapsed_time(ends[g]) / 1e3) / 2**30 for g in subset}


def profile(spec, gpus, copies=64, repeats=5, spin_cycles=100_000_000, max_subset=None):
    rig = Rig(gpus, spec.expert_elements)
    top = len(gpus) if max_subset is None else max_subset
    subsets = [s for n in range(1, top + 1) for s in itertools.combinations(gpus, n)]
    for g in gpus:  # warm every copy engine
        rig.measure((g,), 8, 0)
    samples = {s: [] for s in subsets}
    for rep in range(repeats):
        for s in (subsets if rep % 2 == 0 else subsets[::-1]):
            samples[s].append(rig.measure(s, copies, spin_cycles))
    domains = []
    for s in subsets:
        per_gpu = {g: statistics.median(x[g] for x in samples[s]) for g in s}
        domains.append(dict(gpus=list(s), mask=sum(1 << gpus.index(g) for g in s),
                            gib_per_s=sum(per_gpu.values()),
                            per_gpu_gib_per_s=[per_gpu[g] for g in s]))
    return domains


def profile_ranks(rank, world, target, source, copies=16, repeats=2, group=None):
    """The same profile taken by the ranks of a torch.distributed job, one GPU
    each: for every subset of ranks, after a barrier, the ranks of the subset
    copy `source` (pinned host row) into `target` (device row) `copies` times
    at once; returns the profile's domain list (masks over ranks)."""
    import torch.distributed as dist
    nbytes = source.numel() * source.element_size()
    stream = torch.cuda.Stream()
    ranks = list(range(world))
    subsets = [s for n in range(1, world + 1) for s in itertools.combinations(ranks, n)]
    with torch.cuda.stream(stream):  # warm the copy engine
        for _ in range(4):
            target.copy_(source, non_blocking=True)
    stream.synchronize()
    mine = torch.zeros((repeats, len(subsets)), dtype=torch.float64, device=target.device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for rep in range(repeats):
        for i, s in enumerate(subsets):
            dist.barrier(group=group)
            if rank in s:
                with torch.cuda.stream(stream):
                    e0.record(stream)
                    for _ in range(copies):
                        target.copy_(source, non_blocking=True)
                    e1.record(stream)
                e1.synchronize()
                mine[rep, i] = copies * nbytes / (e0.elapsed_time(e1) / 1e3) / 2**30
    allv = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(allv, mine, group=group)
    per = torch.stack(allv).median(dim=1).values.cpu().numpy()  # [world, subsets]
    domains = []
    for i, s in enumerate(subsets):
        vals = [float(per[g, i]) for g in s]
        domains.append(dict(gpus=list(s), mask=sum(1 << g for g in s), gib_per_s=sum(vals),
                            per_gpu_gib_per_s=vals))
    return domains


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    p.add_argument('--model', choices=sorted(MODELS), default='qwen3',
                   help='size the copies like one expert of this model')
    p.add_argument('--model-path', help='or read the model config from a checkpoint directory')
    p.add_argument('--output', required=True)
    p.add_argument('--copies', type=int, default=64, help='back-to-back copies per GPU per sample')
    p.add_argument('--repeats', type=int, default=5)
    p.add_argument('--spin-cycles', type=int, default=100_000_000,
                   help='GPU spin before the copies so that all GPUs start together')
    p.add_argument('--max-subset', type=int, help='profile subsets up to this size only')
    a = p.parse_args(argv)
    spec = model_spec(a.model, a.model_path)
    world = torch.cuda.device_count()
    gpus = list(range(world))
    domains = profile(spec, gpus, a.copies, a.repeats, a.spin_cycles, a.max_subset)
    for d in domains:
        if len(d['gpus']) in (1, 2, world):
            print(f"GPUs {d['gpus']}: aggregate {d['gib_per_s']:.2f} GiB/s, per GPU "
                  + ', '.join(f'{v:.2f}' for v in d['per_gpu_gib_per_s']))
    visible = os.environ.get('CUDA_VISIBLE_DEVICES')
    out = Path(a.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(dict(world=world, physical_gpus=visible.split(',') if visible else gpus,
                                   expert_bytes=spec.expert_bytes, copies=a.copies, repeats=a.repeats,
                                   domains=domains), indent=1) + '\n')
    print(f'wrote {out}')
    return 0


if __name__ == '__main__':
    raise SystemExit(main())
