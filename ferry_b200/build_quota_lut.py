"""Bandwidth domains and the Step-2 quota lookup table from an H2D profile
(the reference's scripts/build_quota_lut.py; same input and output JSON, read
by ferry_b200.quota.Topology and ferry.quota.Topology alike).

Every GPU is a singleton domain.  The shared domains are either every
profiled subset (default) or explicit groups such as PCIe switches or NUMA
nodes (--groups 0,1:2,3).  Row m of the table is greedy_quota(m) without
capacity limits (ferry/quota.py:70-74), computed on the GPU.
"""
import argparse
import json
import sys
from pathlib import Path

from .profile_h2d import MODELS, model_spec


def select_domains(profile, groups=None):
    """(masks, gib_per_s, gpus) of the domains the table is built over."""
    world = profile['world']
    by_mask = {d['mask']: d for d in profile['domains']}
    if groups:
        masks = [1 << r for r in range(world)]
        masks += [sum(1 << int(g) for g in grp.split(',')) for grp in groups.split(':')]
    else:
        masks = sorted(by_mask, key=lambda m: (bin(m).count('1'), m))
    missing = [m for m in masks if m not in by_mask]
    if missing:
        raise ValueError(f'profile has no measurement for GPU sets {missing}')
    return [dict(gpus=by_mask[m]['gpus'], mask=m, gib_per_s=by_mask[m]['gib_per_s']) for m in masks]


def build(profile, spec, groups=None, lut_fn=None):
    """The topology JSON object; lut_fn(max_misses, world, masks, seconds)
    defaults to the device build_lut."""
    if lut_fn is None:
        from .quota import build_lut as lut_fn
    domains = select_domains(profile, groups)
    world = profile['world']
    lut = lut_fn(spec.experts, world, [d['mask'] for d in domains], [1.0 / d['gib_per_s'] for d in domains])
    return dict(world=world, physical_gpus=profile['physical_gpus'], expert_bytes=profile['expert_bytes'],
                model_type=spec.model_type, domains=domains, quota_lut=[list(map(int, r)) for r in lut])


def topology_for_run(topology, spec, rank, world, pool_row=None, device=None, group=None):
    """(Topology, note) of a run.  topology: None or 'uniform' (equal
    singleton links), a topology JSON path, or 'auto': with several ranks,
    every subset of ranks copies `pool_row` (one pinned expert row) into HBM
    at once (profile_h2d.profile_ranks), rank 0 builds the table and
    broadcasts it; one rank needs no profile (the even table is exact)."""
    import time

    import torch
    import torch.distributed as dist

    from .profile_h2d import profile_ranks
    from .quota import Topology
    if topology in (None, '', 'uniform') or (topology == 'auto' and world == 1):
        return Topology.uniform(world, spec.experts), 'uniform'
    if topology != 'auto':
        return Topology(topology, world, spec.experts), str(topology)
    if pool_row is None:
        raise ValueError("topology 'auto' needs a pinned expert row to copy")
    target = torch.empty(pool_row.numel(), dtype=pool_row.dtype, device=device)
    t0 = time.time()
    domains = profile_ranks(rank, world, target, pool_row, copies=16, repeats=2, group=group)
    profile = dict(world=world, physical_gpus=list(range(world)), expert_bytes=spec.expert_bytes,
                   domains=domains)
    box = [build(profile, spec)['quota_lut'] if rank == 0 else None]
    dist.broadcast_object_list(box, src=0, group=group)
    masks = sorted((d['mask'] for d in domains), key=lambda m: (bin(m).count('1'), m))
    by_mask = {d['mask']: d for d in domains}
    topo = Topology.from_arrays(masks, [1.0 / by_mask[m]['gib_per_s'] for m in masks], box[0])
    singles = [round(by_mask[1 << r]['gib_per_s'], 1) for r in range(world)]
    return topo, (f'auto: profiled {len(domains)} rank subsets in {time.time() - t0:.1f} s; '
                  f'single-GPU GiB/s {singles}, all-GPU {round(by_mask[(1 << world) - 1]["gib_per_s"], 1)}')


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    p.add_argument('--profile', required=True)
    p.add_argument('--model', choices=sorted(MODELS), default='qwen3')
    p.add_argument('--model-path')
    p.add_argument('--output', required=True)
    p.add_argument('--groups', help='explicit shared domains, e.g. 0,1:2,3 (default: every profiled subset)')
    a = p.parse_args(argv)
    profile = json.loads(Path(a.profile).read_text())
    spec = model_spec(a.model, a.model_path)
    if profile['expert_bytes'] != spec.expert_bytes:
        print(f"warning: profiled with {profile['expert_bytes']} B copies, model experts are "
              f"{spec.expert_bytes} B", file=sys.stderr)
    topo = build(profile, spec, a.groups)
    out = Path(a.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(topo) + '\n')
    lut = topo['quota_lut']
    for m in sorted({1, topo['world'], spec.experts // 4, spec.experts // 2, spec.experts}):
        print(f'm={m:4d}: quota {lut[m]}')
    print(f'wrote {out}')
    return 0


if __name__ == '__main__':
    raise SystemExit(main())
