"""Generate the golden vectors in tests/golden/ by running the REFERENCE code.

Run in a container where the FERRY reference is mounted (read-only):

    python tests/golden/make_golden.py --reference /path/to/FERRY

It imports the reference's own ferry.policy, ferry.quota, ferry.layout and
ferry.metadata (numba/numpy, CPU), drives them on seeded synthetic inputs at
the benchmark configurations' shapes and on edge cases, and writes compressed .npz
fixtures.  The fixtures travel with the repository; nothing at test time reads
the reference.  Routing ids are drawn as Zipf(1.1)-skewed top-k (Gumbel top-k
over log-popularity of a seeded expert permutation), the same distribution as
softmax top-k under a Zipf gate bias.
"""
import argparse
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def zipf_topk(rng, tokens, experts, topk, s=1.1):
    perm = rng.permutation(experts)
    logp = np.empty(experts)
    logp[perm] = -s * np.log(np.arange(1, experts + 1))
    g = rng.gumbel(size=(tokens, experts)) + logp
    return np.argsort(-g, axis=1, kind='stable')[:, :topk].astype(np.int64)


class Spec:
    def __init__(self, layers, experts):
        self.layers, self.experts = layers, experts


def plan_sequence(ref, name, *, layers, experts, topk, world, tokens, caps, policy, topology,
                  steps, bps=200, salt=1, window=128, event0=0, seed=0, layer_order=None,
                  score='frequency', state_every=1):
    """Drive the reference Controller + GateHistory over `steps` layer events."""
    policy_mod, metadata_mod = ref['policy'], ref['metadata']
    rng = np.random.default_rng(seed)
    spec = Spec(layers, experts)
    ctl = policy_mod.Controller(spec, caps, policy, topology, bps, salt)
    hist = metadata_mod.GateHistory(layers, experts, window)
    rec = dict(layers=layers, experts=experts, topk=topk, world=world, tokens=tokens,
               caps=np.asarray(caps, np.int64), policy=policy_mod.POLICIES[policy], bps=bps,
               salt=salt, window=window, masks=topology.masks, seconds=topology.seconds,
               lut=topology.lut, steps=steps, state_every=state_every)
    tail = min(tokens, -(-window // world))
    ev = event0
    for step in range(steps):
        layer = layer_order[step % len(layer_order)] if layer_order else step % layers
        sel = zipf_topk(rng, world * tokens, experts, topk)
        origins = np.repeat(np.arange(world, dtype=np.int64), tokens)
        if score == 'frequency':
            recent = sel.reshape(world, tokens, topk)[:, tokens - tail:].reshape(-1, topk)
            rows = np.zeros((len(recent), experts), np.float64)
            np.put_along_axis(rows, recent, 1.0, axis=1)
        else:
            rows = rng.dirichlet(np.ones(experts), size=world * tail).astype(np.float32)
        hist.update(layer, rows)
        gs = hist.scores(layer)
        rec[f's{step}_layer'] = np.int64(layer)
        rec[f's{step}_event'] = np.int64(ev)
        rec[f's{step}_selected'] = sel.astype(np.uint8)
        rec[f's{step}_rows'] = rows.astype(np.float32) if score != 'frequency' else np.zeros(0)
        rec[f's{step}_scores'] = gs
        try:
            f, d, c = ctl.plan(ev, layer, sel, origins, gs)
            rec[f's{step}_ok'] = np.int64(1)
            rec[f's{step}_fetches'] = f
            rec[f's{step}_dest'] = d.astype(np.int8)
            rec[f's{step}_counts'] = c
            if step % state_every == 0 or step == steps - 1:
                rec[f's{step}_slots'] = ctl.slots.astype(np.int16)
                rec[f's{step}_owner'] = ctl.owner.astype(np.int8)
                rec[f's{step}_last'] = ctl.last.astype(np.int32)
            # the layout of every rank for this step
            for r in range(world):
                si, sids, sc, rc, st, rows_, cols_ = ref['layout'].build_layout(sel, d, tokens, r, experts)
                rec[f's{step}_r{r}_send_idx'] = si
                rec[f's{step}_r{r}_send_ids'] = sids
                rec[f's{step}_r{r}_send_counts'] = sc
                rec[f's{step}_r{r}_recv_counts'] = rc
                rec[f's{step}_r{r}_starts'] = st
                rec[f's{step}_r{r}_rows'] = rows_
                rec[f's{step}_r{r}_cols'] = cols_
                rec[f's{step}_r{r}_layer_slots'] = policy_mod.layer_slots(ctl.slots[r], caps[r], layer, experts)
        except AssertionError:
            rec[f's{step}_ok'] = np.int64(0)
            rec['steps'] = step + 1
            break
        ev += 1
    np.savez_compressed(OUT / f'plan_{name}.npz', **rec)
    oks = [int(rec[f's{i}_ok']) for i in range(rec['steps'])]
    nf = [len(rec[f's{i}_fetches']) for i in range(rec['steps']) if rec[f's{i}_ok']]
    print(f'plan_{name}: steps={rec["steps"]} ok={sum(oks)} fetches/step={nf[:12]}')


def topology_random(quota_mod, world, experts, rng, subsets=True):
    topo = quota_mod.Topology.__new__(quota_mod.Topology)
    masks = [1 << r for r in range(world)]
    if subsets:
        masks = sorted(range(1, 1 << world), key=lambda m: (bin(m).count('1'), m))
    gib = []
    for m in masks:
        n = bin(m).count('1')
        gib.append(float(rng.uniform(20, 60)) * (n ** 0.6))
    topo.masks = np.asarray(masks, np.int64)
    topo.seconds = np.asarray([1.0 / g for g in gib], np.float64)
    topo.lut = quota_mod.build_lut(experts, world, topo.masks, topo.seconds)
    topo.gpus = None
    return topo


def quota_cases(quota_mod, rng, write=True):
    rec = {}
    n = 0
    for world in (1, 2, 3, 4, 8):
        for kind in ('uniform', 'singleton', 'subsets', 'ties'):
            if kind == 'uniform':
                masks = np.asarray([1 << r for r in range(world)], np.int64)
                seconds = np.ones(world)
            elif kind == 'singleton':
                masks = np.asarray([1 << r for r in range(world)], np.int64)
                seconds = rng.uniform(0.5, 2.0, world)
            elif kind == 'ties':
                masks = np.asarray(sorted(range(1, 1 << world), key=lambda m: (bin(m).count('1'), m)), np.int64)
                # bandwidths that are exact multiples make many makespans tie exactly
                seconds = np.asarray([1.0 / (25.0 * bin(int(m)).count('1')) for m in masks])
            else:
                masks = np.asarray(sorted(range(1, 1 << world), key=lambda m: (bin(m).count('1'), m)), np.int64)
                seconds = np.asarray([1.0 / (rng.uniform(20, 60) * bin(int(m)).count('1') ** 0.6)
                                      for m in masks])
            for trial in range(3):
                m = int(rng.integers(0, 64))
                cap = rng.integers(0, 40, world).astype(np.int64)
                if trial == 0:
                    cap[:] = 1 << 30
                try:
                    q = quota_mod.greedy_quota(m, cap, masks, seconds)
                    ok = 1
                except AssertionError:
                    q, ok = np.zeros(world, np.int64), 0
                rec[f'c{n}_m'] = np.int64(m)
                rec[f'c{n}_cap'] = cap
                rec[f'c{n}_masks'] = masks
                rec[f'c{n}_seconds'] = seconds
                rec[f'c{n}_quota'] = q
                rec[f'c{n}_ok'] = np.int64(ok)
                n += 1
            rec[f'lut{world}_{kind}_masks'] = masks
            rec[f'lut{world}_{kind}_seconds'] = seconds
            rec[f'lut{world}_{kind}'] = quota_mod.build_lut(64, world, masks, seconds)
    rec['n'] = np.int64(n)
    if write:
        np.savez_compressed(OUT / 'quota.npz', **rec)
    print('quota cases', n)


def assignment_cases(policy_mod, rng, write=True):
    rec = {}
    n = 0
    for world in (1, 2, 4, 8):
        for bps in (0, 200, 5000):
            for trial in range(4):
                experts = int(rng.choice([16, 64, 128]))
                layer, layers = int(rng.integers(0, 3)), 3
                demand = rng.integers(0, 6, (experts, world)).astype(np.int64)
                demand[rng.random(experts) < 0.3] = 0
                if trial == 3:  # heavy ties
                    demand = (demand > 2).astype(np.int64)
                owner = np.full(layers * experts, -1, np.int64)
                cached = rng.random(experts) < 0.4
                owner[layer * experts + np.flatnonzero(cached)] = rng.integers(0, world, cached.sum())
                active = demand.sum(1) > 0
                misses = np.flatnonzero(active & (owner[layer * experts:(layer + 1) * experts] < 0)).astype(np.int64)
                m = len(misses)
                quota = np.zeros(world, np.int64)
                for _ in range(m):
                    quota[rng.integers(0, world)] += 1
                ans = policy_mod.load_balanced_assignment(demand, misses, owner, layer, quota, bps)
                for k, v in dict(demand=demand, misses=misses, owner=owner, layer=np.int64(layer),
                                 quota=quota, bps=np.int64(bps), ans=ans).items():
                    rec[f'c{n}_{k}'] = v
                n += 1
    rec['n'] = np.int64(n)
    if write:
        np.savez_compressed(OUT / 'assignment.npz', **rec)
    print('assignment cases', n)


def choose_slot_cases(policy_mod, rng, write=True):
    rec = {}
    n = 0
    for trial in range(60):
        world = int(rng.choice([1, 2, 4]))
        experts, layers = int(rng.choice([8, 64])), int(rng.choice([1, 3]))
        caps = rng.integers(1, 12, world).astype(np.int64)
        slots = np.full((world, caps.max()), -1, np.int64)
        keys = rng.permutation(layers * experts)
        used = 0
        for r in range(world):
            for i in range(caps[r]):
                if rng.random() < (0.9 if trial % 3 else 0.5) and used < len(keys):
                    slots[r, i] = keys[used]
                    used += 1
        last = rng.integers(0, 4, layers * experts).astype(np.int64)
        # quantised scores make score ties (and then last-use ties) common
        scores = (rng.integers(0, 4, (layers, experts)) / 4.0).astype(np.float32)
        active = rng.random(experts) < 0.4
        layer = int(rng.integers(0, layers))
        rank = int(rng.integers(0, world))
        s = policy_mod._choose_slot(rank, layer, active, slots, caps, last, scores, experts)
        for k, v in dict(world=np.int64(world), experts=np.int64(experts), caps=caps, slots=slots,
                         last=last, scores=scores, active=active.astype(np.uint8),
                         layer=np.int64(layer), rank=np.int64(rank), slot=np.int64(s)).items():
            rec[f'c{n}_{k}'] = v
        n += 1
    rec['n'] = np.int64(n)
    if write:
        np.savez_compressed(OUT / 'choose_slot.npz', **rec)
    print('choose_slot cases', n)


def history_cases(metadata_mod, rng, write=True):
    rec = {}
    layers, experts, window = 2, 16, 8
    h = metadata_mod.GateHistory(layers, experts, window)
    n = 0
    for step, size in enumerate([3, 4, 2, 9, 1, 8, 5, 0, 20, 7]):
        layer = step % layers
        if step % 3 == 0:
            rows = rng.random((size, experts)).astype(np.float32).astype(np.float64)
        else:
            rows = np.zeros((size, experts))
            for i in range(size):
                rows[i, rng.choice(experts, 3, replace=False)] = 1.0
        h.update(layer, rows)
        rec[f'c{n}_layer'] = np.int64(layer)
        rec[f'c{n}_rows'] = rows
        rec[f'c{n}_scores'] = h.scores(layer)
        n += 1
    rec['n'] = np.int64(n)
    rec['layers'], rec['experts'], rec['window'] = np.int64(layers), np.int64(experts), np.int64(window)
    if write:
        np.savez_compressed(OUT / 'history.npz', **rec)
    print('history cases', n)


def mt_cases():
    from numba import njit

    @njit
    def draws(seed, n, count):
        np.random.seed(seed)
        out = np.empty(count, np.int64)
        for i in range(count):
            out[i] = np.random.randint(0, n)
        return out

    rec = {}
    n = 0
    for seed in (0, 1, 1000004, 2**32 - 1, 2**32 + 5, 7919 * 1000003 + 123456):
        for world in (1, 2, 3, 4, 5, 7, 8):
            rec[f'c{n}_seed'] = np.int64(seed)
            rec[f'c{n}_n'] = np.int64(world)
            rec[f'c{n}_draws'] = draws(seed, world, 700)
            n += 1
    rec['n'] = np.int64(n)
    np.savez_compressed(OUT / 'mt19937.npz', **rec)
    print('mt cases', n)


def _route_gather_worker(rank, world, port, reference, out_dir, score):
    """One gloo rank running the reference RouteGather with CPU buffers."""
    import torch
    import torch.distributed as dist
    sys.path.insert(0, reference)
    import ferry.metadata as md

    class _TorchShim:
        """Forwards to torch but drops device='cuda' / pin_memory (CPU-only ranks)."""
        def __getattr__(self, name):
            return getattr(torch, name)

        @staticmethod
        def empty(*a, **k):
            k.pop('device', None)
            k.pop('pin_memory', None)
            return torch.empty(*a, **k)

    md.torch = _TorchShim()
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    rng = np.random.default_rng(100 + rank)
    gather = md.RouteGather(topk=6, experts=64, window=128, score=score)
    res = {}
    for step, tokens in enumerate([16, 16, 48, 3]):
        sel = torch.from_numpy(zipf_topk(rng, tokens, 64, 6))
        probs = torch.from_numpy(rng.dirichlet(np.ones(64), size=tokens).astype(np.float32))
        ids, origins, rows = gather.collect(sel, probs)
        res[f's{step}_sel'] = sel.numpy()
        res[f's{step}_probs'] = probs.numpy()
        res[f's{step}_ids'] = ids
        res[f's{step}_origins'] = origins
        res[f's{step}_rows'] = np.asarray(rows)
    np.savez_compressed(Path(out_dir) / f'rg_{score}_{rank}.npz', **res)
    dist.barrier()
    dist.destroy_process_group()


def route_gather_cases(reference):
    import torch.multiprocessing as mp
    for score in ('frequency', 'probability'):
        world = 4
        with tempfile.TemporaryDirectory() as tmp:
            port = 29600 + (7 if score == 'frequency' else 8)
            mp.spawn(_route_gather_worker, args=(world, port, reference, tmp, score), nprocs=world)
            rec = {}
            for r in range(world):
                d = np.load(Path(tmp) / f'rg_{score}_{r}.npz')
                for k in d.files:
                    rec[f'r{r}_{k}'] = d[k]
            rec['world'] = np.int64(world)
            np.savez_compressed(OUT / f'route_gather_{score}.npz', **rec)
    print('route_gather cases written')


def main(a):
    sys.path.insert(0, a.reference)
    import ferry.layout as layout
    import ferry.metadata as metadata
    import ferry.policy as policy
    import ferry.quota as quota
    ref = dict(policy=policy, quota=quota, layout=layout, metadata=metadata)
    rng = np.random.default_rng(2024)
    only = set(a.only.split(',')) if a.only else None

    if only is None:
        mt_cases()
        quota_cases(quota, rng)
        assignment_cases(policy, rng)
        choose_slot_cases(policy, rng)
        history_cases(metadata, rng)
        route_gather_cases(a.reference)
    else:  # the random topologies below draw from rng after the cases above
        quota_cases(quota, rng, write=False)
        assignment_cases(policy, rng, write=False)
        choose_slot_cases(policy, rng, write=False)
        history_cases(metadata, rng, write=False)

    def plan_sequence_sel(ref_, name, **kw):
        if only is None or name in only:
            plan_sequence(ref_, name, **kw)

    U = quota.Topology.uniform
    # config 0: DeepSeek-V2-Lite layer, 4 ranks x 16 tokens, top-6 of 64, 8 steps
    plan_sequence_sel(ref, 'cfg0_caps19', layers=1, experts=64, topk=6, world=4, tokens=16,
                  caps=[19] * 4, policy='ferry', topology=U(4, 64), steps=8)
    plan_sequence_sel(ref, 'cfg0_caps5554', layers=1, experts=64, topk=6, world=4, tokens=16,
                  caps=[5, 5, 5, 4], policy='ferry', topology=U(4, 64), steps=8)
    # config 0 inside a 26-layer DeepSeek-V2-Lite stack (global 30% budget, 499 slots)
    plan_sequence_sel(ref, 'cfg0_stack', layers=26, experts=64, topk=6, world=4, tokens=16,
                  caps=[125, 125, 125, 124], policy='ferry', topology=U(4, 64), steps=52, state_every=4)
    # config 1: Qwen3 layer at one GPU, 64 tokens, top-8 of 128; 30% of a 4-layer stack
    plan_sequence_sel(ref, 'cfg1_l4', layers=4, experts=128, topk=8, world=1, tokens=64,
                  caps=[153], policy='ferry', topology=U(1, 128), steps=24)
    # multi-rank Qwen3 shapes, tight caches so eviction and the greedy fallback run
    plan_sequence_sel(ref, 'qwen_r4', layers=3, experts=128, topk=8, world=4, tokens=64,
                  caps=[40, 40, 35, 30], policy='ferry', topology=U(4, 128), steps=18)
    plan_sequence_sel(ref, 'qwen_r4_strict', layers=3, experts=128, topk=8, world=4, tokens=64,
                  caps=[40, 40, 35, 30], policy='ferry', topology=U(4, 128), steps=12, bps=0)
    plan_sequence_sel(ref, 'qwen_r8', layers=2, experts=128, topk=8, world=8, tokens=64,
                  caps=[20] * 8, policy='ferry', topology=U(8, 128), steps=12)
    plan_sequence_sel(ref, 'qwen_r4_topo', layers=3, experts=128, topk=8, world=4, tokens=64,
                  caps=[48, 30, 30, 24], policy='ferry', topology=topology_random(quota, 4, 128, rng),
                  steps=18)
    plan_sequence_sel(ref, 'qwen_r8_topo', layers=2, experts=128, topk=8, world=8, tokens=16,
                  caps=[20, 20, 20, 20, 18, 18, 18, 18], policy='ferry',
                  topology=topology_random(quota, 8, 128, rng, subsets=False), steps=10)
    plan_sequence_sel(ref, 'random_r4', layers=3, experts=128, topk=8, world=4, tokens=64,
                  caps=[40, 40, 35, 30], policy='random', topology=U(4, 128), steps=18, salt=1)
    plan_sequence_sel(ref, 'random_r3_bigseed', layers=2, experts=64, topk=6, world=3, tokens=16,
                  caps=[30, 25, 25], policy='random', topology=U(3, 64), steps=10, salt=7919,
                  event0=5000)
    plan_sequence_sel(ref, 'r2_t1', layers=2, experts=16, topk=2, world=2, tokens=1,
                  caps=[3, 2], policy='ferry', topology=U(2, 16), steps=20)
    plan_sequence_sel(ref, 'r1_small', layers=3, experts=8, topk=2, world=1, tokens=2,
                  caps=[5], policy='ferry', topology=U(1, 8), steps=20)
    plan_sequence_sel(ref, 'overflow', layers=1, experts=64, topk=6, world=2, tokens=16,
                  caps=[4, 4], policy='ferry', topology=U(2, 64), steps=2)
    plan_sequence_sel(ref, 'prob_r2', layers=2, experts=64, topk=6, world=2, tokens=16,
                  caps=[34, 30], policy='ferry', topology=U(2, 64), steps=12, score='probability')
    # the bench workload: config 1's layer inside Qwen3's 48-layer MoE stack, 30% cache
    plan_sequence_sel(ref, 'cfg1_stack48', layers=48, experts=128, topk=8, world=1, tokens=64,
                  caps=[1843], policy='ferry', topology=U(1, 128), steps=56, state_every=8)
    # the 8-GPU bench workload: the 48-layer stack's 30% cache over 8 ranks, a
    # profiled-style LUT over all 255 rank subsets; layers 0-7 revisited after
    # the cache has filled
    plan_sequence_sel(ref, 'cfg4_stack48_r8', layers=48, experts=128, topk=8, world=8, tokens=64,
                      caps=[231, 231, 231, 230, 230, 230, 230, 230], policy='ferry',
                      topology=topology_random(quota, 8, 128, rng), steps=24, state_every=8,
                      layer_order=list(range(16)) + list(range(8)))
    # DeepSeek-V2-Lite's 26-layer stack over 8 ranks (30% cache: 499 slots)
    plan_sequence_sel(ref, 'dsv2_stack26_r8', layers=26, experts=64, topk=6, world=8, tokens=16,
                      caps=[63, 63, 63, 62, 62, 62, 62, 62], policy='ferry', topology=U(8, 64),
                      steps=30, state_every=6, layer_order=list(range(20)) + list(range(10)))
    # history windows other than 128: probability rows replacing the ring
    # every update (4 x 16 rows = W), frequency rows appending and wrapping
    plan_sequence_sel(ref, 'prob_qwen_r4_w64', layers=3, experts=128, topk=8, world=4, tokens=64,
                      caps=[40, 40, 35, 30], policy='ferry', topology=U(4, 128), steps=12,
                      window=64, score='probability')
    plan_sequence_sel(ref, 'qwen_r2_w256', layers=2, experts=128, topk=8, world=2, tokens=64,
                      caps=[80, 70], policy='ferry', topology=U(2, 128), steps=12, window=256)
    # the largest expert count the uint8 ids carry, with top-16
    plan_sequence_sel(ref, 'e256_k16_r2', layers=2, experts=256, topk=16, world=2, tokens=8,
                      caps=[100, 100], policy='ferry', topology=U(2, 256), steps=12)
    # prefill-sized layers (every expert active), several layout chunks per rank
    plan_sequence_sel(ref, 'prefill_r2_t1024', layers=2, experts=128, topk=8, world=2, tokens=1024,
                      caps=[100, 90], policy='ferry', topology=U(2, 128), steps=4)
    # six ranks over a 63-subset LUT, a wide balance tolerance, RANDOM at eight
    # ranks and RANDOM with the probability score
    plan_sequence_sel(ref, 'qwen_r6_topo', layers=3, experts=128, topk=8, world=6, tokens=32,
                      caps=[30, 30, 28, 28, 26, 26], policy='ferry',
                      topology=topology_random(quota, 6, 128, rng), steps=12)
    plan_sequence_sel(ref, 'qwen_r4_bps1000', layers=3, experts=128, topk=8, world=4, tokens=64,
                      caps=[40, 40, 35, 30], policy='ferry', topology=U(4, 128), steps=12, bps=1000)
    plan_sequence_sel(ref, 'random_r8', layers=2, experts=128, topk=8, world=8, tokens=16,
                      caps=[20] * 8, policy='random', topology=U(8, 128), steps=10, salt=3)
    plan_sequence_sel(ref, 'random_prob_r4', layers=2, experts=64, topk=6, world=4, tokens=16,
                      caps=[20, 20, 18, 18], policy='random', topology=U(4, 64), steps=10,
                      score='probability')


if __name__ == '__main__':
    p = argparse.ArgumentParser()
    p.add_argument('--reference', default=os.environ.get('FERRY_REFERENCE'),
                   required='FERRY_REFERENCE' not in os.environ,
                   help='FERRY checkout (default: $FERRY_REFERENCE)')
    p.add_argument('--only', default='', help='comma-separated plan_<name> cases to (re)generate')
    main(p.parse_args())
