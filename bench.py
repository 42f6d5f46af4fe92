#!/usr/bin/env python
"""Decode throughput of FERRY's per-MoE-layer hot path on B200.

Workload (the benchmark's config 1; config 4 scales it over GPUs): Qwen3-30B-A3B
MoE layers (hidden 2048, 128 experts top-8 with renormalised softmax,
moe_intermediate 768, SwiGLU, bf16, random init N(0, 0.02)) stacked as the
model's 48 MoE layers, decode batch of 64 tokens per GPU, Zipf(1.1) router
bias and step-to-step hidden-state correlation rho = 0.5, expert cache = the
reference's global 30 % budget (floor(0.3 * 48 * 128) = 1843 slots split over
the GPUs), every expert resident in pinned host memory.  A lone 38-slot layer
cannot be planned by the reference (~45 experts are active per step and its
greedy quota asserts), so config 1's 38/128 is read as the per-layer share of
the 30 % cache of the 48-layer stack.

One step = one decode step through the 48 MoE layers (attention is not part
of the hot path): layer l routes h_l = x_l + out_{l-1} (a residual
dependency, so a layer cannot start before the previous one ends), and every
layer runs FERRY's full path: router + metadata all-gather, planner, layout,
copy-engine expert fetches, dispatch, grouped SwiGLU GEMM, combine.

value    = tokens decoded per second by the whole job (R * 64 * K / max-over-
           ranks time of K steps), inputs resident in HBM.
e2e      = the same through the public API with each step's inputs copied from
           pinned host memory and the step's output read back.
--impl reference times the reference's CPU path (the oracle port of
           ferry's planner/layout + the torch-CPU restatement of expert_ops)
           on this host's cores: the same full 48-layer steps, on the same
           seeded inputs and weights, with one persistent runtime whose cache
           warms over the warm-up steps exactly like the GPU arm's (rank 0
           alone, every rank of the job emulated in its process; the GPU only
           fills the expert pool before timing).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
METRIC = 'decode tokens/s through the 48-layer Qwen3-30B-A3B MoE stack (box, max over ranks)'


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=10)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impl', default='ferry_b200', choices=['ferry_b200', 'reference', 'reference-gpu'],
                   help='reference: the reference CPU path on the host cores (the driver\'s arm); '
                        'reference-gpu: the reference runtime on the GPUs (oracle/ref_runtime.py), '
                        'an extra comparator record')
    p.add_argument('--layers', type=int, default=48)
    p.add_argument('--tokens', type=int, default=64)
    p.add_argument('--cache-ratio', type=float, default=0.3)
    p.add_argument('--pool-layers', type=int, default=0, help='0 = as many as host RAM allows')
    p.add_argument('--policy', default='ferry', choices=['ferry', 'random'])
    # the reference's run_cell.py options of the policy
    p.add_argument('--history-window', type=int, default=128)
    p.add_argument('--eviction-score', default='frequency', choices=['frequency', 'probability'])
    p.add_argument('--balance-tol-bps', type=int, default=200)
    p.add_argument('--salt', type=int, default=1)
    p.add_argument('--copy-streams', type=int, default=1)
    p.add_argument('--no-e2e', action='store_true')
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--cpu-seconds', type=float, default=12.0)
    p.add_argument('--ep-sweep', default='',
                   help='comma-separated tokens per rank: time the EP dispatch + combine of one Qwen3 '
                        'MoE layer with every expert cached (no fetches) instead of the decode bench')
    p.add_argument('--gemm-compare', type=int, default=0, metavar='EXPERTS',
                   help='time the routed-expert GEMM of one decode layer (64 tokens, top-8 of 128, '
                        'Zipf(1.1), this many cached experts) through this library\'s execute_experts '
                        '(the fused tcgen05 kernel) and the reference\'s (oracle/_ref, cuBLAS per expert)')
    p.add_argument('--full-model', choices=['qwen3', 'deepseek'],
                   help='the benchmark\'s configs 2-4: the whole model (transformers 5.5, random weights) with '
                        'its MoE blocks on this runtime; reports TTFT, TPOT and decode tokens/s')
    p.add_argument('--checkpoint', default='',
                   help='--full-model: a local checkpoint directory (config.json + safetensors) '
                        'to load instead of random weights')
    p.add_argument('--batch', type=int, default=64, help='--full-model: sequences per GPU')
    p.add_argument('--prompt-len', type=int, default=1024, help='--full-model: input tokens')
    p.add_argument('--new-tokens', type=int, default=64, help='--full-model: greedy output tokens')
    p.add_argument('--topology', default='auto',
                   help='quota LUT for N > 1: "auto" (default) profiles the host links of these GPUs '
                        'at start-up (every subset of ranks copying at once) and builds the LUT; '
                        '"uniform"; or a topology JSON from ferry_b200.build_quota_lut')
    p.add_argument('--per-rank-pool', action='store_true',
                   help='one pinned expert pool per rank (the reference\'s layout) instead of one '
                        'shared pool per node')
    p.add_argument('--launch-log', default='',
                   help='write, for every layer run (warm-up and timed, in order), its cached and '
                        'fetched expert counts as JSON: the expert-GEMM launches an ncu capture '
                        'of this command lists, with their algorithmic bytes')
    p.add_argument('--phase-stamps', action='store_true',
                   help='after timing, run one more step with the planner\'s and the layout\'s '
                        'device-clock phase stamps on (a host sync after every layer) and report '
                        'the median of each phase')
    p.add_argument('--sync-fetch', action='store_true',
                   help='issue each layer\'s copies before its fetched-expert GEMM and wait on '
                        'them from the stream (for profilers that serialise GPU work)')
    return p.parse_args()


def init_dist(n_gpus):
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group('nccl', device_id=torch.device('cuda', local),
                                timeout=timedelta(seconds=180))
    return rank, world, local


def max_over_ranks(x, world):
    t = torch.tensor([x], dtype=torch.float64, device='cuda')
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self):
        self.rows, self.proc, self.thread = [], None, None

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(',')])

    def stop(self, gpu_indices):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for r in self.rows:
            try:
                if int(r[0]) not in gpu_indices:
                    continue
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for name, v in zip(names, r[5:9]):
                    if v.lower() == 'active':
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': max(mx), 'reasons': sorted(reasons),
                'samples': len(sm)}


def measured_peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        d = json.loads(path.read_text())
        return d.get('hbm_gbs', 6650.0), d.get('bf16_tflops_sustained', 1400.0), 'measured'
    return 6650.0, 1400.0, 'fallback'


def ncu_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = ROOT / 'profiles' / 'swiglu_fused_kernel_traffic.json'
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            return None
    return None


def host_link_gbs(cache_row, pool, n=12):
    """Pinned host -> HBM bandwidth of expert-sized copies on a copy stream."""
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for i in range(4):
            cache_row[i % cache_row.shape[0]].copy_(pool[i % pool.shape[0]], non_blocking=True)
    s.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for i in range(n):
            cache_row[i % cache_row.shape[0]].copy_(pool[(i * 7) % pool.shape[0]], non_blocking=True)
        e1.record(s)
    e1.synchronize()
    return n * pool[0].numel() * 2 / (e0.elapsed_time(e1) / 1e3) / 1e9


def auto_pool_layers(spec, world, requested):
    if requested:
        return min(requested, spec.layers)
    per_layer = spec.experts * spec.expert_bytes
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except ImportError:
        avail = 64 << 30
    fit = int(avail * 0.55 // (per_layer * world))
    return max(1, min(spec.layers, fit))


def policy_opts(a):
    return dict(window=a.history_window, balance_tol_bps=a.balance_tol_bps, salt=a.salt,
                score=a.eviction_score)


def bench_config(a, spec, world, T, caps):
    """The workload both arms run; the driver compares the two lines' config."""
    return {'workload': f'config 1 (Qwen3-30B-A3B MoE layer, decode batch {T}/GPU) in the '
                        f'{spec.layers}-layer MoE stack, 30% global expert cache, all experts in '
                        'pinned host memory',
            'moe_layers': spec.layers, 'global_batch': world * T, 'tokens_per_gpu': T, 'seq_len': 1,
            'parallelism': f'dp{world}-ep{world}', 'cache_slots_per_rank': caps, 'policy': a.policy,
            **policy_opts(a),
            'inputs': 'seeded: router gates + Zipf(1.1) biases seed 0, expert pool seed 1 '
                      '(N(0,0.02) bf16), hidden states seed 1000+rank (N(0,1), rho 0.5), '
                      'layer l routes x_l + out_(l-1)',
            'l2': 'no flush: each layer step reads > 126 MB of expert weights (> L2)'}


def make_inputs(spec, T, world, ranks, n_steps):
    """inputs[r][i]: rank r's [layers, T, H] bf16 hidden states of step i (CPU),
    the same for every arm."""
    from ferry_b200.workload import HiddenStream
    out = {}
    for r in ranks:
        hs = HiddenStream(spec, T, 0.5, 1000 + r, 'cpu')
        out[r] = [torch.stack([hs.next(l) for l in range(spec.layers)]) for _ in range(n_steps)]
    return out


PARITY_LAYERS = 3  # layers of the first warm-up step the parity gate replays
SPAN_LAYERS = 4096  # device-clock spans recorded per collect (ferryb_layer_stats.kernel_us)
KERNELS = ['router', 'planner', 'layout', 'dispatch', 'permute', 'gemm_cached', 'gemm_fetched',
           'combine', 'final_scatter']


def make_topology(a, spec, rank, world, pool, dev):
    """(Topology, note): the quota LUT of this run (see --topology)."""
    from ferry_b200.build_quota_lut import topology_for_run
    return topology_for_run(a.topology, spec, rank, world, pool_row=pool[0], device=dev)


def qwen3_spec(layers):
    from ferry_b200.model import QWEN3_30B_A3B, spec_from_config
    c = dict(QWEN3_30B_A3B)
    c['num_hidden_layers'] = layers
    return spec_from_config(c)


# ---------------------------------------------------------------------------
def run_ours(a, rank, world, local):
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import SyntheticMoE
    dev = torch.device('cuda', local)
    spec = qwen3_spec(a.layers)
    T, L = a.tokens, spec.layers
    caps = spec.cache_slots(a.cache_ratio, world)
    shared = world > 1 and not a.per_rank_pool
    pool_layers = auto_pool_layers(spec, 1 if shared else world, a.pool_layers)
    t0 = time.time()
    wl = SyntheticMoE(spec, seed=0, device=dev, pool_layers=pool_layers, shared=shared)
    setup_s = time.time() - t0
    topo, topo_note = make_topology(a, spec, rank, world, wl.pool, dev)
    rt = OffloadRuntime(spec, wl.pool, caps, a.policy, topo, history_window=a.history_window,
                        balance_tol_bps=a.balance_tol_bps, salt=a.salt, eviction_score=a.eviction_score,
                        n_copy_streams=a.copy_streams, timing=True, sync_fetch=a.sync_fetch)
    # this rank's link alone (ranks take turns), then with every rank copying at once
    b_alone = 0.0
    for r in range(world):
        barrier(world)
        if r == rank:
            b_alone = host_link_gbs(rt.cache, wl.pool)
    barrier(world)
    b_host = host_link_gbs(rt.cache, wl.pool)
    n_steps = a.warmup + a.steps
    host = make_inputs(spec, T, world, [rank], n_steps)[rank]
    inputs = [x.to(dev) for x in host]

    def step(inp, capture=None):
        prev = None
        for l in range(L):
            h = inp[l] if prev is None else inp[l] + prev
            if capture is not None and l < PARITY_LAYERS:
                sel = torch.empty((T, spec.topk), dtype=torch.int64, device=dev)
                w = torch.empty((T, spec.topk), dtype=torch.bfloat16, device=dev)
                prev = rt.forward(l, h, wl.gate[l], wl.bias[l], sel, w)
                capture['layers'].append((h.cpu(), sel.cpu(), w.cpu(), prev.cpu()))
                if l == PARITY_LAYERS - 1:
                    ctl = rt.controller
                    capture['state'] = (ctl.slots.copy(), ctl.owner.copy(), ctl.last.copy())
            else:
                prev = rt.forward(l, h, wl.gate[l], wl.bias[l])
            if launch_log is not None:
                summ = rt.last_summary(T)
                launch_log.append({'layer': l, 'cached_experts': int(summ.n_hit),
                                   'fetched_experts': int(summ.n_fetch_mine), 'routes': int(summ.n_routes)})
        return prev

    launch_log = [] if a.launch_log else None
    # the first layers of the first warm-up step are recorded (inputs, this
    # rank's routing and outputs, the replicated cache state) for the parity
    # gate that runs after timing
    capture = {'layers': [], 'state': None}
    for i in range(a.warmup):
        step(inputs[i], capture if i == 0 else None)
    torch.cuda.synchronize()
    ex = rt._executor(T)
    from ferry_b200._lib import call
    call('ferryb_layer_collect_timing', ex.h)
    call('ferryb_layer_reset_stats', ex.h)
    copies0 = rt.h2d.copies
    fetch0 = rt.fetches_per_rank.copy()  # every rank's fetches (the replicated plan's counts)
    barrier(world)
    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(a.steps):
        step(inputs[a.warmup + i])
    ev1.record()
    ev1.synchronize()
    barrier(world)
    clocks = sampler.stop([local]) if sampler else None
    ms_local = ev0.elapsed_time(ev1)
    call('ferryb_layer_collect_timing', ex.h)
    st = ex.stats()
    fetch_copies = rt.h2d.copies - copies0
    f_job = (rt.fetches_per_rank - fetch0).astype(np.float64)  # the timed steps only
    ms = max_over_ranks(ms_local, world)

    # e2e: inputs from pinned host memory each step, output read back each step
    e2e = None
    if not a.no_e2e:
        host_inputs = [x.pin_memory() for x in host[a.warmup:]]
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(a.steps):
            inp = host_inputs[i].to(dev, non_blocking=True)
            out = step(inp)
            out.cpu()
        e1.record()
        e1.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
        e2e = {'value': world * T * a.steps / (e2e_ms / 1e3), 'unit': 'tokens/s',
               'h2d_bytes_per_step': int(host_inputs[0].numel() * 2),
               'd2h_bytes_per_step': int(T * spec.hidden * 2), 'ms_per_step': e2e_ms / a.steps}

    hbm_gbs, bf16_tflops, peak_kind = measured_peaks()
    layers_timed = max(1, st.timed_layers)
    sampled = max(1, min(st.timed_layers, SPAN_LAYERS))
    # dominant kernel: the grouped SwiGLU over cached experts (HBM-bound at decode)
    gemm_us = st.phase_us[2]
    achieved = st.hit_weight_bytes / (gemm_us * 1e-6) / 1e9 if gemm_us > 0 else 0.0
    traffic = ncu_traffic()
    roofline = {'kernel': 'swiglu_gemm_kernel (cached experts, both phases)', 'bound': 'hbm',
                'achieved': round(achieved, 1), 'peak': hbm_gbs, 'unit': 'GB/s',
                'frac': round(achieved / hbm_gbs, 4), 'peak_source': peak_kind,
                'algorithmic_bytes_per_layer': st.hit_weight_bytes / layers_timed,
                'traffic': (round(traffic['traffic_per_algorithmic_byte'] * st.hit_weight_bytes /
                                  max(1, st.layers)) if traffic and st.hit_experts else None),
                'traffic_note': (traffic.get('note') if traffic else 'no ncu capture committed')}
    if st.hit_gemm_kernel_launches:
        # the same launches on the device clock (earliest CTA start to latest CTA
        # end), over exactly the launches whose spans were recorded: CUDA events
        # on the compute stream also absorb the command-fetch delay the host
        # link's saturating expert copies impose on every compute-stream command
        clk_us = st.hit_gemm_kernel_us / st.hit_gemm_kernel_launches
        clk = st.hit_gemm_kernel_bytes / (st.hit_gemm_kernel_us * 1e-6) / 1e9
        roofline['device_clock'] = {'achieved': round(clk, 1), 'frac': round(clk / hbm_gbs, 4),
                                    'launch_us': round(clk_us, 1),
                                    'launches': int(st.hit_gemm_kernel_launches),
                                    'event_launch_us': round(gemm_us / layers_timed, 1)}
    # per-layer roofline: slowest of host-link fetch, NVLink exchange, tensor FLOPs
    expert_bytes = spec.expert_bytes
    fetch_bytes = st.fetches * expert_bytes
    nvl_bytes = st.dispatch_bytes + st.combine_bytes
    flops = st.routes * 6 * spec.hidden * spec.intermediate
    t_host = fetch_bytes / (b_host * 1e9)
    t_nvl = nvl_bytes / 770e9
    t_flops = flops / (bf16_tflops * 1e12)
    t_roof = max(t_host, t_nvl, t_flops)
    t_meas = ms_local / 1e3
    # host-link term of the job: ranks that share a host path move their
    # fetched bytes at that path's measured aggregate bandwidth
    alone = [b_alone] * world
    if world > 1:
        dist.all_gather_object(alone, b_alone)
    t_host_job, limiting = host_link_time(topo, topo_note, f_job * expert_bytes, alone, b_host, world)
    t_roof_job = max(t_host_job, max_over_ranks(t_nvl, world), max_over_ranks(t_flops, world))
    # the job's layer is as slow as its slowest rank
    t_meas_job = max_over_ranks(t_meas, world)
    terms = [t_host_job, max_over_ranks(t_nvl, world), max_over_ranks(t_flops, world)]
    layer_roofline = {'bound': ['host_link', 'nvlink', 'tensor'][int(np.argmax(terms))],
                      'frac': round(t_roof_job / t_meas_job, 4) if t_meas_job > 0 else None,
                      'host_link_limiting': limiting,
                      'fetches_per_layer_by_rank': [round(x / max(1, st.layers), 2) for x in f_job],
                      'frac_rank0_own_link': round(t_roof / t_meas, 4) if t_meas > 0 else None,
                      'host_link_gbs_measured': round(b_host, 2),
                      'host_link_gbs_alone': round(b_alone, 2),
                      'host_link_note': 'measured with every rank copying at once (shared PCIe '
                                        'switches / host memory); alone = this rank only',
                      'topology': topo_note,
                      'fetch_gbs_achieved': round(fetch_bytes / t_meas / 1e9, 2),
                      'fetches_per_layer': st.fetches / max(1, st.layers),
                      'nvlink_bytes_per_layer': nvl_bytes / max(1, st.layers),
                      'rank': rank}
    split = {name: round(st.phase_us[i] / layers_timed, 1) for i, name in enumerate(
        ['route_plan', 'layout_summary_dispatch_permute', 'gemm_cached', 'gemm_fetched_incl_wait',
         'combine'])}
    result = {
        'metric': METRIC, 'value': world * T * a.steps / (ms / 1e3), 'unit': 'tokens/s',
        'n_gpus': world, 'steps': a.steps, 'warmup': a.warmup, 'ms_per_step': ms / a.steps,
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16',
        'data': 'synthetic: random-init N(0,0.02) weights, N(0,1) hidden states rho=0.5, Zipf(1.1) router bias',
        'config': bench_config(a, spec, world, T, caps),
        'pool': {'layers': pool_layers,
                 'kind': 'one shared pinned pool per node' if shared else 'pinned pool per rank'},
        'topology': topo_note,
        'roofline': roofline, 'layer_roofline': layer_roofline, 'layer_split_us': split,
        'gpu_launches': int(st.launches), 'h2d_expert_copies': int(fetch_copies),
        'host_wait_us_per_layer': round(st.host_wait_us / max(1, st.layers), 1),
        'host_issue_us_per_layer': {name: round(st.host_us[i] / max(1, st.layers), 1) for i, name in enumerate(
            ['route_plan_layout', 'first_fetch', 'dispatch_permute', 'gemm_cached', 'gemm_fetched_fetches',
             'combine'])},
        'copy_lane_us_per_layer': {name: round(st.copy_us[i] / layers_timed, 1) for i, name in enumerate(
            ['plan_end_to_first_copy', 'copies', 'last_copy_to_combine_end'])},
        # per-MoE-layer split on the device clock: each kernel's span (earliest
        # CTA start to latest CTA end), summed over the layers whose spans were
        # recorded (the first 4096 timed layers) and divided by their number
        'kernel_us_per_layer_device_clock': {name: round(st.kernel_us[i] / sampled, 1)
                                             for i, name in enumerate(KERNELS) if st.kernel_launches[i]},
        'kernel_us_per_launch_device_clock': {
            name: {'us': round(st.kernel_us[i] / st.kernel_launches[i], 1),
                   'launches': int(st.kernel_launches[i])}
            for i, name in enumerate(KERNELS) if st.kernel_launches[i]},
        'setup_s': round(setup_s, 1), 'e2e': e2e, 'clocks': clocks,
    }
    if launch_log is not None:
        Path(a.launch_log).write_text(json.dumps({
            'expert_bytes': spec.expert_bytes,
            'note': 'per layer in run order; the expert GEMM launches once for the cached experts '
                    '(if any) and once for the fetched experts (if any)',
            'layers': launch_log}))
    if a.phase_stamps:
        result['phase_stamps_ns'] = phase_stamps(rt, wl, spec, inputs[a.warmup], dev)
    result['parity'] = parity_gate(spec, wl.pool, caps, a, topo, capture, rank, world)
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        result['cpu_baseline'] = cpu_baseline(spec, wl, caps, T, a.cpu_seconds, a, host)
    result['self_check'] = self_check(result)
    rt.close()
    return result


PLAN_PHASES = ['gate_history', 'demand_capacity', 'quota_assignment', 'victim_positions',
               'victim_order', 'commit', 'tail']
ORDER_STEPS = ['read_classify', 'clean_dirty_split', 'dirty_sort', 'merge']
LAYOUT_PHASES = ['fetched_experts', 'send_side', 'receive_pass1_starts', 'receive_pass2',
                 'groups_summary', 'host_mirror']


def phase_stamps(rt, wl, spec, inp, dev):
    """One more decode step, after timing, with the planner's and the layout's
    %globaltimer phase stamps on (ferryb_debug_plan_timestamps /
    ferryb_debug_layout_timestamps) and a host sync after every layer: the
    median over the step's layers of each phase, in ns."""
    from ferry_b200._lib import call, ptr
    pts = torch.zeros(16, dtype=torch.int64, device=dev)
    lts = torch.zeros(8, dtype=torch.int64, device=dev)
    rts = torch.zeros(4, dtype=torch.int64, device=dev)
    plan, order, lay, rout = [], [], [], []
    call('ferryb_debug_plan_timestamps', ptr(pts))
    call('ferryb_debug_layout_timestamps', ptr(lts))
    call('ferryb_debug_router_timestamps', ptr(rts))
    try:
        prev = None
        for l in range(spec.layers):
            pts.zero_()
            lts.zero_()
            rts.zero_()
            rts[0] = torch.iinfo(torch.int64).max
            h = inp[l] if prev is None else inp[l] + prev
            prev = rt.forward(l, h, wl.gate[l], wl.bias[l])
            torch.cuda.synchronize()
            t, u, v = pts.cpu().numpy(), lts.cpu().numpy(), rts.cpu().numpy()
            if np.all(v[1:] > 0) and np.all(np.diff(v) >= 0):
                rout.append(np.append(np.diff(v), t[0] - v[3]))
            if np.all(t[:8] > 0) and np.all(np.diff(t[:8]) >= 0):  # a layer with fetches
                plan.append(np.diff(t[:8]))
                if np.all(t[8:12] > 0):  # the saved victim order was used
                    order.append(np.append(np.diff(np.concatenate([t[4:5], t[8:12]])), t[12]))
            if np.all(u[:7] > 0) and np.all(np.diff(u[:7]) >= 0):
                lay.append(np.diff(u[:7]))
    finally:
        call('ferryb_debug_plan_timestamps', None)
        call('ferryb_debug_layout_timestamps', None)
        call('ferryb_debug_router_timestamps', None)

    def med(rows, names):
        return {n: float(np.median([r[i] for r in rows])) for i, n in enumerate(names)} if rows else None
    return {'layers': {'router': len(rout), 'planner': len(plan), 'victim_order_saved': len(order),
                       'layout': len(lay)},
            'router': med(rout, ['logits', 'softmax_topk', 'gather_writes', 'router_end_to_planner_start']),
            'planner': med(plan, PLAN_PHASES), 'victim_order_steps': med(order, ORDER_STEPS + ['dirty_records']),
            'layout': med(lay, LAYOUT_PHASES),
            'note': 'device-clock stamps of one step run after timing with a host sync per layer: '
                    'no copies in flight while the router and planner run; the layer\'s first '
                    'copy is in flight while the layout runs (its host-mirror fence waits on the link)'}


def parity_gate(spec, pool, caps, a, topo, capture, rank, world):
    """Outside the timed region: the oracle (oracle/layer.py, every rank of the
    job emulated in rank 0's process, on the run's own LUT) replays the first
    PARITY_LAYERS layers of the first warm-up step with each rank's recorded
    inputs and routing.  The replicated cache state (slots, owner, last use)
    of every rank must equal the oracle's bit for bit, and every rank's layer
    outputs must be within the BF16 tolerance (2e-2 abs, 1e-2 of max |ref|)."""
    if a.warmup < 1:
        return None
    mine = {'layers': capture['layers'], 'state': capture['state']}
    gathered = [None] * world
    if world > 1:
        dist.all_gather_object(gathered, mine)
    else:
        gathered = [mine]
    if rank != 0:
        return None
    from oracle.layer import OracleRuntime
    orc = OracleRuntime(spec, pool, caps, a.policy, topo.masks, topo.seconds, topo.lut,
                        window=a.history_window, balance_tol_bps=a.balance_tol_bps, salt=a.salt,
                        score=a.eviction_score)
    if a.eviction_score == 'probability':
        return {'skipped': 'the gate replays the frequency score only'}
    max_abs, max_rel, ok_out = 0.0, 0.0, True
    for l in range(len(mine['layers'])):
        per = [g['layers'][l] for g in gathered]
        want, _, _ = orc.execute(l, [p[0] for p in per], [p[1] for p in per], [p[2] for p in per])
        for r in range(world):
            err = (per[r][3].float() - want[r].float()).abs().max().item()
            scale = want[r].float().abs().max().item()
            max_abs = max(max_abs, err)
            max_rel = max(max_rel, err / max(scale, 1e-30))
            ok_out = ok_out and err <= 2e-2 and err <= 1e-2 * max(scale, 1e-30)
    same = all(np.array_equal(g['state'][0], orc.ctl.slots) and np.array_equal(g['state'][1], orc.ctl.owner)
               and np.array_equal(g['state'][2], orc.ctl.last) for g in gathered)
    res = {'layers': len(mine['layers']), 'ranks': world,
           'decisions': 'bit-exact' if same else 'DIFFER', 'max_abs': max_abs,
           'max_rel': round(max_rel, 6), 'outputs_within_tolerance': ok_out, 'ok': bool(same and ok_out)}
    if not res['ok']:
        print(f'bench parity gate failed: {res}', file=sys.stderr)
    return res


def host_link_time(topo, topo_note, fetch_bytes, alone_gbs, all_gbs, world):
    """Lower bound on the time the job's expert copies take: every group of
    ranks that shares a host path moves the bytes its ranks fetch at that
    group's aggregate bandwidth.  With a profiled topology the groups are its
    domains (every subset of the ranks, each with the bandwidth measured while
    that subset copies at once, as the quota LUT uses them); without one, each
    rank alone at its own measured link and all ranks together at the
    bandwidth measured while every rank copies.  fetch_bytes: per rank.
    Returns (seconds, the limiting group)."""
    groups = []
    if topo_note != 'uniform':  # profiled on this box, or a topology file
        for mask, sec in zip(topo.masks, topo.seconds):
            groups.append((int(mask), (1 << 30) / float(sec)))
    else:
        groups = [(1 << r, alone_gbs[r] * 1e9) for r in range(world)]
        if world > 1:
            groups.append(((1 << world) - 1, all_gbs * 1e9 * world))
    best, lim = 0.0, None
    for mask, bw in groups:
        b = sum(fetch_bytes[r] for r in range(world) if mask >> r & 1)
        t = b / bw
        if t > best:
            best, lim = t, {'ranks': [r for r in range(world) if mask >> r & 1], 'gbs': round(bw / 1e9, 2)}
    return best, lim


def self_check(result):
    """Fractions of a measured peak above 1.2 mean the timed kernel did not do
    the work counted for it (a bookkeeping error): flag them in the line."""
    problems = []
    roof = result.get('roofline') or {}
    for name, frac in (('roofline', roof.get('frac')),
                       ('roofline.device_clock', (roof.get('device_clock') or {}).get('frac')),
                       ('layer_roofline', (result.get('layer_roofline') or {}).get('frac'))):
        if frac is not None and frac > 1.2:
            problems.append(f'{name}.frac = {frac} > 1.2')
    par = result.get('parity')
    if par and par.get('ok') is False:
        problems.append('parity gate failed')
    for p in problems:
        print(f'bench self-check: {p}', file=sys.stderr)
    return {'ok': not problems, 'problems': problems}


# ---------------------------------------------------------------------------
def run_ep_sweep(a, rank, world, local):
    """The benchmark's config-4 EP sweep: one Qwen3 MoE layer (top-8 of 128, Zipf
    1.1 router bias), T tokens per rank, the 128 experts spread over the ranks'
    caches (128 slots in all) so that, once warm, no step fetches: the step is
    router + planner + layout + P2P dispatch + grouped GEMM + P2P combine.
    Reports per T the dispatch (+ permute) and combine times (CUDA events on
    the compute stream, max over ranks) and the NVLink bytes they move."""
    from ferry_b200._lib import call
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import SyntheticMoE
    dev = torch.device('cuda', local)
    spec = qwen3_spec(1)
    caps = spec.cache_slots(1.0, world)
    wl = SyntheticMoE(spec, seed=0, device=dev, shared=world > 1)
    rt = OffloadRuntime(spec, wl.pool, caps, 'ferry', Topology.uniform(world, spec.experts), timing=True)
    rows = []
    for T in [int(t) for t in a.ep_sweep.split(',') if t]:
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        xs = [torch.randn(T, spec.hidden, generator=gen, device=dev).to(torch.bfloat16) for _ in range(4)]
        for i in range(a.warmup):
            rt.forward(0, xs[i % 4], wl.gate[0], wl.bias[0])
        torch.cuda.synchronize()
        ex = rt._executor(T)
        call('ferryb_layer_collect_timing', ex.h)
        call('ferryb_layer_reset_stats', ex.h)
        barrier(world)
        for i in range(a.steps):
            rt.forward(0, xs[i % 4], wl.gate[0], wl.bias[0])
        torch.cuda.synchronize()
        call('ferryb_layer_collect_timing', ex.h)
        st = ex.stats()
        n = max(1, st.timed_layers)
        disp = max_over_ranks(st.dispatch_permute_us / n, world)
        comb = max_over_ranks(st.phase_us[4] / n, world)
        comb_store = max_over_ranks(st.combine_store_us / n, world)
        layer = max_over_ranks(sum(st.phase_us[i] for i in range(5)) / n, world)
        nvl = torch.tensor([float(st.dispatch_bytes + st.combine_bytes) / n], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(nvl)
        fetches = max_over_ranks(float(st.fetches), world)
        rows.append({'tokens_per_rank': T, 'dispatch_permute_us': round(disp, 1),
                     'combine_store_us': round(comb_store, 1), 'combine_incl_peer_wait_us': round(comb, 1),
                     'layer_us': round(layer, 1), 'nvlink_bytes_all_ranks': int(nvl.item()),
                     'nvlink_gbs_per_rank': round(float(nvl.item()) / world / ((disp + comb_store) * 1e-6) / 1e9, 1),
                     'fetches_in_timed_steps': int(fetches)})
    rt.close()
    return {'metric': 'EP dispatch + combine of one Qwen3 MoE layer (P2P over NVSwitch)', 'n_gpus': world,
            'steps': a.steps, 'warmup': a.warmup, 'dtype': 'bf16', 'data': 'synthetic',
            'config': {'workload': 'config 4 EP sweep: H=2048, top-8 of 128, Zipf(1.1), all experts cached',
                       'cache_slots_per_rank': caps},
            'nvlink_peer_gbs_reference': 770.0, 'ep_sweep': rows}


def _reference_gpu_model_run(cfg, a, rank, world, dev, layers):
    """The full model with the reference's MoE hooks (ferry/model.py:137-158)
    over the composed reference GPU runtime (oracle/ref_runtime.py): the same
    model, weights, prompts and metrics as ferry_b200.harness.run."""
    from ferry_b200.build_quota_lut import topology_for_run
    from ferry_b200.harness import build_model, decode_metrics, generate
    from ferry_b200.workload import SyntheticMoE
    from oracle.ref_runtime import RefGpuRuntime
    if not dist.is_initialized():
        os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
        os.environ.setdefault('MASTER_PORT', '29582')
        dist.init_process_group('nccl', rank=0, world_size=1, device_id=dev, timeout=timedelta(seconds=180))
    overrides = {'num_hidden_layers': layers} if layers else {}
    model, spec = build_model(cfg, dev, 0, **overrides)
    wl = SyntheticMoE(spec, seed=1, device=dev, shared=world > 1)
    caps = spec.cache_slots(a.cache_ratio, world)
    topo, topo_note = topology_for_run(a.topology, spec, rank, world, pool_row=wl.pool[0], device=dev)

    def make_rt():
        return RefGpuRuntime(spec, wl.pool, caps, a.policy, topo.masks, topo.seconds, topo.lut)
    state = {'rt': make_rt()}
    scaling = float(cfg.get('routed_scaling_factor', 1.0))
    for layer, idx in enumerate(spec.moe_layers):
        mlp = model.model.layers[idx].mlp
        gate = mlp.gate.weight
        shared = getattr(mlp, 'shared_experts', None)

        def forward(hidden_states, _layer=layer, _gate=gate, _shared=shared):
            rt = state['rt']
            shape = hidden_states.shape
            flat = hidden_states.reshape(-1, shape[-1])
            if spec.model_type == 'qwen3_moe':
                sel, w = rt.route(flat, _gate)
            else:  # transformers' DeepseekV2 greedy routing, no renormalisation
                probs = torch.softmax(torch.nn.functional.linear(flat.float(), _gate.float()), -1)
                w, sel = torch.topk(probs, spec.topk, dim=-1)
                w = (w * scaling).to(flat.dtype)
            out = rt.execute(_layer, flat, sel, w)
            if _shared is not None:
                out = out + _shared(flat)
            return out.view(shape)
        mlp.forward = forward
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    prompts = torch.randint(0, cfg['vocab_size'], (a.batch, a.prompt_len), generator=g, device=dev)
    generate(model, prompts, min(a.new_tokens, 4))
    state['rt'].close()
    state['rt'] = make_rt()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    tokens, times = generate(model, prompts, a.new_tokens)
    m = decode_metrics(times, a.batch, world)
    m.update(fetches_per_rank=state['rt'].fetches_per_rank.tolist(), decode_fetches_per_rank=None,
             topology=topo_note)
    state['rt'].close()
    return m


def run_full_model(a, rank, world, local):
    """The benchmark's configs 2-4 through ferry_b200.harness: seeded random prompts
    (uniform token ids), one warm-up generation, then one timed generation.
    With --impl reference-gpu the same model runs the reference's hooks over
    the composed reference GPU runtime instead."""
    from ferry_b200.harness import run
    from ferry_b200.model import DEEPSEEK_V2_LITE, QWEN3_30B_A3B
    cfg = QWEN3_30B_A3B if a.full_model == 'qwen3' else DEEPSEEK_V2_LITE
    dev = torch.device('cuda', local)
    layers = a.layers if a.layers != 48 else None
    if a.impl == 'reference-gpu':
        m = _reference_gpu_model_run(cfg, a, rank, world, dev, layers)
    else:
        model, rt, tokens, m = run(cfg, batch=a.batch, prompt_len=a.prompt_len, new_tokens=a.new_tokens,
                                   cache_ratio=a.cache_ratio, layers=layers, warmup=1, rank=rank,
                                   world=world, device=dev, policy=a.policy, topology=a.topology,
                                   checkpoint=a.checkpoint or None)
        rt.close()
    name = 'Qwen3-30B-A3B' if a.full_model == 'qwen3' else 'DeepSeek-V2-Lite'
    return {'metric': f'decode tokens/s, full {name} (box, max over ranks)', 'impl': a.impl,
            'value': m['decode_tokens_per_s'], 'unit': 'tokens/s', 'n_gpus': world, 'steps': a.new_tokens,
            'warmup': 1, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16',
            'data': (f'checkpoint {a.checkpoint}, seeded uniform token ids' if a.checkpoint else
                     'synthetic: random-init weights, seeded uniform token ids'),
            'config': {'workload': f'config {"3/4" if a.full_model == "qwen3" else "2"}: full {name}',
                       'batch_per_gpu': a.batch, 'prompt_len': a.prompt_len, 'new_tokens': a.new_tokens,
                       'cache_ratio': a.cache_ratio, 'layers': layers or cfg['num_hidden_layers'],
                       'policy': a.policy, 'topology': m['topology'],
                       'parallelism': f'dp{world}-ep{world}'},
            'ttft_ms': round(m['ttft_ms'], 1), 'tpot_ms': round(m['tpot_ms'], 2),
            'total_tokens_per_s': m['total_tokens_per_s'],
            'fetches_per_rank': m['fetches_per_rank'], 'decode_fetches_per_rank': m['decode_fetches_per_rank']}


def reference_steps(spec, pool, gates, biases, caps, a, inputs, warmup, steps, budget_s=None):
    """The reference's CPU path (oracle port: C planner/layout + torch-CPU
    expert ops, every rank of the job emulated in this process) over full
    decode steps: layer l of step i routes inputs[r][i][l] + out_(l-1) with the
    hook's router, as the GPU arm does, through one persistent runtime.  Runs
    `warmup` untimed steps, then `steps` timed ones (fewer if `budget_s` runs
    out, at least two); returns the timed steps' seconds."""
    from oracle import expert_ops as ops
    from oracle import planner as op
    from oracle.layer import OracleRuntime
    world = len(caps)
    masks = np.asarray([1 << r for r in range(world)], np.int64)
    sec = np.ones(world)
    lut = op.build_lut(spec.experts, world, masks, sec)
    orc = OracleRuntime(spec, pool, caps, a.policy, masks, sec, lut, window=a.history_window,
                        balance_tol_bps=a.balance_tol_bps, salt=a.salt, score=a.eviction_score)
    prob = a.eviction_score == 'probability'
    bf16 = torch.bfloat16

    def step(i):
        prev = [None] * world
        for l in range(spec.layers):
            xs = []
            for r in range(world):
                x = inputs[r][i][l]
                xs.append(x if prev[r] is None else (x.float() + prev[r].float()).to(bf16))
            routed = [ops.route_qwen3(x, gates[l], spec.topk, True, biases[l]) for x in xs]
            prev, _, _ = orc.execute(l, xs, [q[0] for q in routed], [q[1] for q in routed],
                                     [q[2] for q in routed] if prob else None)
        return prev

    for i in range(warmup):
        step(i)
    times, t_start = [], time.perf_counter()
    for i in range(warmup, warmup + steps):
        t0 = time.perf_counter()
        step(i)
        times.append(time.perf_counter() - t0)
        if budget_s is not None and len(times) >= 2 and time.perf_counter() - t_start >= budget_s:
            break
    return times


def cpu_baseline(spec, wl, caps, T, seconds, a, host):
    """cpu_baseline of the GPU arm's line: the reference arm's measurement on a
    bounded sample (one warm-up step, then as many full steps as fit in
    `seconds`) of the same inputs."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gates = [g.cpu() for g in wl.gate]
    biases = [b.cpu() for b in wl.bias]
    n = len(host) - 1
    times = reference_steps(spec, wl.pool, gates, biases, caps, a, {0: host}, 1, n, budget_s=seconds)
    step_s = sum(times) / len(times)
    return {'value': T / step_s, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
            'sample': f'{len(times)} full {spec.layers}-layer decode steps (after 1 warm-up step) of the '
                      f'same inputs through the oracle port (C planner/layout + torch-CPU expert ops), '
                      f'{step_s * 1e3:.0f} ms/step'}


def run_reference(a, rank, world):
    """The reference's CPU path on this host's cores (rank 0 only), on the GPU
    arm's workload: the same config, inputs and weights, full steps."""
    from ferry_b200.workload import SyntheticMoE
    spec = qwen3_spec(a.layers)
    T = a.tokens
    caps = spec.cache_slots(a.cache_ratio, world)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    dev = 'cuda' if torch.cuda.is_available() else 'cpu'
    pool_layers = auto_pool_layers(spec, 1, a.pool_layers)
    # the GPU only draws the expert pool (seeded, as the GPU arm draws it)
    wl = SyntheticMoE(spec, seed=0, device=dev, pool_layers=pool_layers)
    gates = [g.cpu() for g in wl.gate]
    biases = [b.cpu() for b in wl.bias]
    inputs = make_inputs(spec, T, world, range(world), a.warmup + a.steps)
    times = reference_steps(spec, wl.pool, gates, biases, caps, a, inputs, a.warmup, a.steps)
    step_s = sum(times) / len(times)
    value = world * T / step_s
    return {'metric': METRIC, 'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': len(times),
            'warmup': a.warmup, 'ms_per_step': step_s * 1e3, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'impl': 'reference',
            'data': 'synthetic: random-init N(0,0.02) weights, N(0,1) hidden states rho=0.5, Zipf(1.1) router bias',
            'config': bench_config(a, spec, world, T, caps),
            'pool': {'layers': pool_layers, 'kind': 'one pool in this process'},
            'topology': 'uniform (the CPU emulation has no host links)',
            'execution': f'{world} rank(s) emulated in one host process, {threads} threads',
            'cpu_baseline': {'value': value, 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
                             'sample': f'{len(times)} timed full {spec.layers}-layer decode steps after '
                                       f'{a.warmup} warm-up steps, {world} rank(s) emulated in one '
                                       f'process ({step_s * 1e3:.0f} ms/step)'},
            'e2e': {'value': value, 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}


def run_reference_gpu(a, rank, world, local):
    """The reference's GPU runtime (oracle/ref_runtime.py: ferry/runtime.py's
    execute over the reference's compiled ops and NCCL) on this arm's
    workload: same config, inputs, weights, LUT and timing as run_ours.
    Needs the whole pool resident (its H2DEngine indexes the pool by key)."""
    from oracle.ref_runtime import RefGpuRuntime
    from ferry_b200.workload import SyntheticMoE
    dev = torch.device('cuda', local)
    if not dist.is_initialized():  # the reference's collectives need a process group
        os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
        os.environ.setdefault('MASTER_PORT', '29581')
        dist.init_process_group('nccl', rank=0, world_size=1, device_id=dev,
                                timeout=timedelta(seconds=180))
    spec = qwen3_spec(a.layers)
    T, L = a.tokens, spec.layers
    caps = spec.cache_slots(a.cache_ratio, world)
    base = {'metric': METRIC, 'impl': 'reference-gpu', 'n_gpus': world,
            'config': bench_config(a, spec, world, T, caps)}
    if a.eviction_score != 'frequency':
        return dict(base, unavailable='the composed reference runtime replays the frequency score only')
    shared = world > 1
    pool_layers = auto_pool_layers(spec, 1 if shared else world, a.pool_layers)
    if pool_layers < spec.layers:
        return dict(base, unavailable=f'host memory holds {pool_layers} of {spec.layers} layers of '
                                      'experts; the reference H2DEngine indexes the pool by key')
    wl = SyntheticMoE(spec, seed=0, device=dev, pool_layers=pool_layers, shared=shared)
    topo, topo_note = make_topology(a, spec, rank, world, wl.pool, dev)
    rt = RefGpuRuntime(spec, wl.pool, caps, a.policy, topo.masks, topo.seconds, topo.lut,
                       window=a.history_window, balance_tol_bps=a.balance_tol_bps, salt=a.salt)
    n_steps = a.warmup + a.steps
    host = make_inputs(spec, T, world, [rank], n_steps)[rank]
    inputs = [x.to(dev) for x in host]

    def step(inp):
        prev = None
        for l in range(L):
            h = inp[l] if prev is None else inp[l] + prev
            sel, w = rt.route(h, wl.gate[l], wl.bias[l])
            prev = rt.execute(l, h, sel, w)
        return prev

    for i in range(a.warmup):
        step(inputs[i])
    barrier(world)
    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(a.steps):
        step(inputs[a.warmup + i])
    ev1.record()
    ev1.synchronize()
    barrier(world)
    clocks = sampler.stop([local]) if sampler else None
    ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    host_inputs = [x.pin_memory() for x in host[a.warmup:]]
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(a.steps):
        step(host_inputs[i].to(dev, non_blocking=True)).cpu()
    e1.record()
    e1.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    fetches = int(rt.fetches_per_rank.sum())
    rt.close()
    return dict(base, value=world * T * a.steps / (ms / 1e3), unit='tokens/s', steps=a.steps,
                warmup=a.warmup, ms_per_step=ms / a.steps, higher_is_better=True, scaling='weak',
                vs_baseline=None, dtype='bf16',
                data='synthetic: random-init N(0,0.02) weights, N(0,1) hidden states rho=0.5, Zipf(1.1) router bias',
                pool={'layers': pool_layers, 'kind': 'one shared pinned pool per node' if shared else
                      'pinned pool per rank'},
                topology=topo_note, clocks=clocks,
                execution='ferry/runtime.py execute: reference compiled ops (oracle/_ref: H2DEngine, '
                          'pack/unpack, execute_experts, reduce/scatter), oracle planner/layout, NCCL '
                          'all_gather_into_tensor + all_to_all_single, torch router',
                fetches_per_layer=fetches / max(1, rt.event),
                e2e={'value': world * T * a.steps / (e2e_ms / 1e3), 'unit': 'tokens/s',
                     'h2d_bytes_per_step': int(host_inputs[0].numel() * 2),
                     'd2h_bytes_per_step': int(T * spec.hidden * 2), 'ms_per_step': e2e_ms / a.steps})


def run_gemm_compare(a, local):
    """Routed-expert GEMM of one decode layer, the same groups through both
    execute_experts implementations: this library's (gather + the fused
    tcgen05 kernel, ferryb_execute_experts) and the reference's compiled one
    (ferry/csrc/expert_ops.cpp:16-45, cuBLAS per expert).  Each call is timed
    with CUDA events around it on the current stream after a synchronisation,
    as a caller sees it; the weights (> L2) are read from HBM every call."""
    from ferry_b200 import expert_ops as ours
    from ferry_b200.workload import zipf_bias
    from oracle.build_ref import load_ref
    ref = load_ref()
    dev = torch.device('cuda', local)
    spec = qwen3_spec(1)
    H, I, E, K, T = spec.hidden, spec.intermediate, spec.experts, spec.topk, a.tokens
    g = torch.Generator(device=dev).manual_seed(5)
    cg = torch.Generator().manual_seed(5)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    gate = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    logits = (x.float() @ gate.float().t() + zipf_bias(E, 1.1, cg).to(dev)).to(torch.bfloat16)
    probs = torch.softmax(logits, -1, dtype=torch.float32)
    w, sel = torch.topk(probs, K, -1)
    w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16)
    active = torch.unique(sel).tolist()[:a.gemm_compare]
    cache = (torch.randn(len(active), spec.expert_elements, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    slots, rows, cols = [], [], []
    for i, e in enumerate(active):
        r, c = (sel == e).nonzero(as_tuple=True)
        slots.append(i); rows.append(r.contiguous()); cols.append(c.contiguous())
    routes = sum(int(r.numel()) for r in rows)

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(); fn(); e1.record(); e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    args = (cache, x, w, slots, rows, cols, H, I)
    got = ours.execute_experts(*args)
    res = {'metric': 'routed-expert GEMM of one decode layer (us per call, median)', 'experts': len(active),
           'routes': routes, 'tokens': T, 'weight_bytes': len(active) * spec.expert_bytes,
           'ours_us': round(timed(lambda: ours.execute_experts(*args), a.steps), 1)}
    if ref is None:
        res['reference'] = 'unavailable: oracle/_ref not built'
        return res
    want = ref.execute_experts(*args)
    err = max((p.float() - q.float()).abs().max().item() for p, q in zip(got, want))
    res['reference_us'] = round(timed(lambda: ref.execute_experts(*args), a.steps), 1)
    res['speedup'] = round(res['reference_us'] / res['ours_us'], 2)
    res['ours_gbs'] = round(res['weight_bytes'] / (res['ours_us'] * 1e-6) / 1e9, 1)
    res['reference_gbs'] = round(res['weight_bytes'] / (res['reference_us'] * 1e-6) / 1e9, 1)
    res['max_abs_diff'] = err
    return res


def main():
    a = parse()
    if a.impl == 'reference':
        rank = int(os.environ.get('RANK', '0'))
        world = int(os.environ.get('WORLD_SIZE', str(a.gpus)))
        if rank != 0:
            return 0
        print(json.dumps(run_reference(a, rank, world)), flush=True)
        return 0
    rank, world, local = init_dist(a.gpus)
    try:
        if a.gemm_compare:
            result = run_gemm_compare(a, local)
        elif a.full_model:
            result = run_full_model(a, rank, world, local)
        elif a.impl == 'reference-gpu':
            result = run_reference_gpu(a, rank, world, local)
        elif a.ep_sweep:
            result = run_ep_sweep(a, rank, world, local)
        else:
            result = run_ours(a, rank, world, local)
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if dist.is_initialized():
            if world > 1:
                dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == '__main__':
    sys.exit(main())
