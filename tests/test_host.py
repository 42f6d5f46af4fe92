"""Host-side pieces with no GPU: model geometry (ferry/model.py:24-70 rules),
the expert row layout, and the synthetic workload's router bias."""
import math

import numpy as np

import pytest
import torch

from ferry_b200.model import DEEPSEEK_V2_LITE, QWEN3_30B_A3B, pack_expert, spec_from_config
from ferry_b200.workload import zipf_bias


def test_qwen3_spec():
    s = spec_from_config(QWEN3_30B_A3B)
    assert s.layers == 48 and s.moe_layers == tuple(range(48))
    assert (s.experts, s.topk, s.hidden, s.intermediate) == (128, 8, 2048, 768)
    assert s.shared_intermediate == 0
    assert s.expert_bytes == 9_437_184
    # global 30 % budget split with the remainder on the lower ranks
    assert s.cache_slots(0.3, 1) == [1843]
    assert s.cache_slots(0.3, 4) == [461, 461, 461, 460]
    assert sum(s.cache_slots(0.3, 8)) == 1843


def test_deepseek_spec():
    s = spec_from_config(DEEPSEEK_V2_LITE)
    assert s.layers == 26 and s.moe_layers[0] == 1  # first_k_dense_replace = 1
    assert (s.experts, s.topk, s.intermediate) == (64, 6, 1408)
    assert s.shared_intermediate == 2 * 1408
    assert s.expert_bytes == 17_301_504
    assert s.cache_slots(0.3, 4) == [125, 125, 125, 124]  # floor(0.3 * 26 * 64) = 499


def test_spec_rejects_non_greedy_deepseek():
    c = dict(DEEPSEEK_V2_LITE, topk_method='group_limited_greedy')
    with pytest.raises(NotImplementedError):
        spec_from_config(c)


def test_qwen3_sparse_step_and_dense_layers():
    c = dict(QWEN3_30B_A3B, num_hidden_layers=8, decoder_sparse_step=2, mlp_only_layers=[3])
    assert spec_from_config(c).moe_layers == (1, 5, 7)


def test_pack_expert_layout():
    H, I = 8, 4
    g = torch.arange(I * H, dtype=torch.float32).reshape(I, H)
    u = g + 64  # small integers: exact in bf16
    d = torch.arange(H * I, dtype=torch.float32).reshape(H, I) + 128
    row = pack_expert(g, u, d)
    assert row.dtype == torch.bfloat16 and row.numel() == 3 * H * I
    assert torch.equal(row[:I * H].float(), g.reshape(-1))
    assert torch.equal(row[I * H:2 * I * H].float(), u.reshape(-1))
    assert torch.equal(row[2 * I * H:].float(), d.reshape(-1))


def test_zipf_bias_is_log_of_normalised_zipf():
    g = torch.Generator().manual_seed(0)
    b = zipf_bias(64, 1.1, g)
    p = torch.exp(b.double())
    assert math.isclose(float(p.sum()), 1.0, rel_tol=1e-6)
    ranks = torch.argsort(torch.argsort(-p)) + 1  # 1 = most popular
    want = ranks.double() ** -1.1
    assert torch.allclose(p, want / want.sum(), rtol=1e-5)


def _profile(world):
    import itertools
    doms = []
    for n in range(1, world + 1):
        for s in itertools.combinations(range(world), n):
            # pairs (0,1), (2,3) share a switch uplink of 50 GiB/s; 40 GiB/s per GPU alone
            per = {g: 40.0 for g in s}
            for pair in ((0, 1), (2, 3)):
                if all(g in s for g in pair):
                    for g in pair:
                        per[g] = 25.0
            doms.append(dict(gpus=list(s), mask=sum(1 << g for g in s), gib_per_s=sum(per.values()),
                             per_gpu_gib_per_s=[per[g] for g in s]))
    return dict(world=world, physical_gpus=list(range(world)), expert_bytes=9437184, copies=64, repeats=5,
                domains=doms)


def test_quota_lut_builder_and_topology_file(tmp_path):
    """build_quota_lut over a synthetic 4-GPU profile (two GPU pairs sharing an
    uplink), the LUT rows from the oracle's build_lut, read back through
    Topology with the reference's checks."""
    import json
    import numpy as np
    from ferry_b200.build_quota_lut import build, select_domains
    from ferry_b200.model import QWEN3_30B_A3B, spec_from_config
    from ferry_b200.quota import Topology
    from oracle import planner as op
    spec = spec_from_config(QWEN3_30B_A3B)
    prof = _profile(4)
    assert len(select_domains(prof)) == 15
    doms = select_domains(prof, '0,1:2,3')
    assert [d['mask'] for d in doms] == [1, 2, 4, 8, 3, 12]
    topo = build(prof, spec, '0,1:2,3', lut_fn=lambda *a: op.build_lut(*a))
    path = tmp_path / 'topo.json'
    path.write_text(json.dumps(topo))
    t = Topology(path, 4, spec.experts)
    assert list(t.masks) == [1, 2, 4, 8, 3, 12]
    np.testing.assert_allclose(t.seconds, [1 / 40.0] * 4 + [1 / 50.0] * 2)
    assert t.lut.shape == (129, 4) and all(int(t.lut[m].sum()) == m for m in range(129))
    # the pairs are symmetric, so quotas split evenly between them
    assert abs(int(t.lut[64][:2].sum()) - int(t.lut[64][2:].sum())) <= 1
    with pytest.raises(ValueError):
        Topology(path, 8, spec.experts)
    with pytest.raises(ValueError):
        select_domains(dict(prof, domains=prof['domains'][:4]), '0,1:2,3')


def test_decode_metrics_run_cell_semantics():
    """TTFT = first token, TPOT = (last - first) / (n - 1), decode tokens/s =
    R * B * (n - 1) / (last - first) (scripts/run_cell.py:147-158)."""
    from ferry_b200.harness import decode_metrics
    m = decode_metrics([100.0, 110.0, 120.0, 130.0], batch=64, world=1)
    assert m['ttft_ms'] == 100.0 and m['tpot_ms'] == 10.0
    assert abs(m['decode_tokens_per_s'] - 64 * 3 / 0.030) < 1e-6
    assert abs(m['total_tokens_per_s'] - 64 * 4 / 0.130) < 1e-6
    assert decode_metrics([50.0], batch=8, world=1)['decode_tokens_per_s'] is None


def test_bench_helpers():
    """The bench's workload description and pool sizing."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    import argparse
    spec = bench.qwen3_spec(48)
    a = argparse.Namespace(policy='ferry', history_window=128, balance_tol_bps=200, salt=1,
                           eviction_score='frequency')
    cfg = bench.bench_config(a, spec, 2, 64, [922, 921])
    assert cfg['global_batch'] == 128 and cfg['parallelism'] == 'dp2-ep2' and 'model' not in cfg
    assert cfg['window'] == 128 and cfg['score'] == 'frequency'
    assert bench.auto_pool_layers(spec, 8, 5) == 5
    assert 1 <= bench.auto_pool_layers(spec, 1, 0) <= 48
    # both arms draw the same hidden states
    small = bench.qwen3_spec(2)
    x1 = bench.make_inputs(small, 4, 2, [1], 2)[1]
    x2 = bench.make_inputs(small, 4, 2, [0, 1], 2)[1]
    assert all(torch.equal(p, q) for p, q in zip(x1, x2)) and x1[0].shape == (2, 4, 2048)
    # frac above 1.2 is flagged
    assert bench.self_check({'roofline': {'frac': 0.8, 'device_clock': {'frac': 1.47}}})['ok'] is False
    assert bench.self_check({'roofline': {'frac': 0.8}, 'layer_roofline': {'frac': 0.95}})['ok'] is True


def test_reference_arm_small():
    """--impl reference: full steps through the CPU path, the GPU arm's config."""
    import argparse
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    spec = bench.qwen3_spec(2)
    a = argparse.Namespace(policy='ferry', history_window=128, balance_tol_bps=200, salt=1,
                           eviction_score='frequency')
    g = torch.Generator().manual_seed(0)
    pool = (torch.randn(spec.experts, spec.expert_elements, generator=g) * 0.02).to(torch.bfloat16)
    from ferry_b200.workload import zipf_bias
    gates = [(torch.randn(spec.experts, spec.hidden, generator=g) * 0.02).to(torch.bfloat16) for _ in range(2)]
    biases = [zipf_bias(spec.experts, 1.1, g) for _ in range(2)]
    inputs = bench.make_inputs(spec, 8, 1, [0], 3)
    times = bench.reference_steps(spec, pool, gates, biases, [60], a, inputs, 1, 2)
    assert len(times) == 2 and all(t > 0 for t in times)


def test_clock_sampler_parses_reasons():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    cs = bench.ClockSampler()
    cs.proc = type('P', (), {'terminate': lambda self: None, 'wait': lambda self, timeout=None: 0})()
    cs.thread = type('T', (), {'join': lambda self, timeout=None: None})()
    cs.rows = [['0', '1965', '1965', '700', '0x0', 'Not Active', 'Not Active', 'Not Active', 'Not Active'],
               ['0', '1700', '1965', '990', '0x4', 'Not Active', 'Not Active', 'Not Active', 'Active'],
               ['1', '900', '1965', '100', '0x0', 'Active', 'Not Active', 'Not Active', 'Not Active']]
    out = cs.stop([0])
    assert out['sm_max_mhz'] == 1965.0 and out['samples'] == 2
    assert out['reasons'] == ['sw_power_cap']


def test_topology_for_run(tmp_path, monkeypatch):
    """--topology resolution shared by bench.py and the full-model harness:
    'uniform'/None and 'auto' at one rank give the even table, a path is read
    with the reference's checks, 'auto' at several ranks needs a pinned row."""
    import json
    from ferry_b200 import quota
    from ferry_b200.build_quota_lut import build, topology_for_run
    from ferry_b200.model import QWEN3_30B_A3B, spec_from_config
    from oracle import planner as op
    spec = spec_from_config(QWEN3_30B_A3B)
    monkeypatch.setattr(quota, 'build_lut', lambda *a: op.build_lut(*a))  # no GPU here
    for arg, world in ((None, 1), ('uniform', 4), ('auto', 1)):
        topo, note = topology_for_run(arg, spec, 0, world)
        assert note == 'uniform' and list(topo.masks) == [1 << r for r in range(world)]
    path = tmp_path / 'topo.json'
    path.write_text(json.dumps(build(_profile(4), spec, lut_fn=lambda *a: op.build_lut(*a))))
    topo, note = topology_for_run(str(path), spec, 0, 4)
    assert note == str(path) and len(topo.masks) == 15
    with pytest.raises(ValueError):
        topology_for_run(str(path), spec, 0, 2)
    with pytest.raises(ValueError):
        topology_for_run('auto', spec, 0, 4)


def test_bench_host_link_time_model():
    """The job's host-link term: the slowest group of ranks that shares a host
    path (profiled domains), or each rank alone plus all ranks together."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench

    class _Topo:
        masks = np.array([1, 2, 4, 8, 3, 12, 15])
        seconds = np.array([1 / 50.0] * 4 + [1 / 50.0, 1 / 100.0, 1 / 110.0])
    fb = np.array([4.0, 4.0, 1.0, 1.0]) * 2 ** 30
    t, lim = bench.host_link_time(_Topo, 'auto: profiled', fb, [50.0] * 4, 27.5, 4)
    assert lim['ranks'] == [0, 1] and abs(t - 8.0 / 50.0) < 1e-9  # ranks 0-1 share 50 GiB/s
    t, lim = bench.host_link_time(_Topo, 'uniform', fb, [60.0] * 4, 27.5, 4)
    assert lim['ranks'] == [0, 1, 2, 3] and abs(t - 10 * 2 ** 30 / 110e9) < 1e-9
    t, lim = bench.host_link_time(_Topo, 'uniform', fb[:1], [50.0], 50.0, 1)
    assert lim['ranks'] == [0] and abs(t - 4 * 2 ** 30 / 50e9) < 1e-9


def test_bench_phase_stamps_medians(monkeypatch):
    """bench.phase_stamps turns the kernels' stamp buffers into per-phase
    medians: layers whose planner had no fetch (its victim stamps unset) or
    that did not use the saved victim order are left out of those medians."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    import ferry_b200._lib as fl
    bufs = {}
    monkeypatch.setattr(fl, 'ptr', lambda t: t)
    monkeypatch.setattr(fl, 'call', lambda name, t: bufs.__setitem__(name, t))
    monkeypatch.setattr(torch.cuda, 'synchronize', lambda *a: None)

    class _Spec:
        layers = 4

    class _Wl:
        gate = bias = [None] * 4

    class _Rt:
        def forward(self, l, h, g, b):
            p = bufs['ferryb_debug_plan_timestamps']
            lay = bufs['ferryb_debug_layout_timestamps']
            r = bufs['ferryb_debug_router_timestamps']
            r[:] = torch.tensor([100, 110, 120, 121])
            p[:8] = 130 + torch.tensor([0, 4, 8, 10, 12, 22, 23, 24]) * (l + 1)
            if l == 1:
                p[4] = p[5] = 0  # no fetch: the victim stamps stay unset
            if l != 2:
                p[8:13] = torch.tensor([int(p[4]) + 3, int(p[4]) + 4, int(p[4]) + 6, int(p[4]) + 9, 80])
            lay[:7] = 500 + torch.arange(7) * 2
            return torch.zeros(1)

    out = bench.phase_stamps(_Rt(), _Wl(), _Spec(), torch.zeros(4, 1), 'cpu')
    assert out['layers'] == {'router': 4, 'planner': 3, 'victim_order_saved': 2, 'layout': 4}
    assert out['router'] == {'logits': 10.0, 'softmax_topk': 10.0, 'gather_writes': 1.0,
                             'router_end_to_planner_start': np.median([9 + 0, 9, 9, 9])}
    # planner layers 0, 2, 3 (scales 1, 3, 4): gate history 4 * scale -> median 12
    assert out['planner']['gate_history'] == 12.0 and out['planner']['victim_order'] == 30.0
    assert out['victim_order_steps'] == {'read_classify': 3.0, 'clean_dirty_split': 1.0,
                                         'dirty_sort': 2.0, 'merge': 3.0, 'dirty_records': 80.0}
    assert out['layout']['receive_pass2'] == 2.0 and len(out['layout']) == 6
    assert all(v is None for v in bufs.values())  # the hooks are switched off again
