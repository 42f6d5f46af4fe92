"""Failure detection without a GPU fault: every device wait is bounded
(about 2 s on %globaltimer); when it runs out the kernel records an error
code, returns, and the host raises — the context stays usable.  Here the
waits run out because nothing ever raises the flags they wait for: a
sequence flag no rank sets, and a peer rank that never joins the layer."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def _context_still_usable():
    a = torch.randn(256, 256, device=DEV)
    assert torch.isfinite((a @ a).sum()).item()
    from ferry_b200 import expert_ops as ops
    x = torch.randn(4, 256, device=DEV).to(torch.bfloat16)
    sel = torch.tensor([[0, 1], [1, 2], [2, 3], [3, 0]], device=DEV)
    w = torch.ones(4, 2, device=DEV).to(torch.bfloat16)
    idx = torch.arange(4, device=DEV)
    payload = ops.pack_dispatch(x, sel, w, idx, sel, 4)
    assert payload.shape == (4, 2 * 256 + 6)


def test_flag_wait_times_out():
    from ferry_b200 import _lib
    p = ctypes.c_void_p()
    _lib.call('ferryb_symm_alloc', 4096, ctypes.byref(p), None)  # zeroed: no flag is ever raised
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    t0 = time.time()
    _lib.call('ferryb_symm_wait', p, 0, 4, ctypes.c_uint64(1), _lib.ptr(err), _lib.stream_ptr(DEV))
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert int(err.item()) == 1  # DEV_WAIT_TIMEOUT
    assert 1.0 < waited < 30.0
    _lib.call('ferryb_symm_free', p)
    _context_still_usable()


def test_missing_peer_rank_times_out(monkeypatch):
    """A 2-rank layer whose second rank never runs: rank 0's planner waits for
    rank 1's routing metadata, gives up, and execute() raises FERRYB_ETIMEOUT
    before any fetch, dispatch or GEMM is issued.  Rank 1's buffer is rank 0's
    own (one process, one GPU), so every store stays in this process's memory."""
    from ferry_b200 import _lib
    from ferry_b200 import runtime as rtmod
    from ferry_b200.expert_ops import H2DEngine
    from ferry_b200.model import ModelSpec
    from ferry_b200.policy import Controller
    from ferry_b200.quota import Topology
    from ferry_b200.symm import SymmetricBuffer
    from ferry_b200.workload import cpu_pool

    class _TwoRankView(SymmetricBuffer):
        def __init__(self, nbytes, rank=0, world=1, group=None):
            super().__init__(nbytes, 0, 1)
            self.world = 2
            self.bases = [self.local, self.local]
            self.bases_arr = (ctypes.c_uint64 * 2)(*self.bases)
            self.bases_c = ctypes.cast(self.bases_arr, ctypes.c_void_p)

    monkeypatch.setattr(rtmod, 'SymmetricBuffer', _TwoRankView)
    spec = ModelSpec('qwen3_moe', (0,), 16, 4, 256, 128)
    caps = [8, 8]
    topo = Topology.uniform(2, spec.experts)

    class _Rt:  # the fields _Executor reads, for rank 0 of a 2-rank job
        pass
    rt = _Rt()
    rt.spec, rt.world, rt.rank, rt.group, rt.device, rt.window = spec, 2, 0, None, DEV, 128
    rt.norm_topk_prob, rt.routed_scaling_factor, rt.eviction_score = True, 1.0, 'frequency'
    rt.timing, rt.sync_fetch, rt.shared_intermediate, rt.shared_experts = False, False, 0, None
    rt.cache = torch.empty((caps[0], spec.expert_elements), dtype=torch.bfloat16, device=DEV)
    rt.controller = Controller(spec, caps, 'ferry', topo, device=DEV, topk=spec.topk)
    rt.h2d = H2DEngine(rt.cache, cpu_pool(spec, 1, 0).pin_memory(), 1)
    ex = rtmod._Executor(rt, 8)
    x = torch.randn(8, 256, device=DEV).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(16)[:4] for _ in range(8)]).to(DEV)
    w = torch.full((8, 4), 0.25, device=DEV).to(torch.bfloat16)
    out = torch.empty_like(x)
    t0 = time.time()
    with pytest.raises(_lib.FerrybError, match='timed out'):
        _lib.call('ferryb_layer_execute', ex.h, 0, 0, _lib.ptr(x), _lib.ptr(sel), _lib.ptr(w), None, 0,
                  _lib.ptr(out), _lib.stream_ptr(DEV))
    assert time.time() - t0 > 1.0
    assert rt.h2d.copies == 0  # nothing was fetched
    ex.close()
    rt.h2d.close()
    _context_still_usable()


def _small_runtime(sync_fetch=False):
    from ferry_b200.model import ModelSpec
    from ferry_b200.quota import Topology
    from ferry_b200.runtime import OffloadRuntime
    from ferry_b200.workload import cpu_pool
    spec = ModelSpec('qwen3_moe', (0, 1), 32, 4, 256, 128)
    pool = cpu_pool(spec, spec.layers, 0).pin_memory()
    return spec, OffloadRuntime(spec, pool, [12], 'ferry', Topology.uniform(1, spec.experts),
                                sync_fetch=sync_fetch)


def _routing(spec, T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, spec.hidden, generator=g).to(torch.bfloat16)
    # routes among 8 of the experts, so that every layer fits the 12-slot cache
    sel = torch.stack([torch.randperm(8, generator=g)[:spec.topk] for _ in range(T)]) + 8 * seed
    w = torch.full((T, spec.topk), 1.0 / spec.topk).to(torch.bfloat16)
    return x.to(DEV), sel.to(DEV), w.to(DEV)


def test_fetched_expert_gemm_wait_times_out():
    """The fetched-expert GEMM waits on the device for each copy's readiness
    flag.  With the flag stores left out on the host (FERRYB_HOOK_NO_READY_FLAGS)
    and a 0.3 s limit, that wait runs out: the layer's output is NaN (never a
    sum that silently lacks the fetched experts), check() raises FerrybError
    naming the MoE layer, the next execute() raises before any fetch or GEMM
    of its own, and reset() leaves a runtime that runs the next layer
    correctly."""
    from ferry_b200 import _lib
    spec, rt = _small_runtime()
    T = 16
    x, sel, w = _routing(spec, T, 0)
    rt.set_fault_hooks(T, _lib.HOOK_NO_READY_FLAGS, wait_ns=300_000_000)
    t0 = time.time()
    out = rt.execute(0, x, sel, w, None)  # enqueued; the failure is found on the device
    with pytest.raises(_lib.FerrybError, match=r'MoE layer 0 \(event 0\).*fetched expert'):
        rt.check()
    assert time.time() - t0 > 0.25
    assert torch.isnan(out.float()).all()
    with pytest.raises(_lib.FerrybError, match='MoE layer 0'):
        rt.execute(1, x, sel, w, None)  # errors are sticky until reset
    rt.reset()  # already reported: the reset itself does not raise
    out = rt.execute(0, x, sel, w, None)
    rt.check()
    assert torch.isfinite(out.float()).all()
    rt.close()
    _context_still_usable()


def test_unreported_failure_raises_at_reset_and_close():
    """A failed layer that nobody checked is reported by reset() (after the
    runtime has been reset) and by close() (after it has been released)."""
    from ferry_b200 import _lib
    spec, rt = _small_runtime()
    T = 16
    x, sel, w = _routing(spec, T, 1)
    rt.set_fault_hooks(T, _lib.HOOK_NO_READY_FLAGS, wait_ns=200_000_000)
    rt.execute(0, x, sel, w, None)
    with pytest.raises(_lib.FerrybError, match='MoE layer 0'):
        rt.reset()
    out = rt.execute(0, x, sel, w, None)  # the reset took effect
    rt.check()
    assert torch.isfinite(out.float()).all()
    rt.set_fault_hooks(T, _lib.HOOK_NO_READY_FLAGS, wait_ns=200_000_000)
    rt.execute(1, x, sel, w, None)
    with pytest.raises(_lib.FerrybError, match='MoE layer 1'):
        rt.close()
    _context_still_usable()
