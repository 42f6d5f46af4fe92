"""Drop-in for ferry/runtime.py: the multi-GPU offloading runtime
(DP attention + EP routed experts with per-GPU expert caches).

OffloadRuntime keeps the reference's constructor, reset/execute/close and
counters (ferry/runtime.py:34-93).  execute() runs the whole layer through
libferryb's fused executor (ferryb_layer_execute): P2P all-gather of the
routing metadata, the device planner, the device layout, copy-engine
fetches, P2P dispatch, the tcgen05 grouped SwiGLU and the P2P combine; the
host only polls mapped memory (the planner's fetch list, then the layout's
summary), with no copy or stream sync per layer.  forward() additionally moves the MoE hook's router
into kernel 1 (ferryb_layer_forward).

Ranks and world size come from torch.distributed when it is initialised
(one process per GPU); torch.distributed only exchanges the CUDA IPC handles
of the symmetric buffers at construction.  No NCCL call sits on the layer
path.
"""
import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._lib import call, check_tensor, ptr, stream_ptr
from .expert_ops import H2DEngine
from .policy import Controller
from .symm import SymmetricBuffer


def expert_ops():
    """The expert-op module that ferry/runtime.py:26-31 compiles and returns:
    here ferry_b200.expert_ops (execute_experts, pack_dispatch,
    unpack_dispatch, reduce_partials, scatter_returned, H2DEngine), whose
    kernels are in libferryb.so."""
    from . import expert_ops as ops
    return ops


def _rank_world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


class _Executor:
    """One ferryb_layer (buffers sized for `tokens` tokens per rank)."""

    def __init__(self, rt, tokens):
        spec = rt.spec
        cfg = _lib.LayerConfig()
        cfg.world, cfg.rank, cfg.tokens_per_rank = rt.world, rt.rank, tokens
        cfg.topk, cfg.experts, cfg.hidden, cfg.intermediate = spec.topk, spec.experts, spec.hidden, spec.intermediate
        cfg.router_mode = 1 if spec.model_type == 'deepseek_v2' else 0
        cfg.norm_topk = int(rt.norm_topk_prob)
        cfg.scaling = float(rt.routed_scaling_factor)
        cfg.probability_score = int(rt.eviction_score == 'probability')
        cfg.timing = int(rt.timing)
        cfg.sync_fetch = int(rt.sync_fetch)
        cfg.shared_intermediate = rt.shared_intermediate
        self.cfg = cfg
        lib = _lib.lib()
        ws_bytes = lib.ferryb_layer_workspace_bytes(ctypes.byref(cfg))
        sym_bytes = lib.ferryb_layer_symm_bytes(ctypes.byref(cfg), rt.window)
        if ws_bytes < 0 or sym_bytes < 0:
            raise _lib.FerrybError('invalid layer configuration: ' + lib.ferryb_last_error().decode())
        self.workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=rt.device)
        self.symm = SymmetricBuffer(sym_bytes, rt.rank, rt.world, rt.group)
        h = ctypes.c_void_p()
        call('ferryb_layer_create', ctypes.byref(cfg), ctypes.byref(rt.controller._struct),
             ptr(rt.cache), rt.cache.shape[0], rt.h2d.handle, ctypes.c_void_p(self.symm.local),
             self.symm.bases_c, ptr(self.workspace), ws_bytes, ctypes.byref(h))
        self.h = h
        for layer, w in enumerate(rt.shared_experts or ()):
            if w is not None:
                call('ferryb_layer_set_shared', h, layer, ptr(w))

    def stats(self):
        st = _lib.LayerStats()
        call('ferryb_layer_get_stats', self.h, ctypes.byref(st))
        return st

    def status(self, device):
        """Raise FerrybError if a layer enqueued on this executor failed on the
        device (its GEMM or transport error words; ferryb_layer_status)."""
        call('ferryb_layer_status', self.h, stream_ptr(device))

    def close(self):
        if self.h:
            _lib.lib().ferryb_layer_destroy(self.h)
            self.h = None
        self.symm.close()


class OffloadRuntime:
    def __init__(self, spec, pool, capacities, policy, topology, history_window=128,
                 balance_tol_bps=200, salt=1, eviction_score='frequency', *, n_copy_streams=1,
                 norm_topk_prob=True, routed_scaling_factor=1.0, timing=False, group=None,
                 device=None, sync_fetch=False, shared_experts=None):
        """shared_experts: per MoE layer, the DeepSeek-V2 shared-expert MLP as one
        bf16 device row (ferry_b200.model.pack_expert) or None; forward() adds
        it to the routed output, execute() leaves it to the caller as the
        reference does."""
        self.spec = spec
        self.sync_fetch = sync_fetch
        self.shared_experts = list(shared_experts) if shared_experts is not None else None
        self.shared_intermediate = 0
        if self.shared_experts:
            sizes = {w.numel() for w in self.shared_experts if w is not None}
            if len(sizes) != 1 or next(iter(sizes)) % (3 * spec.hidden):
                raise ValueError('shared experts must be equal-size [3 * hidden * I] rows')
            self.shared_intermediate = next(iter(sizes)) // (3 * spec.hidden)
            for w in self.shared_experts:
                if w is not None and (w.dtype != torch.bfloat16 or not w.is_cuda or not w.is_contiguous()):
                    raise ValueError('shared experts must be contiguous bf16 CUDA tensors')
        self.pool = pool
        self.group = group
        self.rank, self.world = _rank_world(group)
        self.device = torch.device(device if device is not None else 'cuda')
        if self.device.index is None:
            self.device = torch.device('cuda', torch.cuda.current_device())
        self.capacities = list(capacities)
        self.cap = self.capacities[self.rank]
        self.window = history_window
        self.eviction_score = eviction_score
        self.norm_topk_prob = norm_topk_prob
        self.routed_scaling_factor = routed_scaling_factor
        self.timing = timing
        self.n_copy_streams = n_copy_streams
        self.cache = torch.empty((self.cap, spec.expert_elements), dtype=torch.bfloat16, device=self.device)
        self.controller = Controller(spec, capacities, policy, topology, balance_tol_bps, salt,
                                     device=self.device, window=history_window,
                                     score=eviction_score, topk=spec.topk)
        self.h2d = None
        self._executors = {}
        self._error_reported = False
        self.reset()

    def _executor(self, tokens):
        ex = self._executors.get(tokens)
        if ex is None:
            ex = self._executors[tokens] = _Executor(self, tokens)
        return ex

    def check(self):
        """Raise FerrybError if any layer run so far failed on the device.

        execute()/forward() return once the layer is enqueued, so a device
        error of a layer's expert GEMM or dispatch/combine (a bounded wait that
        ran out, an index out of range) surfaces at the next execute()/forward()
        or here; this waits for the runtime's stream.  The failed layer's
        output rows are NaN.  The reference raises inside the op itself
        (TORCH_CHECK, ferry/csrc/expert_ops.cpp:20-34)."""
        try:
            for ex in self._executors.values():
                ex.status(self.device)
        except _lib.FerrybError:
            self._error_reported = True
            raise

    def _pending_error(self):
        """A device error not yet raised to the caller, or None."""
        if self._error_reported:
            return None
        try:
            self.check()
        except _lib.FerrybError as exc:
            return exc
        return None

    def _run(self, name, *args):
        try:
            call(name, *args)
        except _lib.FerrybError:
            self._error_reported = True
            raise

    def set_fault_hooks(self, tokens, hooks, wait_ns=0):
        """Failure injection for the failure-detection tests (host-side
        omissions of flag stores; ferryb_layer_set_fault_hooks)."""
        call('ferryb_layer_set_fault_hooks', self._executor(tokens).h, int(hooks), int(wait_ns))

    def reset(self):
        """Empty expert cache and routing history (start of every measured run,
        ferry/runtime.py:51-62).  A device error of an earlier layer that was
        not yet reported is raised after the reset, so the runtime is clean
        for the next run either way."""
        if self.h2d is not None:
            self.h2d.synchronize()
        torch.cuda.synchronize(self.device)
        pending = self._pending_error() if self.h2d is not None else None
        for ex in self._executors.values():
            ex.close()
        self._executors = {}
        self.controller.reset()
        if self.h2d is not None:
            self.h2d.close()
        self.h2d = H2DEngine(self.cache, self.pool, self.n_copy_streams)
        self.event = 0
        self.fetches_per_rank = np.zeros(self.world, np.int64)
        self.decode_fetches_per_rank = np.zeros(self.world, np.int64)
        self.serial_wait_ns = 0
        self._error_reported = False
        if pending is not None:
            raise pending

    def _check_inputs(self, tensors):
        """Shapes, dtypes and device of the tensors handed to the executor as
        bare pointers (the reference's TORCH_CHECKs, ferry/csrc/expert_ops.cpp:20-25)."""
        for name, t, shape, dtype in tensors:
            if t is None:
                continue
            check_tensor(t, name, shape, dtype)
            if t.device != self.device:
                raise _lib.FerrybError(f'{name} is on {t.device}, the runtime on {self.device}')

    def execute(self, layer, hidden, selected, weights, probs_tail):
        """ferry/runtime.py:64-89: routing given by the MoE hook."""
        tokens, k = hidden.shape[0], self.spec.topk
        score = self.eviction_score == 'probability'
        self._check_inputs([('hidden', hidden, (tokens, self.spec.hidden), torch.bfloat16),
                            ('selected', selected, (tokens, k), None),
                            ('weights', weights, (tokens, k), None),
                            ('probs_tail', probs_tail if score else None, (None, self.spec.experts), None)])
        ex = self._executor(tokens)
        out = torch.empty_like(hidden)
        h = hidden.contiguous()
        sel = selected.contiguous().long()
        w = weights.contiguous().to(torch.bfloat16)
        pt = probs_tail.float().contiguous() if (probs_tail is not None and score) else None
        before = ex.stats().host_wait_us
        self._run('ferryb_layer_execute', ex.h, self.event, int(layer), ptr(h), ptr(sel), ptr(w), ptr(pt),
             0 if pt is None else pt.shape[0], ptr(out), stream_ptr(self.device))
        self._after(ex, before)
        return out

    def forward(self, layer, hidden, gate_weight, gate_bias=None, selected_out=None, weights_out=None):
        """execute() with the MoE hook's router fused into kernel 1."""
        tokens, k, spec = hidden.shape[0], self.spec.topk, self.spec
        self._check_inputs([('hidden', hidden, (tokens, spec.hidden), torch.bfloat16),
                            ('gate_weight', gate_weight, (spec.experts, spec.hidden), torch.bfloat16),
                            ('gate_bias', gate_bias, (spec.experts,), torch.float32),
                            ('selected_out', selected_out, (tokens, k), torch.int64),
                            ('weights_out', weights_out, (tokens, k), torch.bfloat16)])
        for name, t in (('gate_weight', gate_weight), ('gate_bias', gate_bias),
                        ('selected_out', selected_out), ('weights_out', weights_out)):
            if t is not None and not t.is_contiguous():
                raise _lib.FerrybError(f'{name} must be contiguous')
        hidden = hidden.contiguous()
        ex = self._executor(tokens)
        out = torch.empty_like(hidden)
        before = ex.stats().host_wait_us
        self._run('ferryb_layer_forward', ex.h, self.event, int(layer), ptr(hidden), ptr(gate_weight),
             ptr(gate_bias), ptr(out), ptr(selected_out), ptr(weights_out), stream_ptr(self.device))
        self._after(ex, before)
        return out

    def _after(self, ex, before):
        """Counters of ferry/runtime.py:58-62, :70-72, :80-81 (fetches of every
        rank come from the replicated plan's summary)."""
        st = ex.stats()
        self.serial_wait_ns += int((st.host_wait_us - before) * 1000)
        summ = _lib.LayoutSummary()
        call('ferryb_layer_last_summary', ex.h, ctypes.byref(summ))
        counts = np.asarray(summ.fetch_counts[:self.world], np.int64)
        self.fetches_per_rank += counts
        if self.event >= self.spec.layers:
            self.decode_fetches_per_rank += counts
        self.event += 1

    def last_summary(self, tokens):
        """The plan summary of the last layer run with `tokens` tokens."""
        summ = _lib.LayoutSummary()
        call('ferryb_layer_last_summary', self._executors[tokens].h, ctypes.byref(summ))
        return summ

    def stats(self):
        """Per-executor counters (layers, fetches, routes, bytes, phase times)."""
        return {t: ex.stats() for t, ex in self._executors.items()}

    @property
    def dispatch_bytes(self):
        return sum(ex.stats().dispatch_bytes for ex in self._executors.values())

    @property
    def combine_bytes(self):
        return sum(ex.stats().combine_bytes for ex in self._executors.values())

    def close(self):
        """Release the executors; raises a device error of an earlier layer
        that was not yet reported (after releasing them)."""
        if self.h2d is not None:
            self.h2d.synchronize()
        pending = self._pending_error()
        for ex in self._executors.values():
            ex.close()
        self._executors = {}
        if pending is not None:
            raise pending
