"""Drop-in for ferry/policy.py: the global placement controller on the GPU.

Controller keeps the reference's constructor and plan() signature
(ferry/policy.py:208-228); its cache state (slots, owner, last, scores) and
the GateHistory ring live in device memory and are updated by kernel 2
(ferryb_plan_layer) in one CTA, bit-exact with the reference's decisions.
plan() takes and returns numpy arrays like the reference; plan_device() is
the fused path's asynchronous variant (device ids in, device outputs, no
host synchronisation).

The step functions (_demand, _admission_capacity, load_balanced_assignment,
_choose_slot, layer_slots, plan_layer) keep their reference signatures and
run the same device code one step at a time.
"""
import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import addr, call, ptr, stream_ptr

FERRY, RANDOM = 0, 1
POLICIES = {'ferry': FERRY, 'random': RANDOM}


def _dev(device=None):
    return torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)


def _t(a, dtype, dev):
    return torch.as_tensor(np.ascontiguousarray(a), device=dev).to(dtype)


def _require(cond, msg):
    """The kernels get bare pointers: every array length they rely on is
    checked here (the reference's numba code would read out of bounds)."""
    if not cond:
        raise _lib.FerrybError(msg)


def _demand(selected, origins, experts, world):
    """ferry/policy.py:25-33."""
    dev = _dev()
    sel, org = _t(selected, torch.int64, dev), _t(origins, torch.int64, dev)
    _require(sel.dim() == 2 and org.shape == (sel.shape[0],), 'origins must have one entry per token')
    d = torch.zeros((experts, world), dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    call('ferryb_demand', ptr(sel), ptr(org), sel.shape[0], sel.shape[1], experts, world, ptr(d),
         ptr(err), stream_ptr(dev))
    _lib.check_device_error(err, '_demand')
    return d.cpu().numpy()


def _admission_capacity(slots, capacities, layer, active, experts):
    """ferry/policy.py:36-46."""
    dev = _dev()
    sl = _t(slots, torch.int32, dev)
    caps = _t(capacities, torch.int32, dev)
    act = _t(np.asarray(active, np.uint8), torch.uint8, dev)
    _require(sl.dim() == 2 and sl.shape[0] == len(capacities) and max(capacities) <= sl.shape[1],
             'slots must be [world, maxcap] with maxcap >= every capacity')
    _require(act.numel() >= experts, 'active must have one entry per expert')
    u = torch.zeros(len(capacities), dtype=torch.int64, device=dev)
    call('ferryb_admission_capacity', ptr(sl), sl.shape[1], ptr(caps), len(capacities), layer,
         ptr(act), experts, ptr(u), stream_ptr(dev))
    return u.cpu().numpy()


def load_balanced_assignment(demand, misses, owner, layer, quota, balance_tol_bps):
    """ferry/policy.py:49-106."""
    dev = _dev()
    demand = np.asarray(demand, np.int64)
    experts, world = demand.shape
    m = len(misses)
    _require(len(quota) == world and np.asarray(owner).size >= (layer + 1) * experts,
             'quota must be [world] and owner cover the layer')
    _require(m == 0 or (0 <= np.min(misses) and np.max(misses) < experts), 'miss out of range')
    ans = torch.zeros(max(m, 1), dtype=torch.int64, device=dev)
    # keep every argument tensor referenced until the kernel has run
    d_t = _t(demand, torch.int64, dev)
    m_t = _t(np.asarray(misses, np.int64).reshape(-1) if m else np.zeros(1, np.int64), torch.int64, dev)
    o_t = _t(owner, torch.int32, dev)
    q_t = _t(quota, torch.int64, dev)
    call('ferryb_load_balanced_assignment', ptr(d_t), experts, world, ptr(m_t), m, ptr(o_t), layer,
         ptr(q_t), int(balance_tol_bps), ptr(ans), stream_ptr(dev))
    return ans[:m].cpu().numpy()


def _choose_slot(rank, layer, active, slots, capacities, last, scores, experts):
    """ferry/policy.py:109-127 -> slot index or -1."""
    dev = _dev()
    slots = np.asarray(slots)
    keys = np.asarray(scores).size
    _require(slots.ndim == 2 and slots.shape[0] == len(capacities) and 0 <= rank < len(capacities)
             and capacities[rank] <= slots.shape[1], 'slots must be [world, maxcap], rank < world')
    _require(np.asarray(last).size == keys and np.asarray(active).size >= experts
             and np.max(slots[rank, :capacities[rank]], initial=-1) < keys,
             'last and scores must cover every cached key, active every expert')
    res = torch.zeros(1, dtype=torch.int64, device=dev)
    a_t = _t(np.asarray(active, np.uint8), torch.uint8, dev)
    s_t = _t(slots, torch.int32, dev)
    c_t = _t(capacities, torch.int32, dev)
    l_t = _t(last, torch.int64, dev)
    sc_t = _t(scores, torch.float32, dev)
    call('ferryb_choose_slot', rank, layer, ptr(a_t), ptr(s_t), slots.shape[1], ptr(c_t), ptr(l_t),
         ptr(sc_t), experts, ptr(res), stream_ptr(dev))
    return int(res.item())


def layer_slots(slots_row, capacity, layer, experts):
    """ferry/policy.py:197-205."""
    dev = _dev()
    row = _t(slots_row, torch.int32, dev)
    _require(row.dim() == 1 and row.numel() >= capacity, 'slots_row must hold capacity entries')
    out = torch.empty(experts, dtype=torch.int32, device=dev)
    call('ferryb_layer_slots', ptr(row), int(capacity), int(layer), int(experts), ptr(out),
         stream_ptr(dev))
    return out.cpu().numpy().astype(np.int64)


class _Spec:
    def __init__(self, layers, experts, topk):
        self.layers, self.experts, self.topk = layers, experts, topk


class Controller:
    """Replicated placement controller (ferry/policy.py:208-228) with device state."""

    def __init__(self, spec, capacities, policy, topology, balance_tol_bps=200, salt=1, *,
                 device=None, window=128, score='frequency', topk=None):
        self.spec = spec
        self.policy = POLICIES[policy] if isinstance(policy, str) else int(policy)
        self.capacities = np.asarray(capacities, np.int64)
        self.balance_tol_bps, self.salt = int(balance_tol_bps), int(salt)
        self.masks, self.seconds, self.lut = topology.masks, topology.seconds, topology.lut
        self.device = _dev(device)
        self.window = int(window)
        self.score = score
        self.topk = int(topk if topk is not None else getattr(spec, 'topk', 8))
        dev = self.device
        world = len(self.capacities)
        self.world = world
        self.maxcap = int(self.capacities.max())
        rank_of = np.concatenate([np.full(c, r, np.int32) for r, c in enumerate(self.capacities)])
        index_of = np.concatenate([r * self.maxcap + np.arange(c, dtype=np.int32)
                                   for r, c in enumerate(self.capacities)])
        self._caps = torch.as_tensor(self.capacities.astype(np.int32), device=dev)
        self._slot_rank = torch.as_tensor(rank_of, device=dev)
        self._slot_index = torch.as_tensor(index_of, device=dev)
        self._lut = torch.as_tensor(np.asarray(self.lut, np.int64), device=dev)
        self._masks = torch.as_tensor(np.asarray(self.masks, np.int64), device=dev)
        self._seconds = torch.as_tensor(np.asarray(self.seconds, np.float64), device=dev)
        E = spec.experts
        self._fetches = torch.zeros((E, 3), dtype=torch.int32, device=dev)
        self._n_fetches = torch.zeros(1, dtype=torch.int32, device=dev)
        self._counts = torch.zeros(world, dtype=torch.int32, device=dev)
        self._err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.reset()

    def reset(self):
        """Empty cache state and history.  The device arrays keep their
        addresses (an executor built on this controller stays valid)."""
        if getattr(self, '_struct', None) is not None:
            self._slots.fill_(-1)
            self._owner.fill_(-1)
            self._last.zero_()
            self._scores.zero_()
            self._ring.zero_()
            if self._ring_p is not None:
                self._ring_p.zero_()
            self._hist_count.zero_()
            self._hist_head.zero_()
            self._order_meta.zero_()  # the saved victim order is rebuilt on the next plan
            return
        dev, L, E, W, K = self.device, self.spec.layers, self.spec.experts, self.window, self.topk
        self._slots = torch.full((self.world, self.maxcap), -1, dtype=torch.int32, device=dev)
        self._owner = torch.full((L * E,), -1, dtype=torch.int32, device=dev)
        self._last = torch.zeros(L * E, dtype=torch.int64, device=dev)
        self._scores = torch.zeros((L, E), dtype=torch.float32, device=dev)
        self._ring = torch.zeros((L, W, K), dtype=torch.uint8, device=dev)
        self._ring_p = (torch.zeros((L, W, E), dtype=torch.float32, device=dev)
                        if self.score == 'probability' else None)
        self._hist_count = torch.zeros(L, dtype=torch.int32, device=dev)
        self._hist_head = torch.zeros(L, dtype=torch.int32, device=dev)
        # saved victim order: [valid, bitmask of changed layers], records of
        # order_cap slots (the planner's sort size: a power of two >= 64)
        total = int(self.capacities.sum())
        cap = 64
        while cap < total:
            cap <<= 1
        self._order_meta = torch.zeros(1 + (L + 63) // 64, dtype=torch.int64, device=dev)
        self._order_rec = torch.zeros(cap * 20, dtype=torch.uint8, device=dev)
        s = _lib.Planner()
        s.world, s.experts, s.layers, s.topk, s.window = self.world, E, L, K, W
        s.policy, s.balance_tol_bps, s.salt = self.policy, self.balance_tol_bps, self.salt
        s.maxcap, s.total_slots = self.maxcap, int(self.capacities.sum())
        s.n_domains, s.lut_rows = len(self._masks), int(self._lut.shape[0])
        for name, t in (('capacities', self._caps), ('slot_rank', self._slot_rank),
                        ('slot_index', self._slot_index), ('lut', self._lut), ('masks', self._masks),
                        ('seconds', self._seconds), ('slots', self._slots), ('owner', self._owner),
                        ('last', self._last), ('scores', self._scores), ('ring', self._ring),
                        ('ring_p', self._ring_p), ('hist_count', self._hist_count),
                        ('hist_head', self._hist_head), ('order_meta', self._order_meta),
                        ('order_rec', self._order_rec)):
            setattr(s, name, addr(t))
        s.order_cap = cap
        self._struct = s

    # host views of the device state (the reference exposes numpy arrays)
    @property
    def slots(self):
        return self._slots.cpu().numpy().astype(np.int64)

    @property
    def owner(self):
        return self._owner.cpu().numpy().astype(np.int64)

    @property
    def last(self):
        return self._last.cpu().numpy()

    @property
    def scores(self):
        return self._scores.cpu().numpy()

    def plan_device(self, event, layer, ids, dest, *, tokens_per_rank=0, origins=None,
                    gate_scores=None, prob_rows=None, stream=None):
        """Asynchronous plan on `stream`: ids [n, k] uint8 (device), dest [n, k]
        int32 (device, written).  Outputs stay in self._fetches/_n_fetches/
        _counts/_err.  gate_scores None = use the device GateHistory."""
        st = stream if stream is not None else stream_ptr(self.device)
        call('ferryb_plan_layer', ctypes.byref(self._struct), int(event), int(layer), ptr(ids),
             ids.shape[0], int(tokens_per_rank), ptr(origins), ptr(gate_scores), ptr(prob_rows),
             0 if prob_rows is None else prob_rows.shape[0], ptr(self._fetches),
             ptr(self._n_fetches), ptr(dest), ptr(self._counts), ptr(self._err), st)

    def plan(self, event, layer, selected, origins, gate_scores):
        """ferry/policy.py:225-228 -> (fetches [m, 3], destinations, counts), numpy int64."""
        dev = self.device
        sel = np.asarray(selected)
        _require(sel.ndim == 2 and sel.shape[1] == self.topk and np.asarray(origins).shape == (sel.shape[0],)
                 and np.asarray(gate_scores).size == self.spec.experts,
                 'selected must be [n, topk], origins [n], gate_scores [experts]')
        ids = torch.as_tensor(sel.astype(np.uint8), device=dev)
        org = torch.as_tensor(np.asarray(origins, np.int64), device=dev)
        gs = torch.as_tensor(np.asarray(gate_scores, np.float32), device=dev)
        dest = torch.empty(ids.shape, dtype=torch.int32, device=dev)
        self._err.zero_()
        self.plan_device(event, layer, ids, dest, origins=org, gate_scores=gs)
        _lib.check_device_error(self._err, 'plan')
        n = int(self._n_fetches.item())
        return (self._fetches[:n].cpu().numpy().astype(np.int64),
                dest.cpu().numpy().astype(np.int64), self._counts.cpu().numpy().astype(np.int64))


def plan_layer(event, layer, selected, origins, gate_scores, policy, slots, capacities, owner,
               last, scores, quota_lut, masks, seconds, balance_tol_bps, salt):
    """ferry/policy.py:130-194 on host arrays: uploads the state, plans on the
    device, writes the state back in place, returns (fetches, destinations, counts)."""
    from .quota import Topology
    layers, experts = scores.shape
    spec = _Spec(layers, experts, np.asarray(selected).shape[1])
    ctl = Controller(spec, capacities, policy, Topology.from_arrays(masks, seconds, quota_lut),
                     balance_tol_bps, salt)
    dev = ctl.device
    ctl._slots.copy_(torch.as_tensor(np.asarray(slots), device=dev).to(torch.int32))
    ctl._owner.copy_(torch.as_tensor(np.asarray(owner), device=dev).to(torch.int32))
    ctl._last.copy_(torch.as_tensor(np.asarray(last), device=dev))
    ctl._scores.copy_(torch.as_tensor(np.asarray(scores), device=dev))
    result = ctl.plan(event, layer, selected, origins, gate_scores)
    slots[...] = ctl.slots
    owner[...] = ctl.owner
    last[...] = ctl.last
    scores[...] = ctl.scores
    return result
