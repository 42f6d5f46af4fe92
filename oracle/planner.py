"""ctypes binding of oracle/ferry_oracle.c (test infrastructure only).

Each wrapper takes and returns numpy arrays shaped like the reference's numba
functions (ferry/policy.py, ferry/quota.py, ferry/layout.py) so that tests can
call the oracle and the reference side by side.
"""
import ctypes
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / 'libferry_oracle.so'
_lib = None

FERRY, RANDOM = 0, 1
POLICIES = {'ferry': FERRY, 'random': RANDOM}


class OracleAssertion(AssertionError):
    """Raised where the reference raises (or, for RANDOM, would never return)."""


def build():
    subprocess.run(['make', '-s', '-C', str(_HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _check(status):
    if status == 1:
        raise OracleAssertion('missing experts exceed the total admission capacity')
    if status == 2:
        raise OracleAssertion('no slot to evict (slot >= 0 violated)')
    if status != 0:
        raise ValueError(f'oracle: bad arguments (status {status})')


def demand(selected, origins, experts, world):
    selected, origins = _i64(selected), _i64(origins)
    d = np.zeros((experts, world), np.int64)
    lib().fo_demand(_p(selected), _p(origins), ctypes.c_int64(selected.shape[0]),
                    ctypes.c_int64(selected.shape[1]), ctypes.c_int64(experts),
                    ctypes.c_int64(world), _p(d))
    return d


def admission_capacity(slots, capacities, layer, active, experts):
    slots, capacities = _i64(slots), _i64(capacities)
    active = np.ascontiguousarray(active, dtype=np.uint8)
    u = np.zeros(len(capacities), np.int64)
    lib().fo_admission_capacity(_p(slots), ctypes.c_int64(slots.shape[1]), _p(capacities),
                                ctypes.c_int64(len(capacities)), ctypes.c_int64(layer),
                                _p(active), ctypes.c_int64(experts), _p(u))
    return u


def greedy_quota(m, capacity, masks, seconds):
    capacity, masks = _i64(capacity), _i64(masks)
    seconds = np.ascontiguousarray(seconds, dtype=np.float64)
    q = np.zeros(len(capacity), np.int64)
    _check(lib().fo_greedy_quota(ctypes.c_int64(m), _p(capacity), ctypes.c_int64(len(capacity)),
                                 _p(masks), _p(seconds), ctypes.c_int64(len(masks)), _p(q)))
    return q


def build_lut(max_misses, world, masks, seconds):
    masks = _i64(masks)
    seconds = np.ascontiguousarray(seconds, dtype=np.float64)
    lut = np.zeros((max_misses + 1, world), np.int64)
    _check(lib().fo_build_lut(ctypes.c_int64(max_misses), ctypes.c_int64(world), _p(masks),
                              _p(seconds), ctypes.c_int64(len(masks)), _p(lut)))
    return lut


def load_balanced_assignment(demand_, misses, owner, layer, quota, balance_tol_bps):
    demand_, misses, owner, quota = _i64(demand_), _i64(misses), _i64(owner), _i64(quota)
    ans = np.zeros(len(misses), np.int64)
    lib().fo_load_balanced_assignment(_p(demand_), ctypes.c_int64(demand_.shape[0]),
                                      ctypes.c_int64(demand_.shape[1]), _p(misses),
                                      ctypes.c_int64(len(misses)), _p(owner),
                                      ctypes.c_int64(layer), _p(quota),
                                      ctypes.c_int64(balance_tol_bps), _p(ans))
    return ans


def choose_slot(rank, layer, active, slots, capacities, last, scores, experts):
    active = np.ascontiguousarray(active, dtype=np.uint8)
    slots, capacities, last = _i64(slots), _i64(capacities), _i64(last)
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    f = lib().fo_choose_slot
    f.restype = ctypes.c_int64
    return int(f(ctypes.c_int64(rank), ctypes.c_int64(layer), _p(active), _p(slots),
                 ctypes.c_int64(slots.shape[1]), _p(capacities), _p(last), _p(scores),
                 ctypes.c_int64(experts)))


def mt_randint_draws(seed, n, count):
    out = np.zeros(count, np.int64)
    lib().fo_mt_draws(ctypes.c_uint32(seed & 0xffffffff), ctypes.c_int64(n),
                      ctypes.c_int64(count), _p(out))
    return out


def plan_layer(event, layer, selected, origins, gate_scores, policy, slots, capacities, owner,
               last, scores, quota_lut, masks, seconds, balance_tol_bps, salt):
    """Same contract as ferry/policy.py:130 plan_layer: updates slots/owner/last/scores
    in place (they must be C-contiguous int64/float32 arrays) and returns
    (fetches[m,3], destinations, counts)."""
    for name, arr, dt in (('slots', slots, np.int64), ('owner', owner, np.int64),
                          ('last', last, np.int64), ('scores', scores, np.float32)):
        if arr.dtype != dt or not arr.flags.c_contiguous:
            raise TypeError(f'{name} must be a C-contiguous {dt.__name__} array')
    selected, origins = _i64(selected), _i64(origins)
    gate_scores = np.ascontiguousarray(gate_scores, dtype=np.float32)
    capacities, quota_lut, masks = _i64(capacities), _i64(quota_lut), _i64(masks)
    seconds = np.ascontiguousarray(seconds, dtype=np.float64)
    experts = scores.shape[1]
    world = len(capacities)
    fetches = np.zeros((experts, 3), np.int64)
    n = np.zeros(1, np.int64)
    dest = np.zeros(selected.shape, np.int64)
    counts = np.zeros(world, np.int64)
    status = lib().fo_plan_layer(
        ctypes.c_int64(event), ctypes.c_int64(layer), _p(selected), _p(origins),
        ctypes.c_int64(selected.shape[0]), ctypes.c_int64(selected.shape[1]), _p(gate_scores),
        ctypes.c_int(policy), _p(slots), ctypes.c_int64(slots.shape[1]), _p(capacities),
        ctypes.c_int64(world), _p(owner), _p(last), _p(scores), ctypes.c_int64(experts),
        _p(quota_lut), ctypes.c_int64(quota_lut.shape[0]), _p(masks), _p(seconds),
        ctypes.c_int64(len(masks)), ctypes.c_int64(balance_tol_bps), ctypes.c_int64(salt),
        _p(fetches), _p(n), _p(dest), _p(counts))
    _check(status)
    return fetches[:int(n[0])].copy(), dest, counts


def layer_slots(slots_row, capacity, layer, experts):
    slots_row = _i64(slots_row)
    out = np.zeros(experts, np.int64)
    lib().fo_layer_slots(_p(slots_row), ctypes.c_int64(capacity), ctypes.c_int64(layer),
                         ctypes.c_int64(experts), _p(out))
    return out


def build_layout(selected, destinations, n_local, rank, experts):
    """Same contract as ferry/layout.py:12 build_layout."""
    selected, destinations = _i64(selected), _i64(destinations)
    n_total, topk = selected.shape
    world = n_total // n_local
    cap = n_local * world
    send_idx = np.zeros(cap, np.int64)
    send_ids = np.zeros((cap, topk), np.int64)
    send_counts = np.zeros(world, np.int64)
    recv_counts = np.zeros(world, np.int64)
    starts = np.zeros(experts + 1, np.int64)
    rows = np.zeros(cap * topk, np.int64)
    cols = np.zeros(cap * topk, np.int64)
    ns, nr = np.zeros(1, np.int64), np.zeros(1, np.int64)
    lib().fo_build_layout(_p(selected), _p(destinations), ctypes.c_int64(n_total),
                          ctypes.c_int64(topk), ctypes.c_int64(n_local), ctypes.c_int64(rank),
                          ctypes.c_int64(experts), _p(send_idx), _p(send_ids), _p(send_counts),
                          _p(recv_counts), _p(starts), _p(rows), _p(cols), _p(ns), _p(nr))
    sent = int(ns[0])
    total = int(starts[-1])
    return (send_idx[:sent].copy(), send_ids[:sent].copy(), send_counts, recv_counts, starts,
            rows[:total].copy(), cols[:total].copy())


class Controller:
    """Oracle twin of ferry/policy.py:208-228 Controller (host numpy state)."""

    def __init__(self, layers, experts, capacities, policy, masks, seconds, lut,
                 balance_tol_bps=200, salt=1):
        self.layers, self.experts = layers, experts
        self.policy = POLICIES[policy] if isinstance(policy, str) else int(policy)
        self.capacities = np.asarray(capacities, np.int64)
        self.masks, self.seconds, self.lut = _i64(masks), np.asarray(seconds, np.float64), _i64(lut)
        self.balance_tol_bps, self.salt = int(balance_tol_bps), int(salt)
        self.reset()

    def reset(self):
        world = len(self.capacities)
        self.slots = np.full((world, int(self.capacities.max())), -1, np.int64)
        self.owner = np.full(self.layers * self.experts, -1, np.int64)
        self.last = np.zeros(self.layers * self.experts, np.int64)
        self.scores = np.zeros((self.layers, self.experts), np.float32)

    def plan(self, event, layer, selected, origins, gate_scores):
        return plan_layer(event, layer, selected, origins, gate_scores, self.policy, self.slots,
                          self.capacities, self.owner, self.last, self.scores, self.lut,
                          self.masks, self.seconds, self.balance_tol_bps, self.salt)
