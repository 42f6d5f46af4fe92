"""Drop-in for ferry/quota.py: topology-aware quota (Step 2) on the GPU.

greedy_quota / build_lut keep the reference's signatures (numpy in, numpy
out) and run the planner's greedy on the device (kernel 2's warp greedy,
float64 without FMA contraction, ties as ferry/quota.py:52-61).  Topology
loads the same JSON files (ferry/quota.py:77-100).
"""
import json
from pathlib import Path

import numpy as np
import torch

from . import _lib
from ._lib import call, ptr, stream_ptr


def _device():
    return torch.device('cuda', torch.cuda.current_device())


def _rows(m_begin, m_end, capacity, masks, seconds):
    dev = _device()
    masks_t = torch.as_tensor(np.asarray(masks, np.int64), device=dev)
    sec_t = torch.as_tensor(np.asarray(seconds, np.float64), device=dev)
    world = None
    if capacity is not None:
        cap = np.asarray(capacity, np.int64)
        world = len(cap)
        cap_t = torch.as_tensor(np.minimum(cap, 1 << 30).astype(np.int32), device=dev)
    else:
        cap_t = None
    return dev, masks_t, sec_t, cap_t, world


def greedy_quota(m, capacity, masks, seconds):
    """ferry/quota.py:25-67 -> quota [world] int64; AssertionError when the
    missing experts exceed the total admission capacity."""
    dev, masks_t, sec_t, cap_t, world = _rows(m, m + 1, capacity, masks, seconds)
    out = torch.zeros((1, world), dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    call('ferryb_greedy_quota_rows', world, ptr(masks_t), ptr(sec_t), len(masks_t), ptr(cap_t),
         int(m), int(m) + 1, ptr(out), ptr(err), stream_ptr(dev))
    _lib.check_device_error(err, 'greedy_quota')
    return out[0].cpu().numpy()


def build_lut(max_misses, world, masks, seconds):
    """ferry/quota.py:70-74 -> [max_misses + 1, world] int64 quota table."""
    dev = _device()
    masks_t = torch.as_tensor(np.asarray(masks, np.int64), device=dev)
    sec_t = torch.as_tensor(np.asarray(seconds, np.float64), device=dev)
    out = torch.zeros((max_misses + 1, world), dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    call('ferryb_greedy_quota_rows', world, ptr(masks_t), ptr(sec_t), len(masks_t), None, 0,
         max_misses + 1, ptr(out), ptr(err), stream_ptr(dev))
    _lib.check_device_error(err, 'build_lut')
    return out.cpu().numpy()


class Topology:
    """Profiled bandwidth domains plus the precomputed quota lookup table
    (ferry/quota.py:77-100).  The constructor and `uniform` keep the
    reference's reading of the file line for line, error messages included:
    a topology file, and the errors it raises, must be the same under either
    implementation.  The greedy that fills the table runs on the GPU
    (build_lut above)."""

    def __init__(self, path, world, experts):
        data = json.loads(Path(path).read_text())
        if data['world'] != world:
            raise ValueError(f"topology file is for {data['world']} GPUs, runtime has {world}")
        self.masks = np.asarray([d['mask'] for d in data['domains']], np.int64)
        self.seconds = np.asarray([1.0 / d['gib_per_s'] for d in data['domains']], np.float64)
        self.lut = np.asarray(data['quota_lut'], np.int64)
        if self.lut.shape[0] < experts + 1 or self.lut.shape[1] != world:
            raise ValueError('quota lookup table does not cover this model; rebuild it')
        assert all(int(self.lut[m].sum()) == m for m in range(len(self.lut)))
        self.gpus = data.get('physical_gpus')

    @classmethod
    def uniform(cls, world, experts):
        """Equal singleton bandwidths, no shared domain: Step 2 is an even split."""
        self = cls.__new__(cls)
        self.masks = np.asarray([1 << r for r in range(world)], np.int64)
        self.seconds = np.ones(world, np.float64)
        self.lut = build_lut(experts, world, self.masks, self.seconds)
        self.gpus = None
        return self

    @classmethod
    def from_arrays(cls, masks, seconds, lut, gpus=None):
        self = cls.__new__(cls)
        self.masks = np.asarray(masks, np.int64)
        self.seconds = np.asarray(seconds, np.float64)
        self.lut = np.asarray(lut, np.int64)
        self.gpus = gpus
        return self
