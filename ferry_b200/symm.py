"""Symmetric device buffers shared by the ranks of one node (libferryb
ferryb_symm_*): every rank allocates the same number of bytes, exchanges its
CUDA IPC handle through torch.distributed (host-side plumbing only), and maps
its peers' buffers so that kernels store packets straight into them over
NVLink/NVSwitch.  With one rank there is nothing to exchange.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call


class SymmetricBuffer:
    def __init__(self, nbytes, rank=0, world=1, group=None):
        self.nbytes, self.rank, self.world = int(nbytes), rank, world
        p = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        call('ferryb_symm_alloc', self.nbytes, ctypes.byref(p), handle if world > 1 else None)
        self.local = p.value
        self._opened = []
        bases = [0] * world
        bases[rank] = self.local
        if world > 1:
            mine = bytes(handle)
            gathered = [None] * world
            dist.all_gather_object(gathered, mine, group=group)
            for r, h in enumerate(gathered):
                if r == rank:
                    continue
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                q = ctypes.c_void_p()
                call('ferryb_symm_open', buf, ctypes.byref(q))
                bases[r] = q.value
                self._opened.append(q.value)
        self.bases = bases
        self.bases_arr = (ctypes.c_uint64 * world)(*bases)
        self.bases_c = ctypes.cast(self.bases_arr, ctypes.c_void_p)

    def close(self):
        for q in self._opened:
            _lib.lib().ferryb_symm_close(ctypes.c_void_p(q))
        self._opened = []
        if self.local:
            _lib.lib().ferryb_symm_free(ctypes.c_void_p(self.local))
            self.local = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
