"""One pinned expert pool shared by every rank of a node.

The reference pins a full copy of the routed-expert pool in every rank
(ferry/model.py:89-90: 54 GiB per rank for Qwen3-30B-A3B).  Here the first
rank creates an anonymous shared-memory file (memfd), fills it once, and every
rank maps the same pages and page-locks its mapping with cudaHostRegister, so
the node holds the pool once and each GPU's copy engine still reads it as
pinned host memory.  The other ranks open the file through
/proc/<pid>/fd/<fd> of the first rank (same node, same user), with the pid and
descriptor passed over torch.distributed (host-side plumbing only).
"""
import mmap
import os

import torch
import torch.distributed as dist

_REGISTER_PORTABLE = 1  # cudaHostRegisterPortable


class SharedPinnedPool:
    """rows x row_elements tensor in shared, page-locked host memory.

    fill(tensor) runs once, on the group's first rank, before the others map
    the pool.  Keep the object alive while the pool is used."""

    def __init__(self, rows, row_elements, dtype=torch.bfloat16, fill=None, group=None):
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        itemsize = torch.empty((), dtype=dtype).element_size()
        self.nbytes = int(rows) * int(row_elements) * itemsize
        if rank == 0:
            self._fd = os.memfd_create('ferry_b200_pool', 0)
            os.ftruncate(self._fd, self.nbytes)
            info = [os.getpid(), self._fd]
        else:
            info = [None, None]
        dist.broadcast_object_list(info, src=dist.get_global_rank(group, 0) if group else 0, group=group)
        if rank != 0:
            self._fd = os.open(f'/proc/{info[0]}/fd/{info[1]}', os.O_RDWR)
        self._mm = mmap.mmap(self._fd, self.nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        self.tensor = torch.frombuffer(self._mm, dtype=dtype).view(int(rows), int(row_elements))
        self._registered = False
        if rank == 0:
            self._register()
            if fill is not None:
                fill(self.tensor)
        dist.barrier(group=group)
        if rank != 0:
            self._register()
        dist.barrier(group=group)

    def _register(self):
        err = torch.cuda.cudart().cudaHostRegister(self.tensor.data_ptr(), self.nbytes, _REGISTER_PORTABLE)
        if int(err) != 0:
            raise RuntimeError(f'cudaHostRegister of the shared expert pool failed ({int(err)})')
        self._registered = True

    def close(self):
        if self._registered:
            torch.cuda.cudart().cudaHostUnregister(self.tensor.data_ptr())
            self._registered = False
        self.tensor = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:
                pass  # a view is still alive; the mapping goes with the process
            self._mm = None
        if self._fd is not None:
            os.close(self._fd)
            self._fd = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
