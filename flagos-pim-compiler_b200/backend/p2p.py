"""Exchange buffers for the one-shot all-reduce over NVLink (one process per GPU).

Every rank allocates one zero-filled buffer (``PIM_P2P_HEADER_BYTES`` of flags, then
two slots of ``size`` rows of ``capacity`` bytes), exports it as a CUDA IPC handle,
and maps every peer's buffer; ``pim_allreduce_p2p`` then writes its partial straight
into every rank's buffer and sums the ranks' rows in rank order (bit-identical to the
host-star all_reduce of comm/lowering.py:137-150).

The group is only formed when every rank sits on its own GPU and every peer mapping
opens; otherwise (``P2PGroup.create`` returns None on every rank) the combines keep
the NCCL all_gather + ordered-sum path.  All ranks must create the group at the same
point, since the handshake is a collective over the default process group.
"""

from __future__ import annotations

import ctypes

import torch

from backend import _native as nat

HEADER_BYTES = 1024  # PIM_P2P_HEADER_BYTES
DEFAULT_CAPACITY = 256 << 10  # bytes of one row: decode activations (8-32 KB) fit many times


class P2PGroup:
    def __init__(self, rank: int, size: int, device, capacity: int, buf, counter, ptrs, opened) -> None:
        self.rank, self.size, self.capacity = rank, size, capacity
        self.device = device
        self.buf, self.counter = buf, counter
        self.ptrs = ptrs  # host array of every rank's buffer as mapped here
        self._opened = opened
        self.desc = None  # device descriptor for fused projection + all-reduce kernels

    def descriptor(self, err_ptr: int) -> int:
        """Device address of the group descriptor (built once; `err_ptr` gets wait failures)."""
        if self.desc is None:
            self.tickets = torch.zeros(2, dtype=torch.int32, device=self.device)
            self.desc = torch.zeros(int(nat.lib.pim_p2p_desc_bytes()), dtype=torch.uint8, device=self.device)
            torch.cuda.synchronize(self.device)
            nat.check(nat.lib.pim_p2p_desc_init(self.desc.data_ptr(), self.rank, self.size, self.ptrs, self.capacity,
                                                self.counter.data_ptr(), self.tickets.data_ptr(), err_ptr),
                      "pim_p2p_desc_init")
        return self.desc.data_ptr()

    @staticmethod
    def create(rank: int, size: int, device, capacity: int = DEFAULT_CAPACITY) -> "P2PGroup | None":
        import torch.distributed as dist

        if size < 2 or size > 64 or not dist.is_initialized():
            return None
        buf = torch.zeros(HEADER_BYTES + 2 * size * capacity, dtype=torch.uint8, device=device)
        counter = torch.zeros(1, dtype=torch.int32, device=device)
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_int64()
        ok = nat.lib.pim_ipc_export(buf.data_ptr(), handle, ctypes.byref(off)) == 0
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        infos = [None] * size
        dist.all_gather_object(infos, (bytes(handle), off.value, uuid, ok))
        usable = all(i[3] for i in infos) and len({i[2] for i in infos}) == size  # one GPU per rank
        opened, ptrs = [], []
        if usable:
            for r, (h, o, _, _) in enumerate(infos):
                if r == rank:
                    ptrs.append(buf.data_ptr())
                    continue
                base = ctypes.c_void_p()
                if nat.lib.pim_ipc_open(h, ctypes.byref(base)) != 0:
                    usable = False
                    break
                opened.append(base.value)
                ptrs.append(base.value + o)
        votes = [None] * size
        dist.all_gather_object(votes, usable)
        if not all(votes):
            for b in opened:
                nat.lib.pim_ipc_close(b)
            return None
        torch.cuda.synchronize(device)
        dist.barrier()  # every buffer is zero and mapped everywhere before the first call
        return P2PGroup(rank, size, device, capacity, buf, counter, nat.ptr_array(ptrs), opened)

    def fits(self, nbytes: int) -> bool:
        return nbytes % 16 == 0 and 0 < nbytes <= self.capacity

    def close(self) -> None:
        for b in self._opened:
            nat.lib.pim_ipc_close(b)
        self._opened = []
