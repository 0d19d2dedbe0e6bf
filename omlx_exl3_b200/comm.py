"""NVLink peer buffers of a tensor-parallel group and the fused all-reduce that uses them.

One process per GPU. Each rank allocates one buffer (exl3_peer_create), the 64-byte CUDA IPC handles
are exchanged with one all_gather over the group's process group, and every rank maps the others'
buffers (exl3_peer_open). A row-parallel projection's GEMV pushes its partial output straight into
every rank's inbox (kernels.TrellisGemvPlan.peer, or `put` for any other producer), as 8-byte words
that carry the call's epoch next to the data; exl3_ar_add_norm_rot then waits on its own inboxes
only, sums the ranks and does the residual add, RMSNorm and input rotations of the next projection
group in the same kernel. This replaces the NCCL all-reduce + add_norm_rot pair of the decode step
(model.Qwen3EXL3); the reference has no tensor parallelism (one Apple GPU).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import PEER_HANDLE_BYTES, PeerGroupDesc, check, dtype_code, lib, stream_ptr

FLAG_OFF = 0
DATA_OFF = 256


class _DevArray:
    """A raw device pointer exposed through __cuda_array_interface__ (viewed, not copied, by torch)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGroup:
    def __init__(self, world: int, rank: int, device: torch.device, max_rows: int, max_k: int, group=None,
                 handles: list[bytes] | None = None, capacity_world: int | None = None):
        """Collective over `group` unless `handles` (every rank's IPC handle, in rank order) is given.
        The buffer holds inboxes for `capacity_world` ranks (default `world`; tests that wire several
        single-rank groups into one emulated group on one GPU size it for the emulated group)."""
        assert 1 <= world <= 8
        self.world, self.rank, self.device = world, rank, device
        self.max_rows, self.max_k = max_rows, max_k
        self.inbox_bytes = ((max_rows * max_k * 4 + 255) // 256) * 256
        self.nbytes = DATA_OFF + 2 * max(world, capacity_world or world) * self.inbox_bytes
        L = lib()
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            handle = (ctypes.c_uint8 * PEER_HANDLE_BYTES)()
            check(L.exl3_peer_create(self.nbytes, ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p)),
                  "exl3_peer_create")
            self.own = ptr.value
            if handles is None and world == 1:
                handles = [bytes(handle)]
            if handles is None:
                mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
                parts = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(parts, mine, group=group)
                handles = [bytes(p.cpu().tolist()) for p in parts]
            self.opened = []
            desc = PeerGroupDesc()
            desc.world, desc.rank = world, rank
            for p in range(world):
                if p == rank:
                    desc.base[p] = self.own
                    continue
                h = (ctypes.c_uint8 * PEER_HANDLE_BYTES).from_buffer_copy(handles[p])
                pp = ctypes.c_void_p()
                check(L.exl3_peer_open(ctypes.cast(h, ctypes.c_void_p), ctypes.byref(pp)), "exl3_peer_open")
                desc.base[p] = pp.value
                self.opened.append(pp.value)
            desc.flag_off, desc.data_off, desc.inbox_bytes = FLAG_OFF, DATA_OFF, self.inbox_bytes
            self.desc = desc
            self._raw = torch.as_tensor(_DevArray(self.own, self.nbytes), device=device)   # int16 view
        self.handle = bytes(handle)

    def flags(self) -> torch.Tensor:
        """The own flag block as int32 words (tests)."""
        return self._raw[: 32].view(torch.int32)

    def put(self, slot: int, src: torch.Tensor):
        """Push this rank's (rows, k) 16-bit partial into inbox (slot, rank) of every rank (exl3_peer_put)."""
        rows, k = src.shape
        assert src.element_size() == 2 and src.is_contiguous()
        check(lib().exl3_peer_put(ctypes.byref(self.desc), slot, src.data_ptr(), rows, k, stream_ptr(src.device)),
              "exl3_peer_put")

    def ar_add_norm_rot(self, slot: int, x: torch.Tensor, w: torch.Tensor, eps: float, suh: torch.Tensor,
                        want_xn: bool = True) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
        """(h, xn, xh): h = x + sum over ranks of this call's partials in slot `slot`, xn = RMSNorm(h) * w
        (None unless want_xn), xh its rotations."""
        rows, k = x.shape
        suh = suh.reshape(-1, k)
        nm = suh.shape[0]
        x = x.contiguous()
        w = w.to(x.dtype).contiguous()
        suh = suh.to(torch.float16).contiguous()
        h = torch.empty_like(x)
        xn = torch.empty_like(x) if want_xn else None
        xh = torch.empty((nm, rows, k), dtype=torch.float16, device=x.device)
        check(lib().exl3_ar_add_norm_rot(ctypes.byref(self.desc), slot, x.data_ptr(), w.data_ptr(),
                                         dtype_code(x.dtype), rows, k, float(eps), suh.data_ptr(), nm, h.data_ptr(),
                                         xn.data_ptr() if xn is not None else None, xh.data_ptr(),
                                         stream_ptr(x.device)), "exl3_ar_add_norm_rot")
        return h, xn, xh

    def status(self) -> int:
        st = ctypes.c_uint32()
        check(lib().exl3_peer_status(ctypes.byref(self.desc), ctypes.byref(st)), "exl3_peer_status")
        return st.value

    def close(self):
        """Unmap the peers' buffers and free the own one (after all ranks are done with it)."""
        L = lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self.opened:
                L.exl3_peer_close(p)
            self.opened = []
            self._raw = None
            if self.own:
                L.exl3_peer_destroy(self.own)
                self.own = None
