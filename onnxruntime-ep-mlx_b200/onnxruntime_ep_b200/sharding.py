"""KV-head sharding of the paged-attention path across GPUs.

Rank r of N owns kv heads [r*KV/N, (r+1)*KV/N) and the q heads that read them,
[r*H/N, (r+1)*H/N) (q head h reads kv head h // (H/KV), so whole groups stay on one rank).
Append and attention need no cross-rank traffic; one all-gather of the per-rank outputs
[nt, H/N*d] plus a head permute rebuilds [nt, H*d]: ``PeerGather`` does both in one kernel of
peer stores over NVLink (include/b200_shard.h); ``all_gather_output`` is the NCCL form.
"""

from __future__ import annotations

import torch


def head_ranges(num_heads: int, kv_heads: int, rank: int, world: int):
    """(q head range, kv head range) of `rank`."""
    if kv_heads % world or num_heads % world:
        raise ValueError(f"{world} ranks must divide {kv_heads} kv heads and {num_heads} q heads")
    kv_per, q_per = kv_heads // world, num_heads // world
    return (rank * q_per, (rank + 1) * q_per), (rank * kv_per, (rank + 1) * kv_per)


def shard_columns(x: torch.Tensor, heads: int, head_range, head_size: int) -> torch.Tensor:
    """Columns of the heads in `head_range` from a packed [nt, heads*d] activation."""
    lo, hi = head_range
    return x[:, lo * head_size:hi * head_size].contiguous()


def reassemble(gathered: torch.Tensor) -> torch.Tensor:
    """[N, nt, H/N*d] (rank-major all-gather) -> [nt, H*d] in q-head order."""
    n, nt, w = gathered.shape
    return gathered.permute(1, 0, 2).reshape(nt, n * w)


def all_gather_output(out: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather this rank's [nt, H/N*d] output and reassemble [nt, H*d]."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    buf = torch.empty((world, *out.shape), dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(buf, out.contiguous(), group=group)
    return reassemble(buf)


class _DeviceArray:
    """A raw device allocation seen by torch through ``__cuda_array_interface__`` (no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3}


class PeerGather:
    """All-gather + head permute of the head-sharded outputs over NVLink peer memory.

    ``b200_shard_gather`` (include/b200_shard.h): every rank stores its ``[rows, H/N*d]`` slice
    into every rank's ``[rows, H*d]`` output at column offset ``rank*H/N*d``, between an entry and
    an exit barrier on flag words in peer memory; one kernel, no NCCL, capturable in a CUDA
    graph.  Set-up allocates this rank's output and flag words (whole allocations, so CUDA IPC
    can name them), exchanges the IPC handles with one all-gather on ``group`` and opens the
    peers'.  ``output`` is this rank's ``[rows, H*d]`` result (valid after a call completes on
    the stream); ``close()`` waits for every rank, then unmaps and frees (call it on every rank).
    """

    def __init__(self, rows: int, slice_cols: int, dtype, device, group=None):
        import ctypes

        import numpy as np
        import torch.distributed as dist

        from . import _capi

        self._capi, self._lib, self._group = _capi, _capi.LIB, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _capi.SHARD_MAX_RANKS:
            raise ValueError(f"at most {_capi.SHARD_MAX_RANKS} ranks")
        self.device = torch.device(device)
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        esz = torch.empty((), dtype=dtype).element_size()
        self.rows, self.slice_bytes = int(rows), int(slice_cols) * esz
        if self.slice_bytes % 16:
            raise ValueError("a row slice must be a multiple of 16 bytes")
        lib, check = self._lib, _capi.check
        out_bytes = max(self.rows * self.world * self.slice_bytes, 16)
        self._own = []

        def alloc(n):
            ptr = ctypes.c_void_p()
            check(lib.b200_ep_device_alloc(self.dev_index, n, ctypes.byref(ptr)))
            self._own.append(ptr.value)
            return ptr.value

        out_ptr, flag_ptr, word_ptr = alloc(out_bytes), alloc(256), alloc(256)
        zeros = (ctypes.c_uint8 * 256)()
        for ptr in (flag_ptr, word_ptr):  # flag, state and status words start at zero
            check(lib.b200_ep_copy(self.dev_index, ptr, ctypes.addressof(zeros), 256, None))
        hs = lib.b200_ipc_handle_size()
        mine = (ctypes.c_uint8 * (2 * hs))()
        check(lib.b200_ipc_get_handle(out_ptr, ctypes.addressof(mine)))
        check(lib.b200_ipc_get_handle(flag_ptr, ctypes.addressof(mine) + hs))
        local = torch.tensor(np.frombuffer(bytes(mine), np.uint8), device=self.device)
        every = torch.empty((self.world, 2 * hs), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, local, group=group)
        every = every.cpu().numpy()
        self._opened = []
        p = _capi.ShardGatherParams()
        p.world, p.rank, p.rows, p.slice_bytes = self.world, self.rank, self.rows, self.slice_bytes
        for t in range(self.world):
            if t == self.rank:
                p.outputs[t], p.flags[t] = out_ptr, flag_ptr
                continue
            for j, slot in ((0, "outputs"), (1, "flags")):
                h = (ctypes.c_uint8 * hs).from_buffer_copy(every[t, j * hs:(j + 1) * hs].tobytes())
                ptr = ctypes.c_void_p()
                check(lib.b200_ipc_open_handle(self.dev_index, ctypes.addressof(h), ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                getattr(p, slot)[t] = ptr.value
        p.state = word_ptr
        p.status = word_ptr + 64
        self._status_ptr = word_ptr + 64
        self.params = p
        typestr = {1: "|u1", 2: "<u2", 4: "<u4"}[esz]
        raw = torch.as_tensor(_DeviceArray(out_ptr, (self.rows, self.world * slice_cols), typestr), device=self.device)
        self.output = raw.view(dtype)
        dist.barrier(group=group)  # every rank has opened every handle before the first gather

    def __call__(self, local: torch.Tensor, stream=None) -> torch.Tensor:
        import ctypes

        if local.shape[0] != self.rows or local.element_size() * local.shape[1] != self.slice_bytes:
            raise ValueError("local output shape differs from the set-up")
        if not local.is_contiguous():
            raise ValueError("local output must be contiguous")
        self.params.local = local.data_ptr()
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        self._capi.check(self._lib.b200_shard_gather(ctypes.byref(self.params), ctypes.c_void_p(s.cuda_stream)))
        return self.output

    def read_status(self) -> int:
        """Synchronise and return the device status word (B200 status bits; 1 << 5 = a bounded
        wait ran out)."""
        import ctypes

        word = ctypes.c_int32()
        torch.cuda.synchronize(self.device)
        self._capi.check(self._lib.b200_ep_copy(self.dev_index, ctypes.addressof(word), self._status_ptr, 4, None))
        return int(word.value)

    def close(self):
        import torch.distributed as dist

        if self._lib is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._group)  # no rank still stores into this rank's output
        for ptr in self._opened:
            self._lib.b200_ipc_close_handle(self.dev_index, ptr)
        dist.barrier(group=self._group)  # no rank still maps this rank's buffers
        for ptr in self._own:
            self._lib.b200_ep_device_free(self.dev_index, ptr)
        self._opened, self._own, self._lib = [], [], None
        self.output = None
