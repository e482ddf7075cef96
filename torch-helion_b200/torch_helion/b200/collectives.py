"""Tensor-parallel all-reduce through NVSwitch multicast (``th_allreduce``).

The tensor-parallel Llama block sums the row-split projections' partial
outputs (o_proj, down_proj) over the ranks.  Instead of handing those
buffers to NCCL, the runtime allocates them in symmetric memory (torch's
``_symmetric_memory``: the same allocation mapped on every rank of the
group, plus one NVLS multicast address for all copies) and reduces them in
place with ``th_allreduce``, one kernel per call and rank, whose grid size
the caller chooses (the SMs the GEMMs beside it leave free).

``multimem_available`` decides once per group whether every rank can do it
(CUDA multicast objects need NVSwitch and driver support); the runtime falls
back to NCCL when not, with every rank taking the same choice.
"""

from __future__ import annotations

import torch

from . import lib


def multimem_available(device: torch.device, group=None) -> bool:
    """True when every rank of ``group`` supports multicast symmetric memory (a collective call)."""
    import torch.distributed as dist
    from torch.distributed import _symmetric_memory as symm

    try:
        ok = bool(symm._SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, device.index))
    except Exception:  # an older torch, or no CUDA multicast API
        ok = False
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


class SymmetricRows:
    """A [rows, cols] tensor in symmetric memory with the multicast address and signal pad that
    ``th_allreduce`` needs, and an fp32 [rows] array for per-row sums of squares that the
    all-reduce fills when ``stats`` is set (the next RMSNorm's statistic).  Creating one is a
    collective call (every rank, same shape)."""

    def __init__(self, rows: int, cols: int, dtype: torch.dtype, device: torch.device, group=None, ctas: int = 0):
        import torch.distributed as dist
        from torch.distributed import _symmetric_memory as symm

        group = group if group is not None else dist.group.WORLD
        esz = torch.empty((), dtype=dtype).element_size()
        data = (rows * cols * esz + 255) // 256 * 256
        sq = (rows * 4 + 255) // 256 * 256
        raw = symm.empty(data + sq + lib.ALLREDUCE_SIGNAL_BYTES, dtype=torch.uint8, device=device)
        hdl = symm.rendezvous(raw, group)
        if not hdl.multicast_ptr:
            raise lib.B200KernelError("symmetric memory has no multicast address on this device")
        # the tensor may sit at an offset inside the symmetric allocation: every mapping shares it
        off = raw.data_ptr() - hdl.buffer_ptrs[hdl.rank]
        self.rank, self.world = hdl.rank, hdl.world_size
        self.mc = hdl.multicast_ptr + off
        self.dtype, self.row_bytes, self.ctas = dtype, cols * esz, ctas
        self.sig = raw[data + sq:]
        self.peer_sig = torch.tensor([p + off + data + sq for p in hdl.buffer_ptrs], dtype=torch.int64,
                                     device=device)
        self.buf = raw[: rows * cols * esz].view(dtype).view(rows, cols)
        self.sumsq = raw[data: data + rows * 4].view(torch.float32)
        self.sumsq_mc = self.mc + data
        self.stats = False
        self._raw, self._hdl = raw, hdl  # keep the mapping alive
        self.sig.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every pad is zero before any rank's first signal

    def allreduce_rows(self, r0: int, r1: int) -> None:
        """Sum rows [r0, r1) over the ranks, in place, on the current stream."""
        if not 0 <= r0 <= r1 <= self.buf.shape[0]:
            raise lib.B200KernelError(f"allreduce_rows: rows [{r0}, {r1}) outside [0, {self.buf.shape[0]})")
        lib.allreduce(self.mc, self.peer_sig, self.sig, r0 * self.row_bytes, (r1 - r0) * self.row_bytes, self.dtype,
                      self.rank, self.world, self.ctas, sumsq_mc=self.sumsq_mc if self.stats else 0,
                      row_bytes=self.row_bytes)
