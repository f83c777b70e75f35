"""Data parallelism over micro-batches: the one exchange step of the LoRA step.

Every rank holds the same frozen IQR base and the same adapter and runs its own micro-batches; the only
collective is the all-reduce (mean) of the flat f32 adapter gradient before AdamW. It is issued in
per-layer buckets -- the adapter's flat buffer is layer-contiguous -- as the reverse walk finishes each
layer, on a side stream, so it overlaps the rest of the backward; ``join`` makes the update wait for it.
The reference has no multi-GPU implementation (its trainer runs one card); the gradient it would
exchange is its grad stage's flat buffer (src/adjoint/device/grad_stage.h), which this buffer mirrors.

Collective order: every rank must issue the same buckets in the same order, which the walk guarantees
by reporting every layer, in reverse order, whatever its micro-batch held. ``join`` then issues, in index
order, any bucket the walk did not report (the same ones on every rank), so the update never reads a
bucket that was not exchanged.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GradBuckets:
    """Per-layer all-reduce (mean over ranks) of ``grad[lo:hi]`` for each ``(lo, hi)`` in ``ranges``.

    With ``overlap=False`` the walk's reports are only recorded and ``join`` exchanges the whole buffer in
    one all-reduce on the compute stream: no collective kernel then shares the SMs with the backward's
    persistent kernels (which size their grids to every SM), at the cost of the exchange's time."""

    def __init__(self, grad: torch.Tensor, ranges, group=None, overlap: bool = True):
        self.grad = grad
        self.ranges = [(int(lo), int(hi)) for lo, hi in ranges]
        self.group = group
        self.overlap = overlap
        self.world = dist.get_world_size(group)
        self.avg = dist.get_backend(group) == "nccl"  # NCCL averages in the collective; gloo sums
        self.stream = torch.cuda.Stream(device=grad.device) if grad.is_cuda else None
        self._works = []
        self._issued = []

    def ready(self, li: int) -> None:
        """Bucket ``li`` is final on this rank: start its all-reduce. Inside a CUDA graph capture the
        collective is captured too: the side stream joins the capture through the event edge from the
        compute stream, and the all-reduce is issued as a stream-ordered (not host-waited) operation there."""
        if li in self._issued:
            raise RuntimeError(f"gradient bucket {li} issued twice in one step")
        if not self.overlap:
            self._issued.append(li)
            return
        lo, hi = self.ranges[li]
        view = self.grad[lo:hi]
        op = dist.ReduceOp.AVG if self.avg else dist.ReduceOp.SUM
        if self.stream is not None:
            ev = torch.cuda.Event()
            ev.record()  # the layer's gradient kernels, on the compute stream
            self.stream.wait_event(ev)
            with torch.cuda.stream(self.stream):
                if torch.cuda.is_current_stream_capturing():
                    dist.all_reduce(view, op=op, group=self.group)  # ordered on the side stream
                    work = None
                else:
                    work = dist.all_reduce(view, op=op, group=self.group, async_op=True)
        else:
            work = dist.all_reduce(view, op=op, group=self.group, async_op=True)
        self._works.append((work, view))
        self._issued.append(li)

    def join(self):
        """Issues the buckets the walk did not, waits for every one, and returns the order they were
        issued in. On return the gradient is the mean over ranks (on the device: once the current stream
        reaches this point)."""
        for li in range(len(self.ranges)):
            if li not in self._issued:
                self.ready(li)
        if not self.overlap:
            op = dist.ReduceOp.AVG if self.avg else dist.ReduceOp.SUM
            if self.grad.is_cuda and torch.cuda.is_current_stream_capturing():
                dist.all_reduce(self.grad, op=op, group=self.group)
            else:
                dist.all_reduce(self.grad, op=op, group=self.group, async_op=True).wait()
            if not self.avg and self.world > 1:
                self.grad.div_(self.world)
            order = list(self._issued)
            self._issued.clear()
            return order
        for work, view in self._works:
            if work is not None:
                work.wait()
            if not self.avg and self.world > 1:
                if self.stream is not None:
                    with torch.cuda.stream(self.stream):
                        view.div_(self.world)
                else:
                    view.div_(self.world)
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)
        order = list(self._issued)
        self._works.clear()
        self._issued.clear()
        return order
