"""Data-parallel gradient averaging for `xdna` models (one process per GPU).

The reference is single-device (docs/compatibility.md:44); data parallelism
over the batch is new here.  ``GradAllReduce`` gives each rank a replica and
averages the gradients after every backward:

* parameters are grouped into flat buckets (``bucket_cap_mb``, 16 MB: several
  buckets per model, so all but the last all-reduce overlap backward) in
  reverse registration order, which is roughly the order backward produces
  them;
* a post-accumulate-grad hook copies a ready gradient into its bucket -- that
  copy is the gradient's first read, so a deferred conv weight gradient is
  computed (enqueued) right there -- and when a bucket is complete its
  all-reduce starts asynchronously, overlapping the rest of backward;
* ``synchronize()`` (called by the optimizer pre-hook, or by hand) waits for
  the buckets and writes the averages back into ``p.grad``.

Every backward must be followed by ``synchronize()`` before the next backward
starts.  To accumulate gradients over several micro-batches, run all but the
last backward inside ``with ar.no_sync():`` (the hooks then leave the buckets
alone and the gradients accumulate in ``p.grad``); the last backward fills the
buckets from the accumulated ``p.grad``.  A hook that fires for a bucket whose
all-reduce is still in flight raises instead of overwriting the buffer NCCL is
reading.

Collectives run through ``torch.distributed``: NCCL on NVLink/NVSwitch for xdna
tensors (handed over as zero-copy CUDA aliases, so NCCL reads and writes the
xdna memory in place), gloo for CPU tensors (the CPU tests).
"""
from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist


def _comm_view(t: torch.Tensor) -> torch.Tensor:
    if t.device.type == "xdna":
        from . import device
        return device.as_cuda(t)
    return t


class GradAllReduce:
    def __init__(self, module: torch.nn.Module, process_group=None, bucket_cap_mb: float = 16.0,
                 overlap: bool = True):
        self.module = module
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        # NCCL averages in the collective; gloo (the CPU tests) sums, then we divide
        self._avg = dist.get_backend(process_group) == "nccl"
        params = [p for p in module.parameters() if p.requires_grad]
        self.params = params
        cap = int(bucket_cap_mb * 1024 * 1024)
        buckets, cur, cur_bytes = [], [], 0
        for p in reversed(params):
            nb = p.numel() * p.element_size()
            if cur and (cur_bytes + nb > cap or p.dtype != cur[0].dtype or p.device != cur[0].device):
                buckets.append(cur)
                cur, cur_bytes = [], 0
            cur.append(p)
            cur_bytes += nb
        if cur:
            buckets.append(cur)
        self.buckets = []
        self._slot = {}
        for bi, ps in enumerate(buckets):
            total = sum(p.numel() for p in ps)
            flat = torch.zeros(total, dtype=ps[0].dtype, device=ps[0].device)
            off = 0
            for p in ps:
                self._slot[p] = (bi, off)
                off += p.numel()
            self.buckets.append({"params": ps, "flat": flat, "ready": 0, "work": None})
        self._hooks = []
        self.overlap = overlap
        self._hooks_on = True
        if overlap:
            for p in params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))

    # -- overlap path --------------------------------------------------------
    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside this context only accumulate into ``p.grad``;
        the next backward outside it launches the all-reduces."""
        prev = self._hooks_on
        self._hooks_on = False
        try:
            yield
        finally:
            self._hooks_on = prev

    def _on_grad(self, p: torch.Tensor) -> None:
        if not self._hooks_on:
            return
        bi, off = self._slot[p]
        b = self.buckets[bi]
        if b["work"] is not None:
            raise RuntimeError(
                "GradAllReduce: a gradient arrived for a bucket whose all-reduce is still in flight; call "
                "synchronize() after every backward, or run the earlier backward passes of an accumulation "
                "inside no_sync()")
        b["flat"][off:off + p.numel()].copy_(p.grad.reshape(-1))
        b["ready"] += 1
        if b["ready"] == len(b["params"]):
            b["work"] = self._all_reduce(b["flat"])

    def _all_reduce(self, flat: torch.Tensor):
        op = dist.ReduceOp.AVG if self._avg else dist.ReduceOp.SUM
        return dist.all_reduce(_comm_view(flat), op=op, group=self.pg, async_op=True)

    def synchronize(self) -> None:
        """Finish all bucket all-reduces and write averaged gradients back."""
        for b in self.buckets:
            if b["work"] is None:
                # not launched by hooks (overlap off, or a param got no grad): do it now
                off = 0
                for p in b["params"]:
                    n = p.numel()
                    if p.grad is not None:
                        b["flat"][off:off + n].copy_(p.grad.reshape(-1))
                    else:
                        b["flat"][off:off + n].zero_()
                    off += n
                b["work"] = self._all_reduce(b["flat"])
        for b in self.buckets:
            b["work"].wait()
            if not self._avg:
                b["flat"].div_(self.world)
            off = 0
            for p in b["params"]:
                n = p.numel()
                src = b["flat"][off:off + n].view_as(p)
                if p.grad is None:
                    p.grad = src.clone()
                else:
                    p.grad.copy_(src)
                off += n
            b["work"] = None
            b["ready"] = 0

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
