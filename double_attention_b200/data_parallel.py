"""Data-parallel gradient averaging for the training step (one process per GPU).

The reference trains with plain data parallelism: every rank runs the whole
model on its own batch slice and gradients are averaged before the
optimiser step (benchmark_lm_training.py:254-293 drives it; the module code
is rank-agnostic).  The only collective on the path is that average.  Here it
is a bucketed all-reduce over the process group (NCCL on GPUs, gloo in the
CPU tests):

* buckets are formed in reverse registration order, the order in which
  backward produces most gradients, so early buckets can be reduced while the
  rest of backward still runs;
* parameters listed as ``last`` (the shared dictionary banks, whose gradient
  is final only after every block that reads the bank has run its backward)
  form the final bucket;
* a bucket is launched (asynchronously) from the gradient-accumulation hook of
  its last parameter; :meth:`finish` waits for every bucket and writes the
  averaged values back into ``param.grad``.
"""

from __future__ import annotations

import datetime
from collections.abc import Iterable

import torch
import torch.distributed as dist
from torch import Tensor, nn


class GradientAllReduce:
    def __init__(self, params: Iterable[nn.Parameter], *, last: Iterable[nn.Parameter] = (),
                 bucket_bytes: int = 8 << 20, group=None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        late_ids = {id(p) for p in last}
        params = [p for p in params if p.requires_grad]
        seen: set[int] = set()
        unique = []
        for p in params:  # tied weights appear once
            if id(p) not in seen:
                seen.add(id(p))
                unique.append(p)
        early = [p for p in reversed(unique) if id(p) not in late_ids]
        late = [p for p in unique if id(p) in late_ids]
        self.buckets: list[list[nn.Parameter]] = []
        cur: list[nn.Parameter] = []
        size = 0
        for p in early:
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        if late:
            self.buckets.append(late)
        self._bucket_of = {id(p): i for i, b in enumerate(self.buckets) for p in b}
        self._pending: list[int] = []
        self._handles: list = []
        self._flat: list[Tensor | None] = []
        self._hooks = []
        self.reset()
        if self.world > 1:
            for p in unique:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))

    def reset(self) -> None:
        """Arm for the next backward pass."""
        self._pending = [len(b) for b in self.buckets]
        self._handles = [None] * len(self.buckets)
        self._flat = [None] * len(self.buckets)

    def _on_grad(self, p: nn.Parameter) -> None:
        i = self._bucket_of.get(id(p))
        if i is None:
            return
        self._pending[i] -= 1
        if self._pending[i] == 0:
            self._launch(i)

    def _launch(self, i: int) -> None:
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in self.buckets[i]]
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        flat.div_(self.world)
        self._flat[i] = flat
        self._handles[i] = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)

    def finish(self, timeout: datetime.timedelta | None = None) -> None:
        """Wait for every bucket (launching any whose hooks did not fire) and write the averages back.

        A rank that stops taking part (it raised, exited or hangs before its own all-reduce) makes the
        others' waits fail: with the process group's timeout, or ``timeout`` for each bucket's wait when
        given, or as soon as the backend sees the peer's connection close.  That failure is raised here
        as a RuntimeError naming the bucket, before the optimiser could step on partial gradients; the
        reducer is reset, and the process group should then be torn down."""
        if self.world == 1:
            self.reset()
            return
        for i in range(len(self.buckets)):
            if self._handles[i] is None:
                self._launch(i)
        for i, bucket in enumerate(self.buckets):
            try:
                if timeout is None:
                    self._handles[i].wait()
                else:
                    self._handles[i].wait(timeout)
            except Exception as exc:  # backend-specific error types (DistBackendError, RuntimeError, ...)
                self.reset()
                raise RuntimeError(f"gradient all-reduce of bucket {i} of {len(self.buckets)} failed "
                                   f"(a rank left the step?): {exc}") from exc
            flat = self._flat[i]
            offset = 0
            for p in bucket:
                n = p.numel()
                avg = flat[offset:offset + n].view_as(p)
                if p.grad is None:
                    p.grad = avg.to(p.dtype).clone()
                else:
                    p.grad.copy_(avg)
                offset += n
        self.reset()

    def close(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
