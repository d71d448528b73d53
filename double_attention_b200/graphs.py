"""One module step replayed from a CUDA graph, with static device buffers.

An eager call of ``SharedDictionaryAttention`` enqueues every launch through Python, autograd and
ctypes: on one B200 about 0.17 ms of host time for the forward of preset ``a1`` at batch 8 x 512
(0.06 ms of device time), about 1.9 ms for the forward and backward of ``qk4-s4`` at 16 x 2048.  When
the per-step device work is small -- short batches, or a global batch split over many GPUs -- the host
sets the pace.  :class:`GraphedModuleStep` captures one call (forward, or forward and backward) once
and replays it with a single graph launch, so the step costs its device time.

The captured step reads the static input buffers ``x`` (and ``dy``) and leaves its result (the output,
or the input gradient) in one static output tensor that the next replay overwrites.  With
``backward=True`` the parameters' ``.grad`` tensors after capture are the graph's own gradient buffers,
overwritten (not accumulated) by every replay; do not set them to ``None`` between replays.  The
module, its parameters' storage and the step's shapes must not change after capture.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn


class GraphedModuleStep:
    """``module(x)`` (and ``.backward(dy)``) captured once, replayed per call.

    ``input_shape``/``dtype`` are those of ``x``; the device is the module's.  Calling the object with
    device tensors copies them into the static inputs (on the current stream), replays the graph and
    returns the static result: ``module(x)`` for a forward step, ``d loss / d x`` for a backward step
    (the loss being ``<module(x), dy>``).  Arguments left out keep the static inputs' contents.
    """

    def __init__(self, module: nn.Module, input_shape: tuple[int, ...], dtype: torch.dtype,
                 backward: bool = False, warmup: int = 2) -> None:
        params = list(module.parameters())
        if not params or not params[0].is_cuda:
            raise RuntimeError("GraphedModuleStep needs a module on a CUDA device")
        self.module = module
        self.backward = backward
        self.device = params[0].device
        self._params = params
        self.x = torch.zeros(input_shape, dtype=dtype, device=self.device)
        self.dy = torch.zeros(input_shape, dtype=dtype, device=self.device) if backward else None
        stream = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):  # warm-up off the capturing stream, as graph capture requires
            for _ in range(max(1, warmup)):
                self._step()
        stream.wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._step()

    def _step(self) -> Tensor:
        if not self.backward:
            with torch.no_grad():
                return self.module(self.x)
        for p in self._params:
            p.grad = None
        x = self.x.detach().requires_grad_(True)
        self.module(x).backward(self.dy)
        return x.grad

    def __call__(self, x: Tensor | None = None, dy: Tensor | None = None) -> Tensor:
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        if dy is not None:
            if self.dy is None:
                raise ValueError("dy given to a forward-only step")
            self.dy.copy_(dy, non_blocking=True)
        self.graph.replay()
        return self.out
