"""CUDA-graph capture of a whole training step.

A logic network's step is a few dozen kernels (layer forwards and backwards, the logit finalize, the
loss, clipping, the optimizer).  For small layers (the 784 -> 12000 layer of the c1 configuration, the
conv model of c3) the GPU finishes each kernel faster than Python and ctypes can issue the next one, so
an eager step is bound by host overhead.  ``GraphedTrainStep`` records the step once into a CUDA graph
and replays it: one host call per step, the same kernels and the same arithmetic.

The layers need nothing special for capture: every kernel is enqueued on the current stream, scratch
tensors come from torch's caching allocator (the graph's private pool during capture), and the step
performs no host synchronisation once the layers' slot tables exist (they are built during the eager
warm-up steps).  Inputs are copied into static buffers before each replay; outputs (the loss, the
parameters' ``.grad``) live in the graph's pool and are overwritten by the next replay.  A layer whose
connection buffers change after capture (resampling) must be re-captured.
"""
from typing import Callable, Iterable, Optional

import torch


class GraphedTrainStep:
    """``step(x, y) -> loss`` for ``optimizer.zero_grad(); loss_fn(model(x), y).backward(); clip; optimizer.step()``.

    The optimizer must be capturable (``torch.optim.Adam(..., capturable=True)``).  ``warmup`` eager steps
    run on a side stream before capture (they update the parameters like any training step)."""

    def __init__(self, model: torch.nn.Module, optimizer: torch.optim.Optimizer, loss_fn: Callable,
                 x: torch.Tensor, y: torch.Tensor, clip: Optional[float] = None,
                 params: Optional[Iterable[torch.nn.Parameter]] = None, warmup: int = 3):
        self.model, self.opt, self.loss_fn, self.clip = model, optimizer, loss_fn, clip
        self.params = [p for p in (params if params is not None else model.parameters()) if p.requires_grad]
        self.x = x.detach().clone()
        self.y = y.detach().clone()
        side = torch.cuda.Stream(device=self.x.device)
        side.wait_stream(torch.cuda.current_stream(self.x.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._body()
        torch.cuda.current_stream(self.x.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = self._body()

    def _body(self):
        self.opt.zero_grad(set_to_none=True)
        loss = self.loss_fn(self.model(self.x), self.y)
        loss.backward()
        if self.clip is not None:
            torch.nn.utils.clip_grad_norm_(self.params, self.clip)
        self.opt.step()
        return loss

    def __call__(self, x: Optional[torch.Tensor] = None, y: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        if y is not None:
            self.y.copy_(y, non_blocking=True)
        self.graph.replay()
        return self.loss


class GraphedLayerPass:
    """Forward + backward of one module for a fixed upstream gradient, captured once:
    ``(grad_input, grad_params...) = pass(x, grad_out)``, the gradients returned by torch.autograd.grad."""

    def __init__(self, module: torch.nn.Module, x: torch.Tensor, grad_out: torch.Tensor, warmup: int = 3):
        self.module = module
        self.params = [p for p in module.parameters() if p.requires_grad]
        self.x = x.detach().clone().requires_grad_(True)
        self.g = grad_out.detach().clone()
        side = torch.cuda.Stream(device=self.x.device)
        side.wait_stream(torch.cuda.current_stream(self.x.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._body()
        torch.cuda.current_stream(self.x.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()

    def _body(self):
        return torch.autograd.grad(self.module(self.x), [self.x] + self.params, self.g)

    def __call__(self, x: Optional[torch.Tensor] = None, grad_out: Optional[torch.Tensor] = None):
        if x is not None:
            self.x.data.copy_(x, non_blocking=True)
        if grad_out is not None:
            self.g.copy_(grad_out, non_blocking=True)
        self.graph.replay()
        return self.out
