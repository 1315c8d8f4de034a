"""CUDA Graph replay of the whole forward (cuda_graph_runner.py:24-129).

``FixedInputCUDAGraph`` captures ONE ``tfx_forward`` call (every kernel of
the forward) for a fixed input object and replays it; ``maybe_cuda_graph``
keeps the reference's contract (eager-vs-replay equality check, fallback to
eager with a reason). ``ForwardGraph`` is the allocation-free variant the
benchmark uses: static input/output buffers, replay without the clone.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn


def _tensor_version(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return -1
    try:
        return t._version
    except RuntimeError:
        return None


class ForwardGraph:
    """Capture ``model.run_into(x, y)`` once; ``replay()`` re-runs it.

    The input and output are the caller's tensors; replay reads ``x`` and
    overwrites ``y`` in place, so write new inputs into ``x`` (``copy_``)
    between replays. The workspace is allocated before capture.
    """

    def __init__(self, model, x: torch.Tensor, y: torch.Tensor,
                 valid_len: Optional[torch.Tensor] = None, warmup: int = 1) -> None:
        if not x.is_cuda:
            raise ValueError("CUDA Graph inputs must be CUDA tensors")
        self.model = model
        self.x = x
        self.y = y
        self.valid_len = valid_len
        device = x.device
        _, _, _, mdl = model._prepare(device)
        self.workspace = model._workspace_for(device, mdl, x.shape[0], x.shape[1])
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                model.run_into(x, y, valid_len, self.workspace)
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        # thread_local: only this thread's CUDA calls are checked during the
        # capture, so another thread of the process (a NCCL process group's
        # watchdog polling its events) cannot invalidate it.
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            model.run_into(x, y, valid_len, self.workspace)
        torch.cuda.synchronize(device)

    def replay(self) -> None:
        self.graph.replay()


class FixedInputCUDAGraph(nn.Module):
    """Replay the captured forward for the exact captured input objects
    (cuda_graph_runner.py:24-93); any other input runs eagerly."""

    def __init__(self, model: nn.Module, example_x: torch.Tensor,
                 example_mask: Optional[torch.Tensor], warmup_iterations: int = 3) -> None:
        super().__init__()
        if not example_x.is_cuda or (example_mask is not None and not example_mask.is_cuda):
            raise ValueError("CUDA Graph inputs must be CUDA tensors")
        if model.training:
            raise ValueError("CUDA Graph inference requires model.eval()")
        self.model = model
        self._captured_x = example_x
        self._captured_mask = example_mask
        self._x_version = _tensor_version(example_x)
        self._mask_version = _tensor_version(example_mask)
        if self._x_version is None or self._mask_version is None:
            raise ValueError("CUDA Graph inputs must expose mutation version counters")
        with torch.inference_mode():
            for _ in range(warmup_iterations):
                model(example_x, example_mask)  # caches mask inspection + weight packing
            valid_len = model._valid_lengths(example_x, example_mask)
        self._output = torch.empty_like(example_x)
        self._graph = ForwardGraph(model, example_x.contiguous(), self._output, valid_len)

    def _matches(self, x, mask) -> bool:
        return (
            x is self._captured_x
            and mask is self._captured_mask
            and _tensor_version(x) == self._x_version
            and _tensor_version(mask) == self._mask_version
        )

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None):
        if not self._matches(x, valid_token_mask):
            return self.model(x, valid_token_mask)
        self._graph.replay()
        # Graph outputs live in persistent storage; clone as the reference does.
        return self._output.clone()


def maybe_cuda_graph(model: nn.Module, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor],
                     enabled: bool) -> Tuple[nn.Module, bool, str]:
    """cuda_graph_runner.py:96-129: graphed module or eager with a reason."""
    if not enabled:
        return model, False, "disabled"
    if not x.is_cuda:
        return model, False, "CUDA Graphs require a CUDA input"
    if bool(getattr(model, "_kv_cache_enabled", False)):
        return model, False, "stateful KV-cache decoding uses the eager path"
    try:
        with torch.inference_mode():
            eager = model(x, valid_token_mask)
        wrapped = FixedInputCUDAGraph(model, x, valid_token_mask)
        with torch.inference_mode():
            replayed = wrapped(x, valid_token_mask)
    except (RuntimeError, ValueError) as error:
        return model, False, f"capture failed: {error}"
    if not torch.equal(eager, replayed):
        err = float((eager.float() - replayed.float()).abs().max().item())
        return model, False, f"replay validation failed (max_abs={err:.3g})"
    return wrapped, True, "whole-forward CUDA Graph replay"
