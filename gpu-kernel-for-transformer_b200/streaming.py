"""Forward of host-resident batches with copy/compute overlap.

The reference streams a long batch one sample at a time through the model on
the device (streamed_shape14.py:122-186) and leaves host transfers to the
caller. Here batches live in (pinned) host memory and a three-stream pipeline
keeps the PCIe link busy in both directions while the forward runs:

    upload stream    x_host[k] -> x_dev[k % depth]
    compute stream   y_dev[k % depth] = forward(x_dev[k % depth])
    download stream  y_dev[k % depth] -> y_host[k]

so step k's download, step k+1's forward and step k+2's upload overlap.
PCIe is full duplex: for a forward that is short next to its transfers (the
c2 workload moves 655 MB each way per 4.5 ms forward) the step time drops
from upload + forward + download to about the slower of the two copies.
Device slots are reused only after the events that prove the previous user is
done: an upload waits for the forward that read the slot, a forward waits for
the download that drained its output slot. All work is enqueued
asynchronously; the caller synchronises (or reads an event) before touching
the host outputs.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch


class StreamingForward:
    """Pipelined forward of many equally-shaped host batches.

    model: a UserOptimizedTransformer on `device`; batch, seq: the shape of
    every batch; depth: device slots per direction (2 = double buffering).
    """

    def __init__(self, model, device: torch.device, batch: int, seq: int, depth: int = 2):
        if depth < 2:
            raise ValueError("depth must be >= 2 for copies to overlap the forward")
        self.model = model
        self.device = torch.device(device)
        shape = (batch, seq, model.config.d_model)
        self.depth = depth
        self.x_dev = [torch.empty(shape, device=self.device) for _ in range(depth)]
        self.y_dev = [torch.empty(shape, device=self.device) for _ in range(depth)]
        _, _, _, mdl = model._prepare(self.device)
        self.workspace = model._workspace_for(self.device, mdl, batch, seq)
        self.up = torch.cuda.Stream(self.device)
        self.compute = torch.cuda.Stream(self.device)
        self.down = torch.cuda.Stream(self.device)
        self.uploaded = [torch.cuda.Event() for _ in range(depth)]
        self.consumed = [torch.cuda.Event() for _ in range(depth)]
        self.drained = [torch.cuda.Event() for _ in range(depth)]
        self._steps = 0  # slot-reuse bookkeeping continues across run() calls

    def run(self, x_host: Sequence[torch.Tensor], y_host: Sequence[torch.Tensor],
            valid_len: Optional[torch.Tensor] = None) -> torch.cuda.Event:
        """Enqueue the forward of every x_host[i] into y_host[i] (pinned fp32
        host tensors of the configured shape; y_host entries may repeat).
        Returns an event recorded after the last download."""
        if len(x_host) != len(y_host):
            raise ValueError("x_host and y_host must have the same length")
        for xh, yh in zip(x_host, y_host):
            if xh.device.type != "cpu" or yh.device.type != "cpu":
                raise ValueError("StreamingForward moves host tensors; got a device tensor")
            if xh.shape != self.x_dev[0].shape or yh.shape != self.y_dev[0].shape:
                raise ValueError(f"batches must have shape {tuple(self.x_dev[0].shape)}")
            if xh.dtype != torch.float32 or yh.dtype != torch.float32:
                raise ValueError("host batches must be float32")
        # Work already queued on the caller's stream (weights, inputs) first.
        caller = torch.cuda.current_stream(self.device)
        for s in (self.up, self.compute, self.down):
            s.wait_stream(caller)
        for xh, yh in zip(x_host, y_host):
            k, slot = self._steps, self._steps % self.depth
            reuse = k >= self.depth
            with torch.cuda.stream(self.up):
                if reuse:
                    self.up.wait_event(self.consumed[slot])
                self.x_dev[slot].copy_(xh, non_blocking=True)
                self.uploaded[slot].record(self.up)
            with torch.cuda.stream(self.compute):
                self.compute.wait_event(self.uploaded[slot])
                if reuse:
                    self.compute.wait_event(self.drained[slot])
                self.model.run_into(self.x_dev[slot], self.y_dev[slot], valid_len,
                                    workspace=self.workspace)
                self.consumed[slot].record(self.compute)
            with torch.cuda.stream(self.down):
                self.down.wait_event(self.consumed[slot])
                yh.copy_(self.y_dev[slot], non_blocking=True)
                self.drained[slot].record(self.down)
            self._steps += 1
        done = torch.cuda.Event()
        done.record(self.down)
        caller.wait_stream(self.down)
        return done

    def capture(self, x_host: Sequence[torch.Tensor], y_host: Sequence[torch.Tensor],
                valid_len: Optional[torch.Tensor] = None) -> torch.cuda.CUDAGraph:
        """The whole pipelined run(x_host, y_host) as one CUDA Graph, for a
        serving loop that refills the same pinned host buffers: each replay
        uploads every x_host[i], runs its forward and downloads into
        y_host[i], with the same stream overlap as run(), and no per-step
        host work. Replay on the caller's stream; read y_host after the
        replay has completed.

        The capture starts from fresh slots, so its waits refer only to events
        recorded inside it; replays are ordered on the stream, so one replay's
        slot reuse never races the next."""
        torch.cuda.synchronize(self.device)
        self._steps = 0
        graph = torch.cuda.CUDAGraph()
        # thread_local: other threads (a NCCL watchdog) stay free to query
        # their events while this thread captures.
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            self.run(x_host, y_host, valid_len)
        self._steps = 0
        return graph
