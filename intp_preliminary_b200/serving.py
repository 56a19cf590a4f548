"""Inference drivers for the half6d3r forward on one GPU.

``GraphedForward``   captures ``model(images)`` for a fixed device buffer in a
                     CUDA graph; ``replay()`` re-runs the ~100 kernels of the
                     forward with one launch.
``PipelinedInference`` streams batches from pinned host memory: while batch i
                     runs (graph replay on the compute stream), batch i+1 is
                     copied host->device on a copy stream into the other of two
                     input buffers, and batch i's logits are copied back.

The reference's evaluation loop (experiments/imagenet100/train_vit.py:433-476)
copies each batch to the device and then runs the model, one after the other;
these drivers keep the same per-batch work and overlap the copies.
"""

from __future__ import annotations

import torch

from .share_vit import IMAGE_SIZE, IN_CHANS


class GraphedForward:
    """``model(images)`` captured in a CUDA graph for one static input buffer."""

    def __init__(self, model, images: torch.Tensor, warmup: int = 2):
        if not images.is_cuda:
            raise ValueError("images must be a CUDA tensor")
        self.model = model
        self.images = images
        if getattr(model, "attention_events", None) is not None:
            raise ValueError("disable attention_events before capturing")
        side = torch.cuda.Stream(images.device)
        side.wait_stream(torch.cuda.current_stream(images.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):  # builds every cache (packed slots, rendered prototypes, cuBLAS handles)
                model(images)
        torch.cuda.current_stream(images.device).wait_stream(side)
        torch.cuda.synchronize(images.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.logits = model(images)

    def replay(self) -> torch.Tensor:
        """Run the captured forward on the current contents of ``images``;
        returns the (static) logits tensor."""
        self.graph.replay()
        return self.logits


class PipelinedInference:
    """Host batches in, host logits out, with copies overlapped with compute."""

    def __init__(self, model, batch: int, device: torch.device, graphed: bool = True):
        self.device = torch.device(device)
        self.batch = batch
        self.copy_stream = torch.cuda.Stream(self.device)
        self.buffers = [torch.zeros(batch, IN_CHANS, IMAGE_SIZE, IMAGE_SIZE, device=self.device) for _ in range(2)]
        if graphed:
            self.runners = [GraphedForward(model, buf) for buf in self.buffers]
            self.forward = [r.replay for r in self.runners]
        else:
            self.forward = [lambda buf=buf: model(buf) for buf in self.buffers]
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]

    def _issue_copy(self, host: torch.Tensor, slot: int) -> None:
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.consumed[slot])  # the forward that read this buffer is done
            self.buffers[slot].copy_(host, non_blocking=True)
            self.copied[slot].record(self.copy_stream)

    def run(self, host_batches, host_logits, after_forward=None) -> None:
        """Enqueue every batch of ``host_batches`` (pinned (batch, 3, 224, 224)
        float32) and its logits copy into ``host_logits[i]`` (pinned); returns
        once everything is enqueued (synchronize the current stream to wait).
        ``after_forward(i, logits)`` may transform the device logits of batch i
        (for example gather them across ranks) and returns the tensor to copy."""
        compute = torch.cuda.current_stream(self.device)
        self.copy_stream.wait_stream(compute)
        n = len(host_batches)
        if n == 0:
            return
        for slot in range(2):
            self.consumed[slot].record(compute)
        self._issue_copy(host_batches[0], 0)
        for i in range(n):
            slot = i % 2
            if i + 1 < n:
                self._issue_copy(host_batches[i + 1], (i + 1) % 2)
            compute.wait_event(self.copied[slot])
            logits = self.forward[slot]()
            self.consumed[slot].record(compute)
            out = after_forward(i, logits) if after_forward is not None else logits
            if out is not None:
                host_logits[i].copy_(out.float(), non_blocking=True)
