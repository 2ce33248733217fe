"""CUDA-graph capture of a whole step (the reference engine's graph mode,
``kairos_ext/kairos_engine.cu:6352-6450``, here over this library's kernels,
cuBLAS and NCCL).

``GraphedStep(fn, *example_inputs)`` runs ``fn`` eagerly on a side stream to
warm it up (cuBLAS handles, tensor-map encoders, NCCL communicators), then
captures one call into a ``torch.cuda.CUDAGraph`` whose inputs and output are
persistent device buffers.  ``step(*inputs)`` copies the new inputs into those
buffers and replays the graph: one launch instead of the ~30 kernels, GEMMs
and exchanges of a DiT block each issued from Python.  The returned tensor is
the persistent output buffer, overwritten by the next replay.

Everything a step allocates (activations, workspaces) comes from the graph's
private memory pool and stays resident between replays.
"""
from __future__ import annotations

import torch


class GraphedStep:
    def __init__(self, fn, *example_inputs, warmup: int = 2, static_inputs: bool = False):
        """``static_inputs=True`` makes the given tensors themselves the graph's
        input buffers (the caller writes them, e.g. by its own copies) instead
        of private clones."""
        if not all(isinstance(x, torch.Tensor) and x.is_cuda for x in example_inputs):
            raise ValueError('GraphedStep: inputs must be CUDA tensors')
        self.fn = fn
        self.inputs = list(example_inputs) if static_inputs else [x.clone() for x in example_inputs]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):
                fn(*self.inputs)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.output = fn(*self.inputs)

    def __call__(self, *inputs):
        """Copy ``inputs`` (if given) into the input buffers and replay."""
        for dst, src in zip(self.inputs, inputs):
            if src is not dst:
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.output
