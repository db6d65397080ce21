"""CUDA-graph capture of a fixed sequence of library calls.

Decode steps issue many short, launch-latency-bound kernels; recording the
sequence once and replaying it removes the per-call host overhead. The
library's compute entry points are stream-ordered and allocation-free once
their context scratch has grown to the shapes used (the warm-up run before
capture does that), so a sequence of them (copies included) can be captured.
"""
import torch


class CapturedSequence:
    def __init__(self, fn, device=None, warmup=1):
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            fn()
        self.fn = fn

    def replay(self):
        self.graph.replay()
