"""Graph-captured batch-1 (or MTP-verify width) decode step of the EXL3 decoder.

The reference's decode speed comes from oMLX's generate loop with MLX's lazy graph and asynchronous
evaluation (src/tools/exl3_decode_bench.py:126-138). Here one decode step (embedding -> all layers ->
head -> greedy token) is captured once in a CUDA graph and replayed, with the token and position
read from static device buffers; tensor-parallel all-reduces and the logit gather are NCCL calls
inside the same graph.
"""
from __future__ import annotations

import os

import torch

from .model import KVCache, Qwen3EXL3


class DecodeRunner:
    def __init__(self, model: Qwen3EXL3, cache: KVCache, rows: int = 1, use_graph: bool = True):
        self.model, self.cache, self.rows = model, cache, rows
        dev = model.rope_cos.device
        self.device = dev
        self.tokens = torch.zeros(rows, dtype=torch.long, device=dev)
        self.pos = torch.arange(cache.length, cache.length + rows, dtype=torch.long, device=dev)
        self.next_tokens = None
        self.logits = None
        self.graph = None
        if os.environ.get("OMLX_EXL3_PEER_AR", "1") != "0":
            model.setup_peers(rows)      # tensor-parallel: fused NVLink all-reduce (collective)
        self._run()                      # eager pass: builds GEMV plans and their scratch
        torch.cuda.synchronize(dev)
        if use_graph:
            self.stream = torch.cuda.Stream(dev)
            self.stream.wait_stream(torch.cuda.current_stream(dev))
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(self.stream):
                self._run()              # second eager pass on the capture stream
                with torch.cuda.graph(self.graph, stream=self.stream):
                    self._run()
            torch.cuda.current_stream(dev).wait_stream(self.stream)
            torch.cuda.synchronize(dev)

    @torch.no_grad()
    def _run(self):
        local = self.model(self.tokens, self.cache, self.pos)
        self.logits = local
        self.next_tokens = self.model.greedy(local)

    @torch.no_grad()
    def step(self, tokens: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step at the cache's current length (the cache length is not advanced: the
        benchmark repeats the same position). Returns the greedy next token(s) on the device."""
        if tokens is not None:
            self.tokens.copy_(tokens, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._run()
        return self.next_tokens

    def release(self):
        """Drop the captured graph (needed before destroying a process group it holds NCCL calls of)."""
        self.graph = None
