"""Graph-captured batch-1 (or MTP-verify width) decode step of the EXL3 decoder.

The reference's decode speed comes from oMLX's generate loop with MLX's lazy graph and asynchronous
evaluation (src/tools/exl3_decode_bench.py:126-138). Here one decode step (embedding -> all layers ->
head -> greedy token) is captured once in a CUDA graph and replayed, with the token and position
read from static device buffers. Under tensor parallelism the row-parallel sums are this package's
NVLink peer kernels (comm.PeerGroup) inside the same graph, or NCCL all-reduces with
OMLX_EXL3_PEER_AR=0; the greedy token's (value, index) pairs are all-gathered with NCCL.

The peer kernels never hang on a stalled rank: each wait gives up after a bounded time and sets a
status bit. `check()` reads those bits (and the prefill GEMM's) and raises; `step()` calls it every
`check_every` steps, outside graph replay.
"""
from __future__ import annotations

import os

import torch

from .kernels import check_gemm_status
from .model import KVCache, Qwen3EXL3


class DecodeRunner:
    def __init__(self, model: Qwen3EXL3, cache: KVCache, rows: int = 1, use_graph: bool = True,
                 check_every: int = 64):
        self.model, self.cache, self.rows = model, cache, rows
        dev = model.rope_cos.device
        self.device = dev
        self.check_every = check_every          # steps between status reads (0: only explicit check())
        self._unchecked = 0
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
        self.check()

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
        self._unchecked += 1
        if self.check_every and self._unchecked >= self.check_every:
            self.check()
        return self.next_tokens

    def check(self):
        """Raise RuntimeError if a bounded wait of the step's kernels ever gave up: a peer rank that
        stopped delivering its all-reduce partials (the step's outputs since then are invalid), or a
        prefill GEMM pipeline wait. Reads device memory, so it waits for the work queued so far."""
        self._unchecked = 0
        peers = self.model.tp.peers
        if peers is not None:
            st = peers.status()
            if st:
                raise RuntimeError(f"tensor-parallel rank {self.model.tp.rank}: a wait for another rank's "
                                   f"all-reduce data timed out (peer status 0x{st:x})")
        check_gemm_status(self.device)

    def release(self):
        """Drop the captured graph (needed before destroying a process group it holds NCCL calls of)."""
        self.graph = None
