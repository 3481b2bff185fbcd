"""Captured decode steps: the CUDA-graph counterpart of the reference's traced decode.

The reference captures the command stream of a decode step once per lane shape, keeps the
step's inputs in persistent device buffers, refreshes those in place and replays
(src/tt_transformers/llm_runtime/trace_compiler.py:314-541; decode.py:684-819). Here a step
in which every request brings exactly one token is padded to the next captured batch size
(padding rows sit at position 0 and write to the scratch page), its metadata is copied into
a persistent device buffer, and the graph captured for that size is replayed. The logits
live in a buffer that the next replay of the same size overwrites.

A graph is captured per batch size AND per context bucket (the longest context in the step,
rounded up to a power of two): what a launch fixes for good (how many key splits the decode
attention uses, how wide the block tables are) then fits the contexts that are live, not the
longest one the engine admits. The reference keys its decode traces by lane batch and
page-table width in the same way (decode.py:949-961).
"""

from __future__ import annotations

import gc
import weakref
from typing import Dict, List

import torch


OWN_ARGMAX = "own argmax"        # token_feedback value: the tokens are the argmax of this graph's replay before


def _nobodys(engine, host, layout) -> None:
    """Point every row of a step's packed metadata at the scratch page and the scratch slot, at position 0. A capture
    warms the step up by running it once for real: with mixers that keep a running state per request (which a second
    run of the same token would advance twice, unlike a key that is written to the same place twice) that run must
    touch nobody's state. The replay that follows the capture refreshes the buffer with the step's own rows."""
    buf, L = host.numpy(), layout
    T, R, W = L["T"], L["R"], L["W"]
    buf[L["o_pos"]:L["o_pos"] + T] = 0
    buf[L["o_p0"]:L["o_p0"] + R] = 0
    buf[L["o_slot"]:L["o_slot"] + R] = engine.cache.scratch_slot
    for i in range(len(L["groups"])):
        start = L["o_tab"] + i * ((R * W + 3) & ~3)
        buf[start:start + R * W] = 0


class DecodeGraphs:
    def __init__(self, engine):
        self._engine = weakref.ref(engine)       # no cycle with the engine: both go when the last user lets go
        limit = engine.config.max_batch_size
        if engine.config.graph_batch_sizes:
            sizes = [b for b in engine.config.graph_batch_sizes if b < limit]
        else:
            sizes, b = [], 1
            while b < limit:
                sizes.append(b)
                b *= 2
        sizes.append(limit)                       # every batch the engine admits fits a captured size
        self.sizes = sizes
        self._graphs: Dict[tuple, tuple] = {}          # (batch size, context bucket) -> captured step
        self.replays = 0
        self.pool = None
        self._last_key = None
        self.greedy = None

    @property
    def engine(self):
        return self._engine()

    def _bucket(self, rows: int) -> int:
        for s in self.sizes:
            if s >= rows:
                return s
        raise ValueError(f"{rows} requests exceed the engine's max_batch_size")

    MIN_CONTEXT_BUCKET = 1024

    def _context_bucket(self, entries) -> int:
        """The longest context of the step (its new token included), rounded up to a power of two."""
        eng = self.engine
        longest = max(eng.cache.length(e.request_id) for e in entries) + 1
        bucket = self.MIN_CONTEXT_BUCKET
        while bucket < longest:
            bucket *= 2
        return min(bucket, eng.max_seq_len)

    def captured_sizes(self):
        return sorted({size for size, _ in self._graphs})

    def _capture(self, size: int, bucket: int, entries) -> tuple:
        eng = self.engine
        W = -(-bucket // eng.cache.page_size)
        host, layout, lists = eng._fill_host(entries, pad_to=size, table_width=W, want_all=True)
        _nobodys(eng, host, layout)
        static = torch.empty(layout["total"], dtype=torch.int32, device=eng.runtime.device)
        static.copy_(host, non_blocking=True)
        eng._record_staging()
        lists = dict(lists, max_context=bucket)               # key splits are sized for the bucket's longest context
        batch = eng._batch_from(static, layout, lists)
        side = torch.cuda.Stream(device=eng.runtime.device)
        side.wait_stream(torch.cuda.current_stream(eng.runtime.device))
        with torch.cuda.stream(side):                         # warm up outside the capture
            eng.model.forward(batch, eng.cache)
        torch.cuda.current_stream(eng.runtime.device).wait_stream(side)
        torch.cuda.synchronize(eng.runtime.device)
        graph = torch.cuda.CUDAGraph()
        before = eng.kernels.launches
        batch.extras.clear()
        # No garbage collection while the stream is capturing: an object that happens to be collected then
        # (an engine used before, with its pinned buffers, events and graphs) would make CUDA calls that
        # are not allowed during a capture and invalidate it.
        gc_was_on = gc.isenabled()
        gc.disable()                  # (torch.cuda.graph collects once on entry, before the capture begins)
        try:
            with torch.cuda.graph(graph, pool=self.pool):
                logits = eng.model.forward(batch, eng.cache)
                # the greedy choice of every row, left where the next replay's embedding looks for its tokens:
                # a greedy decode loop then needs neither a sampling launch nor a copy between two replays
                greedy = eng.kernels.sample(logits)
                static[layout["o_tok"]:layout["o_tok"] + size].copy_(greedy)
        finally:
            if gc_was_on:
                gc.enable()
        if self.pool is None:
            self.pool = graph.pool()
        kernels_in_graph = eng.kernels.launches - before
        return graph, static, layout, logits, kernels_in_graph, greedy

    def run(self, entries: List, token_feedback: torch.Tensor = None) -> torch.Tensor:
        """Replay the captured step for these entries. With token_feedback (int32 on the device, one
        token per entry, typically what the sampler wrote for the step before) the token ids come
        from there instead of from the entries, so the host need not have seen them yet."""
        eng = self.engine
        rows = len(entries)
        size = self._bucket(rows)
        key = (size, self._context_bucket(entries))
        if key not in self._graphs:
            self._graphs[key] = self._capture(size, key[1], entries)
        graph, static, layout, logits, kernels_in_graph, greedy = self._graphs[key]
        host, new_layout, _ = eng._fill_host(entries, pad_to=size, table_width=layout["W"], want_all=True)
        assert new_layout["total"] == layout["total"]
        if isinstance(token_feedback, str) and token_feedback == OWN_ARGMAX:
            if self._last_key is None or self._last_key[0] != size:
                raise ValueError("OWN_ARGMAX needs the step before to have been a replay of the same captured size")
            first = layout["o_pos"]                     # everything but the token ids, which the replay before left in place
            static[first:].copy_(host[first:], non_blocking=True)
            eng.h2d_bytes += 4 * (host.numel() - first)
            if self._last_key != key:                   # the context grew into the next bucket: another graph's buffer
                static[layout["o_tok"]:layout["o_tok"] + size].copy_(self._graphs[self._last_key][5])
        else:
            static.copy_(host, non_blocking=True)
            eng.h2d_bytes += 4 * host.numel()
        eng._record_staging()
        if torch.is_tensor(token_feedback):
            static[layout["o_tok"]:layout["o_tok"] + rows].copy_(token_feedback[:rows])
        graph.replay()
        self._last_key = key
        self.greedy = greedy[:rows]                     # overwritten by the next replay of this graph
        eng.kernels.launches += kernels_in_graph
        self.replays += 1
        want = [i for i, e in enumerate(entries) if len(e.want)]
        if len(want) == rows:
            return logits[:rows]
        return logits[torch.tensor(want, dtype=torch.long, device=logits.device)] if want else logits[:0]


class PromptGraphs:
    """Captured prompt steps for short prompts, the counterpart of the reference's traced prefill per length
    bucket (src/tt_transformers/llm_runtime/trace_compiler.py:314-541; buckets:
    src/tt_transformers/llm_runtime/prefill/plan.py:448-453).

    A step that brings the first tokens of ONE request (nothing cached yet, at least two tokens, at most the
    largest bucket) and wants the logits of at most one place is padded to the next bucket: the rest of the
    bucket is a second segment at position 0 whose block table points at the scratch page, so what it writes
    and reads is nobody's. The step's metadata, with the query-tile lists of its mixers, is copied into a
    persistent buffer and the graph captured for that bucket is replayed: about 150 launches of the host
    become one. What such a step computes for its real tokens is what the eager step computes: the same
    kernels on the same rows (rows of a matrix product do not depend on one another)."""

    BUCKETS = (32, 64, 128, 256, 512)

    def __init__(self, engine):
        self._engine = weakref.ref(engine)
        limit = min(engine.config.max_step_tokens, engine.config.max_chunk_tokens, engine.max_seq_len)
        self.sizes = [b for b in self.BUCKETS if b <= limit]
        self._graphs: Dict[int, tuple] = {}
        self.replays = 0

    @property
    def engine(self):
        return self._engine()

    def takes(self, entries) -> bool:
        if len(entries) != 1 or not self.sizes:
            return False
        e = entries[0]
        return (2 <= len(e.tokens) <= self.sizes[-1] and len(e.want) <= 1
                and self.engine.cache.length(e.request_id) == 0)

    def _bucket(self, tokens: int) -> int:
        for s in self.sizes:
            if s >= tokens:
                return s
        raise ValueError(f"{tokens} tokens exceed the largest captured prompt step")

    def _fill(self, entries, size):
        eng = self.engine
        entry = entries[0]
        if not entry.want:              # the graph always computes one row of logits; nobody reads it then
            entry = type(entry)(entry.request_id, entry.tokens, [0])
        host, layout, lists = eng._fill_host([entry], table_width=eng.cache.table_width, pad_tokens_to=size)
        # everything a kernel's launch depends on is the bucket's, not the prompt's
        lists = dict(lists, max_context=size, seg_lens=[size, 0], wants_every_row=False)
        return host, layout, lists

    def _capture(self, size: int, entries) -> tuple:
        eng = self.engine
        host, layout, lists = self._fill(entries, size)
        _nobodys(eng, host, layout)
        static = torch.empty(layout["total"], dtype=torch.int32, device=eng.runtime.device)
        static.copy_(host, non_blocking=True)
        eng._record_staging()
        batch = eng._batch_from(static, layout, lists)
        tables = dict(batch.extras)                           # device views into `static`: refreshed with it
        side = torch.cuda.Stream(device=eng.runtime.device)
        side.wait_stream(torch.cuda.current_stream(eng.runtime.device))
        with torch.cuda.stream(side):                         # warm up outside the capture
            eng.model.forward(batch, eng.cache)
        torch.cuda.current_stream(eng.runtime.device).wait_stream(side)
        torch.cuda.synchronize(eng.runtime.device)
        graph = torch.cuda.CUDAGraph()
        before = eng.kernels.launches
        batch.extras.clear()
        batch.extras.update(tables)                           # what the warm-up derived on the host is derived again
        gc_was_on = gc.isenabled()
        gc.disable()                  # no collection (of engines used before, with CUDA objects) while capturing
        try:
            pool = eng.graphs.pool if eng.graphs is not None else None
            with torch.cuda.graph(graph, pool=pool):
                logits = eng.model.forward(batch, eng.cache)
        finally:
            if gc_was_on:
                gc.enable()
        if eng.graphs is not None and eng.graphs.pool is None:
            eng.graphs.pool = graph.pool()
        return graph, static, layout, logits, eng.kernels.launches - before

    def run(self, entries) -> torch.Tensor:
        eng = self.engine
        size = self._bucket(len(entries[0].tokens))
        if size not in self._graphs:
            self._graphs[size] = self._capture(size, entries)
        graph, static, layout, logits, kernels_in_graph = self._graphs[size]
        host, new_layout, _ = self._fill(entries, size)
        assert new_layout["total"] == layout["total"] and new_layout["extras"] == layout["extras"]
        static.copy_(host, non_blocking=True)
        eng.h2d_bytes += 4 * host.numel()
        eng._record_staging()
        graph.replay()
        eng.kernels.launches += kernels_in_graph
        self.replays += 1
        return logits if entries[0].want else logits[:0]
