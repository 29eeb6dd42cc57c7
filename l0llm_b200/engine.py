"""Continuous batching of greedy generation requests over one multi-sequence model.

The reference's LevelZeroLlmEngine serves one request at a time: a lock around the whole generation
(src/HFLabs.ML.LLM.LevelZero/LevelZeroLlmEngine.cs:22,55) and one sequence per model. This engine keeps up
to `max_batch` requests in flight on an `LlmModel` created with `max_batch` KV-cache rows:

- a waiting request takes the next free row between decode steps; its prompt is prefilled into that row
  and its first token is the prefill's greedy argmax;
- every step decodes all active rows together with one device-resident batched greedy step (rows
  0..n-1, each at its own position), one token per request;
- a request ends at its token budget, at a stop id, or when its row's cache is full; its row is freed by
  moving the last active row into it (`ForkSequence`, a device-side copy), so the active rows stay
  0..n-1.

Tokens are reported per request in order. Greedy decoding only (the device sampler serves sequence 0).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Request:
    rid: int
    prompt: np.ndarray
    max_new_tokens: int
    stop_ids: frozenset
    tokens: list = field(default_factory=list)
    done: bool = False


class BatchEngine:
    def __init__(self, model, max_batch: int, max_seq: int):
        """`model` is an LlmModel created with cfg.max_batch >= max_batch and `max_seq` cache rows."""
        if max_batch < 1:
            raise ValueError("max_batch must be positive")
        self.model = model
        self.max_batch = max_batch
        self.max_seq = max_seq
        self._waiting: deque[Request] = deque()
        self._active: list[Request] = []  # request of row r = self._active[r]
        self._all: dict[int, Request] = {}
        self._next = 0

    def submit(self, prompt_ids, max_new_tokens: int = 256, stop_ids=()) -> int:
        prompt = np.ascontiguousarray(prompt_ids, np.int32)
        if prompt.size == 0:
            raise ValueError("empty prompt")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be positive")
        if prompt.size >= self.max_seq:
            raise ValueError(f"prompt of {prompt.size} tokens does not fit a {self.max_seq}-row cache")
        r = Request(self._next, prompt, max_new_tokens, frozenset(int(t) for t in stop_ids))
        self._next += 1
        self._waiting.append(r)
        self._all[r.rid] = r
        return r.rid

    @property
    def active(self) -> int:
        return len(self._active)

    @property
    def pending(self) -> int:
        return len(self._waiting) + len(self._active)

    def _emit(self, req: Request, tok: int) -> bool:
        """Appends tok; True when the request is finished: its budget, a stop id, or a cache row that
        holds its prompt and tokens (the last token would not fit another step)."""
        req.tokens.append(tok)
        return (len(req.tokens) >= req.max_new_tokens or tok in req.stop_ids
                or req.prompt.size + len(req.tokens) >= self.max_seq)

    def _free_row(self, row: int):
        last = len(self._active) - 1
        if row != last:
            self.model.ForkSequence(last, row, 0)
            self._active[row] = self._active[last]
        self._active.pop()

    def step(self) -> list[tuple[int, int]]:
        """Admits waiting requests into free rows, then decodes one token for every active row.
        Returns the (request id, token) pairs produced by this call, in row order."""
        out: list[tuple[int, int]] = []
        while self._waiting and len(self._active) < self.max_batch:
            req = self._waiting.popleft()
            row = len(self._active)
            logits = self.model.PrefillSequence(row, req.prompt)
            tok = int(np.argmax(logits))
            out.append((req.rid, tok))
            self._active.append(req)
            if self._emit(req, tok):
                req.done = True
                self._free_row(row)
        if not self._active:
            return out
        n = len(self._active)
        toks = self.model.decode_greedy_device_batch(1, n).reshape(-1, n)[-1]
        finished = []
        for row in range(n):
            req = self._active[row]
            tok = int(toks[row])
            out.append((req.rid, tok))
            if self._emit(req, tok):
                finished.append(row)
        for row in sorted(finished, reverse=True):  # highest first: moves never touch a freed row
            self._active[row].done = True
            self._free_row(row)
        return out

    def run(self) -> dict[int, list[int]]:
        """Steps until every submitted request has finished; returns each request's tokens."""
        while self.pending:
            self.step()
        return {rid: r.tokens for rid, r in self._all.items()}
