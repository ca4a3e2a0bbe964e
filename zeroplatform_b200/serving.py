"""Continuous batching over one device engine: the host mirror of LlmEngine.GenerateStreamAsync / CompleteAsync
(ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs:51-152) for many concurrent callers.

The reference runs each GenerateStreamAsync call's prefill and decode loop on its own over a shared PagedKvCache.
Here every call becomes a request of the engine's scheduler (zcu_engine_submit): concurrent streams share each
decode step (zcu_engine_serve_step), requests join as soon as a page-table row and their pages are free and leave
when they finish, so a stream never waits for another one to end.  Token ids in, token ids out (tokenization is
outside this package).
"""
from __future__ import annotations

import asyncio
import itertools
from dataclasses import dataclass, field

from ._lib import SERVE_CANCELLED, SERVE_REFUSED, SERVE_STOP_TOKEN, ZcError


@dataclass
class SamplingConfig:
    """SamplingConfig (ZeroLlm/src/ZeroLlm.Core/Sampling/SamplingConfig.cs:9-26), numeric fields and stop tokens."""

    temperature: float = 0.7
    top_p: float = 0.9
    min_p: float = 0.0
    top_k: int = 40
    repetition_penalty: float = 1.1
    max_tokens: int = 256
    stop_tokens: set = field(default_factory=set)

    @staticmethod
    def greedy() -> "SamplingConfig":
        return SamplingConfig(temperature=0.0, top_p=1.0, top_k=1, repetition_penalty=1.0)


class ContinuousBatcher:
    """Drives an engine's scheduler for any number of concurrent streams.

    `generate_stream_async(prompt, sampling, seed)` is an async generator of token ids (GenerateStreamAsync);
    `complete_async` collects one (CompleteAsync).  A single driver task calls serve_step while any stream's
    request is unfinished; each step's events are routed to their streams.  `run(requests)` is the synchronous form
    for a fixed set of requests.  eos_token ends a stream like the model's EosTokenId.
    """

    def __init__(self, engine, eos_token: int = -1, first_seq_id: int = 1 << 20):
        self.engine = engine
        self.eos_token = eos_token
        self._ids = itertools.count(first_seq_id)  # Interlocked.Increment(ref _nextSeqId)
        self._queues: dict[int, asyncio.Queue] = {}
        self._open: set[int] = set()  # streams whose request has not finished
        self._driver: asyncio.Task | None = None

    def _submit(self, prompt, sampling: SamplingConfig | None, seed: int) -> int:
        s = sampling or SamplingConfig()
        sid = next(self._ids)
        self.engine.submit(sid, prompt, s.max_tokens, temperature=s.temperature, top_p=s.top_p, min_p=s.min_p,
                           top_k=s.top_k, repetition_penalty=s.repetition_penalty, seed=seed,
                           eos_token=self.eos_token, stop_tokens=s.stop_tokens)
        return sid

    def step(self):
        """One scheduler iteration; returns its events."""
        return self.engine.serve_step()

    def run(self, requests):
        """requests: [(prompt, SamplingConfig | None, seed)] -> [token list] in request order."""
        ids = [self._submit(p, s, seed) for p, s, seed in requests]
        out = {i: [] for i in ids}
        open_ids = set(ids)
        while open_ids:
            for sid, tok, finished, reason in self.step():
                if sid not in out:
                    continue
                if tok >= 0 and reason != SERVE_STOP_TOKEN:
                    out[sid].append(tok)
                if finished:
                    open_ids.discard(sid)
                    if reason == SERVE_REFUSED:
                        raise ZcError(f"request {sid}: more than 4096 sampling candidates after Top-K")
        return [out[i] for i in ids]

    async def _drive(self):
        # runs while a stream's request is unfinished (a stream abandoned without closing runs to its end)
        while self._open:
            for sid, tok, finished, reason in self.step():
                if finished:
                    self._open.discard(sid)
                q = self._queues.get(sid)
                if q is not None:
                    q.put_nowait((tok, finished, reason))
            await asyncio.sleep(0)  # let the streams consume (Task.Yield in the reference's loop)
        self._driver = None

    async def generate_stream_async(self, prompt, sampling: SamplingConfig | None = None, seed: int = 0):
        if len(prompt) == 0:  # GenerateStreamAsync yields nothing for an empty prompt
            return
        sid = self._submit(prompt, sampling, seed)
        q: asyncio.Queue = asyncio.Queue()
        self._queues[sid] = q
        self._open.add(sid)
        if self._driver is None:
            self._driver = asyncio.get_running_loop().create_task(self._drive())
        done = False
        try:
            while True:
                tok, finished, reason = await q.get()
                done = bool(finished)
                if reason == SERVE_REFUSED:
                    raise ZcError(f"request {sid}: more than 4096 sampling candidates after Top-K")
                if tok >= 0 and reason not in (SERVE_STOP_TOKEN, SERVE_CANCELLED):
                    yield tok
                if finished:
                    return
        finally:
            self._queues.pop(sid, None)
            if not done and sid in self._open:  # the caller stopped early (its CancellationToken)
                self.engine.cancel(sid)  # the CANCELLED event of the next step frees the request's pages

    async def complete_async(self, prompt, sampling: SamplingConfig | None = None, seed: int = 0):
        return [t async for t in self.generate_stream_async(prompt, sampling, seed)]
