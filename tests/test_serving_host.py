"""serving.ContinuousBatcher's host logic (event routing, stop / cancel handling, the async driver) against a fake
engine that follows zcu_engine_serve_step's event contract: no GPU."""
import asyncio

from zeroplatform_b200._lib import SERVE_CANCELLED, SERVE_MAX_TOKENS, SERVE_RUNNING, SERVE_STOP_TOKEN
from zeroplatform_b200.serving import ContinuousBatcher, SamplingConfig


class FakeEngine:
    """Runs at most `max_batch` requests; request s emits tokens 1000*s + prompt[0] + i; eos / stop tokens end it."""

    def __init__(self, max_batch=2):
        self.max_batch = max_batch
        self.queue, self.active, self.cancelled = [], {}, []
        self.steps = 0

    def submit(self, sid, prompt, max_new, eos_token=-1, stop_tokens=(), seed=0, **_):
        self.queue.append((sid, int(prompt[0]), max_new, eos_token, set(stop_tokens)))

    def cancel(self, sid):
        for q in self.queue:
            if q[0] == sid:
                self.queue.remove(q)
                self.cancelled.append(sid)
                return
        self.active[sid]["cancel"] = True

    def serve_counts(self):
        return len(self.active), len(self.queue)

    def serve_step(self):
        self.steps += 1
        ev = [(s, -1, 1, SERVE_CANCELLED) for s in self.cancelled]
        self.cancelled = []
        for s in [s for s, r in self.active.items() if r["cancel"]]:
            ev.append((s, -1, 1, SERVE_CANCELLED))
            del self.active[s]
        while self.queue and len(self.active) < self.max_batch:
            sid, p0, n, eos, stop = self.queue.pop(0)
            self.active[sid] = dict(p0=p0, n=n, i=0, eos=eos, stop=stop, cancel=False)
        for s in list(self.active):
            r = self.active[s]
            tok = 1000 * s + r["p0"] + r["i"]
            if tok == r["eos"] or tok in r["stop"]:
                ev.append((s, tok, 1, SERVE_STOP_TOKEN))
                del self.active[s]
                continue
            r["i"] += 1
            fin = r["i"] >= r["n"]
            ev.append((s, tok, int(fin), SERVE_MAX_TOKENS if fin else SERVE_RUNNING))
            if fin:
                del self.active[s]
        return ev


def test_run_routes_events_and_drops_stop_tokens():
    e = FakeEngine()
    b = ContinuousBatcher(e, first_seq_id=1)
    out = b.run([([5], SamplingConfig(max_tokens=4), 0), ([7], SamplingConfig(max_tokens=3, stop_tokens={2009}), 0),
                 ([1], SamplingConfig(max_tokens=2), 0)])
    assert out == [[1005, 1006, 1007, 1008], [2007, 2008], [3001, 3002]]
    assert e.serve_counts() == (0, 0)


def test_async_streams_and_early_close_cancel():
    e = FakeEngine(max_batch=3)
    b = ContinuousBatcher(e, first_seq_id=1)

    async def main():
        outs = await asyncio.gather(b.complete_async([3], SamplingConfig(max_tokens=5)),
                                    b.complete_async([4], SamplingConfig(max_tokens=2)),
                                    b.complete_async([], SamplingConfig(max_tokens=2)))
        stream = b.generate_stream_async([9], SamplingConfig(max_tokens=100))
        got = []
        async for t in stream:
            got.append(t)
            if len(got) == 3:
                break
        await stream.aclose()
        while b._driver is not None:
            await asyncio.sleep(0)
        return outs, got

    outs, got = asyncio.run(main())
    assert outs == [[1003, 1004, 1005, 1006, 1007], [2004, 2005], []]
    assert got == [3009, 3010, 3011]
    assert e.serve_counts() == (0, 0) and e.steps < 20  # the abandoned stream was cancelled, not run to 100
