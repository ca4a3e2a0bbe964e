"""Continuous batching (zcu_engine_submit / zcu_engine_serve_step, serving.ContinuousBatcher) vs the oracle.

Every request must produce what LlmEngine.GenerateStreamAsync (LlmEngine.cs:71-152) produces for it alone: greedy
requests the oracle's greedy tokens exactly (with and without the repetition penalty, prompts on both sides of the
tiled-prefill threshold), sampled requests the oracle's token for the same history and the same draw
zcu_sample_uniform(seed, i) wherever the draw is not within 2e-3 of a boundary of the oracle's distribution -- while
requests of different lengths arrive between steps, queue for rows and pages (max_batch 3), stop on EOS / stop
tokens / MaxTokens, or are cancelled.  Afterwards every page is back on the free stack.
"""
import asyncio

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

CFG = dict(vocab=3000, dim=512, layers=3, heads=8, kv_heads=2, ffn=1024, seed=51)


@pytest.fixture(scope="module")
def model():
    return O.make_model(**CFG)


def _engine(m, **kw):
    from zeroplatform_b200.engine import LlmEngine
    kw.setdefault("total_pages", 96)
    kw.setdefault("max_batch", 3)
    kw.setdefault("max_pages_per_seq", 16)
    kw.setdefault("max_prefill_tokens", 256)
    return LlmEngine(m, **kw)


def _oracle_greedy(m, prompt, n, penalty=1.0):
    ref = O.Engine(m, kv_fp16=True, total_pages=96)
    toks, _ = ref.generate_greedy(1, prompt, n, penalty=penalty)
    ref.close()
    return [int(t) for t in toks]


def _prompts(n, lens, seed=0):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, CFG["vocab"], k).astype(np.int32) for k in lens][:n]


def _drain(e, events_by_id, open_ids):
    from zeroplatform_b200._lib import SERVE_STOP_TOKEN
    while open_ids:
        for sid, tok, fin, reason in e.serve_step():
            if tok >= 0 and reason != SERVE_STOP_TOKEN:
                events_by_id.setdefault(sid, []).append(tok)
            if fin:
                open_ids.discard(sid)


def test_greedy_requests_with_staggered_arrivals_match_oracle(model):
    e = _engine(model)
    total = e.free_pages()
    lens = [5, 70, 17, 100, 40, 66]
    news = [12, 20, 30, 9, 25, 16]
    pens = [1.0, 1.1, 1.0, 1.1, 1.0, 1.05]
    prompts = _prompts(6, lens, seed=1)
    got, open_ids = {}, set()
    for i in range(3):  # three now, three more after some steps
        e.submit(i, prompts[i], news[i], temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=pens[i])
        open_ids.add(i)
    for _ in range(4):
        for sid, tok, fin, reason in e.serve_step():
            got.setdefault(sid, []).append(tok)
            if fin:
                open_ids.discard(sid)
    for i in range(3, 6):
        e.submit(i, prompts[i], news[i], temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=pens[i])
        open_ids.add(i)
    assert e.serve_counts()[1] == 3  # all three queue: the rows are taken
    _drain(e, got, open_ids)
    for i in range(6):
        assert got[i] == _oracle_greedy(model, prompts[i], news[i], pens[i]), i
    assert e.serve_counts() == (0, 0) and e.free_pages() == total
    e.close()


def test_sampled_requests_match_oracle_step_by_step(model):
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    e = _engine(model)
    prompts = _prompts(4, [30, 80, 12, 50], seed=2)
    cfgs = [(0.8, 0.9, 0.0, 40, 1.1), (1.2, 0.95, 0.05, 0, 1.0), (0.5, 0.8, 0.0, 5, 1.3), (1.0, 1.0, 0.02, 100, 1.0)]
    seeds = [11, 12, 13, 14]
    n_new = 24
    for i in range(4):
        t, p, mp, k, pen = cfgs[i]
        e.submit(i, prompts[i], n_new, temperature=t, top_p=p, min_p=mp, top_k=k, repetition_penalty=pen,
                 seed=seeds[i])
    got = {}
    _drain(e, got, set(range(4)))
    checked = 0
    for i in range(4):
        t, p, mp, k, pen = cfgs[i]
        toks = got[i]
        assert len(toks) == n_new
        ref = O.Engine(model, kv_fp16=True, total_pages=96)
        logits = ref.prefill(1, prompts[i], 0)
        past = [int(x) for x in prompts[i]]
        for j, tok in enumerate(toks):
            u = L.zcu_sample_uniform(seeds[i], j)
            want, _, wp, _ = O.sample(logits, past, t, p, mp, k, pen, u)
            if np.min(np.abs(np.cumsum(wp.astype(np.float64)) - u)) > 2e-3:
                assert tok == want, (i, j, tok, want)
                checked += 1
            past.append(tok)
            logits = ref.forward_token(1, tok, len(prompts[i]) + j)
        ref.close()
    assert checked >= 2 * n_new
    e.close()


def test_stop_tokens_max_tokens_and_cancellation(model):
    from zeroplatform_b200._lib import SERVE_CANCELLED, SERVE_MAX_TOKENS, SERVE_STOP_TOKEN
    e = _engine(model, max_batch=2)
    total = e.free_pages()
    prompts = _prompts(5, [20, 33, 9, 64, 15], seed=3)
    want0 = _oracle_greedy(model, prompts[0], 20)
    stop = want0[6]
    cut = want0.index(stop)
    e.submit(0, prompts[0], 20, temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=1.0, stop_tokens=[stop])
    e.submit(1, prompts[1], 7, temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=1.0)
    e.submit(2, prompts[2], 50, temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=1.0)  # queued
    e.submit(3, prompts[3], 0, temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=1.0)   # nothing sampled
    e.submit(4, prompts[4], 40, temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=1.0)
    e.cancel(4)                                        # cancelled while queued
    evs = []
    while e.serve_counts() != (0, 0) or not evs:
        step = e.serve_step()
        evs += step
        if any(s == 2 for s, _, _, _ in step) and not any(s == 2 and f for s, _, f, _ in evs):
            e.cancel(2)                                # cancelled while running
    fin = {s: (t, r) for s, t, f, r in evs if f}
    toks = {}
    for s, t, f, r in evs:
        if t >= 0 and r != SERVE_STOP_TOKEN:
            toks.setdefault(s, []).append(t)
    assert fin[0] == (stop, SERVE_STOP_TOKEN) and toks[0] == want0[:cut]
    assert fin[1][1] == SERVE_MAX_TOKENS and toks[1] == _oracle_greedy(model, prompts[1], 7)
    assert fin[2] == (-1, SERVE_CANCELLED) and 1 <= len(toks[2]) < 50
    assert fin[3] == (-1, SERVE_MAX_TOKENS) and 3 not in toks
    assert fin[4] == (-1, SERVE_CANCELLED) and 4 not in toks
    assert e.free_pages() == total
    e.close()


def test_async_streams_share_steps(model):
    """serving.ContinuousBatcher: four concurrent GenerateStreamAsync-style streams give the synchronous run's
    tokens; a stream the caller abandons early is cancelled and its pages come back."""
    from zeroplatform_b200.serving import ContinuousBatcher, SamplingConfig
    e = _engine(model)
    total = e.free_pages()
    prompts = _prompts(4, [10, 70, 25, 40], seed=4)
    greedy = SamplingConfig.greedy()
    greedy.max_tokens = 16
    cfgs = [greedy, SamplingConfig(max_tokens=18), SamplingConfig(temperature=1.0, top_k=0, max_tokens=10),
            SamplingConfig(repetition_penalty=1.0, max_tokens=14)]
    b = ContinuousBatcher(e)
    want = b.run([(p, c, 7 + i) for i, (p, c) in enumerate(zip(prompts, cfgs))])

    async def main():
        b2 = ContinuousBatcher(e, first_seq_id=1 << 24)
        outs = await asyncio.gather(*[b2.complete_async(p, c, 7 + i) for i, (p, c) in enumerate(zip(prompts, cfgs))])
        got = []
        stream = b2.generate_stream_async(prompts[1], SamplingConfig(max_tokens=40), 3)
        async for t in stream:
            got.append(t)
            if len(got) == 5:
                break
        await stream.aclose()
        while b2._driver is not None:
            await asyncio.sleep(0)
        return outs, got

    outs, partial = asyncio.run(main())
    assert [list(o) for o in outs] == want
    assert len(partial) == 5
    assert e.serve_counts() == (0, 0) and e.free_pages() == total
    e.close()


def test_submit_refusals(model):
    from zeroplatform_b200._lib import ZcError
    e = _engine(model)
    p = _prompts(1, [10])[0]
    e.submit(1, p, 5)
    with pytest.raises(ZcError):
        e.submit(1, p, 5)                  # the id is queued
    with pytest.raises(ZcError):
        e.submit(2, p, 16 * 16)            # beyond max_pages_per_seq * page_size
    with pytest.raises(ZcError):
        e.submit(3, np.zeros(300, np.int32), 4)  # beyond max_prefill_tokens
    with pytest.raises(ZcError):
        e.cancel(99)
    e.cancel(1)
    assert e.serve_step() == [(1, -1, 1, 3)]
    e.close()
