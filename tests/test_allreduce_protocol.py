"""The tensor-parallel all-reduce's epoch-word protocol (csrc/allreduce_p2p.cu), modelled on the CPU.

Each rank owns a receive area of two buffers x W slots.  All-reduce e: every rank stores its term into slot[me] of
buffer e % 2 of every rank as words (value, e) -- one store per element, in any order -- then polls its own
buffer until every rank's word for each element carries e, sums the slots in rank order, and advances its
epoch.  The model runs W ranks as generators under random interleavings, at element granularity, with a
different length n per call, and checks that every reduce returns exactly the sum of the terms of its own call:
no word of an older call (still in the buffer beyond a shorter call's n) and no word of a later call (the buffer
is reused two calls later) is ever taken.
"""
import random

import pytest


def _rank(me, W, areas, calls, terms, out):
    """Rank `me` running len(calls) all-reduces; yields after every store and every poll."""
    for e, n in enumerate(calls, start=1):
        buf = e % 2
        # push: stores of (value, epoch) in a random order, one element at a time
        order = [(r, i) for r in range(W) for i in range(n)]
        random.shuffle(order)
        for r, i in order:
            areas[r][buf][me][i] = (terms[e][me][i], e)
            yield
        # reduce: poll each element until every rank's word carries e
        acc = []
        for i in range(n):
            while True:
                words = [areas[me][buf][q][i] for q in range(W)]
                if all(w[1] == e for w in words):
                    break
                yield
            acc.append(sum(w[0] for w in words))
        out[me].append(acc)
        yield


@pytest.mark.parametrize("W", [2, 3, 4, 8])
@pytest.mark.parametrize("seed", range(6))
def test_epoch_words_never_mix_calls(W, seed):
    random.seed(seed * 100 + W)
    cap = 6
    n_calls = 7
    calls = [random.randint(1, cap) for _ in range(n_calls)]  # n varies: stale words stay beyond a short call
    terms = {e: [[random.randint(-1000, 1000) for _ in range(cap)] for _ in range(W)]
             for e in range(1, n_calls + 1)}
    # epoch 0 = never pushed
    areas = [[[[(0, 0)] * cap for _ in range(W)] for _ in range(2)] for _ in range(W)]
    out = [[] for _ in range(W)]
    ranks = [_rank(me, W, areas, calls, terms, out) for me in range(W)]
    live = list(range(W))
    steps = 0
    while live:
        me = random.choice(live)  # an arbitrary interleaving of the ranks
        try:
            next(ranks[me])
        except StopIteration:
            live.remove(me)
        steps += 1
        assert steps < 2_000_000, "the ranks stopped making progress"
    for e, n in enumerate(calls, start=1):
        want = [sum(terms[e][q][i] for q in range(W)) for i in range(n)]
        for me in range(W):
            assert out[me][e - 1] == want, (e, me)
