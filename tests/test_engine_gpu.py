"""Device decode engine (LlmEngine over a paged fp16 KV cache) vs the oracle engine.

The oracle runs with kv_fp16=True (it rounds every appended K/V to binary16, the device cache's storage
precision) so that the comparison isolates the kernels.  Tolerances: logits max-rel <= 1e-3 (the parity
bound; batched prefill runs on fp16 tensor cores), greedy tokens identical.
"""
import numpy as np
import pytest

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _engine(m, **kw):
    from zeroplatform_b200.engine import LlmEngine
    return LlmEngine(m, **kw)


def test_reference_batched_prefill_equals_sequential():
    """LlmEngineTests.PrefillPrompt_Batched_ProducesValidLogitsAndPopulatesKvCache (LlmEngineTests.cs:92-135)."""
    m = O.make_model(vocab=128, dim=32, layers=2, heads=2, kv_heads=2, ffn=64, seed=777)
    e = _engine(m)
    prompt = np.array([5, 12, 23, 34, 45, 56], np.int32)
    batched = e.prefill(42, prompt, 0)
    assert e.seq_len(42) == len(prompt)
    assert np.all(np.isfinite(batched))
    seq = None
    for t in range(len(prompt)):
        seq = e.prefill(43, prompt[t:t + 1], t)
    assert np.max(np.abs(seq - batched)) < 5e-5          # Assert.Equal(..., precision: 4)
    ref = O.Engine(m, kv_fp16=True)
    assert rel_err(batched, ref.prefill(42, prompt, 0)) <= TOL
    e.close()


def test_kv_cache_accounting_matches_reference_allocator():
    m = O.make_model(vocab=64, dim=32, layers=2, heads=4, kv_heads=2, ffn=64, seed=3)
    e = _engine(m, total_pages=16, page_size=4)
    ref = O.Engine(m, total_pages=16, page_size=4, kv_fp16=True)
    toks = np.arange(10, dtype=np.int32) + 3
    e.prefill(101, toks, 0)
    ref.prefill(101, toks, 0)
    assert e.seq_len(101) == ref.seq_len(101) == 10
    assert e.free_pages() == ref.free_blocks() == 13
    assert list(e.page_table(101)) == list(ref.page_table(101)) == [15, 14, 13]
    for layer in range(2):
        for t in (0, 7, 9):
            assert rel_err(e.get_kv(101, layer, t), ref.get_kv(101, layer, t)) <= TOL
            assert rel_err(e.get_kv(101, layer, t, value=True), ref.get_kv(101, layer, t, value=True)) <= TOL
    e.free_sequence(101)
    assert e.seq_len(101) == 0 and e.free_pages() == 16


@pytest.mark.parametrize("heads,kv_heads,dim,ffn", [(12, 12, 768, 2048), (8, 2, 512, 1024), (32, 32, 4096, 512)])
def test_prefill_and_decode_logits_match_oracle(heads, kv_heads, dim, ffn):
    m = O.make_model(vocab=4096, dim=dim, layers=3, heads=heads, kv_heads=kv_heads, ffn=ffn, seed=11)
    e = _engine(m)
    ref = O.Engine(m, kv_fp16=True)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, 4096, 37).astype(np.int32)
    assert rel_err(e.prefill(1, prompt, 0), ref.prefill(1, prompt, 0)) <= TOL
    pos = len(prompt)
    for tok in (5, 900, 4095, 17):          # ForwardToken with the per-layer causal rule
        assert rel_err(e.forward_token(1, tok, pos), ref.forward_token(1, tok, pos)) <= TOL
        pos += 1
    assert e.seq_len(1) == ref.seq_len(1) == pos


def test_first_token_single_prefill_matches_oracle():
    """T == 1 prefill is ForwardToken at pos 0: non-final layers see an empty context."""
    m = O.make_model(vocab=512, dim=256, layers=3, heads=4, kv_heads=4, ffn=512, seed=4)
    e = _engine(m)
    ref = O.Engine(m, kv_fp16=True)
    assert rel_err(e.prefill(7, [42], 0), ref.prefill(7, [42], 0)) <= TOL


def test_batched_decode_matches_per_sequence_decode():
    m = O.make_model(vocab=2048, dim=256, layers=2, heads=8, kv_heads=4, ffn=512, seed=9)
    e = _engine(m, max_batch=8)
    ref = O.Engine(m, kv_fp16=True)
    rng = np.random.default_rng(1)
    lens = [5, 16, 17, 33]
    for sid, n in enumerate(lens):
        p = rng.integers(0, 2048, n).astype(np.int32)
        e.prefill(sid, p, 0)
        ref.prefill(sid, p, 0)
    toks = rng.integers(0, 2048, len(lens)).astype(np.int32)
    out = e.decode(list(range(len(lens))), toks, lens)
    for sid, n in enumerate(lens):
        assert rel_err(out[sid], ref.forward_token(sid, int(toks[sid]), n)) <= TOL


@pytest.mark.parametrize("penalty", [1.0, 1.1])
def test_greedy_generation_matches_oracle_tokens(penalty):
    m = O.make_model(vocab=4096, dim=384, layers=4, heads=6, kv_heads=6, ffn=1024, seed=21)
    e = _engine(m)
    ref = O.Engine(m, kv_fp16=True)
    prompt = np.random.default_rng(2).integers(0, 4096, 40).astype(np.int32)
    toks, _, _ = e.generate_greedy(3, prompt, 24, repetition_penalty=penalty)
    ref_toks, _ = ref.generate_greedy(3, prompt, 24, penalty=penalty)
    agree = 0
    for a, b in zip(toks, ref_toks):
        if a != b:
            break
        agree += 1
    print(f"greedy agreement {agree}/{len(ref_toks)} (penalty {penalty})")
    assert agree == len(ref_toks)
