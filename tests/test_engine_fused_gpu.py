"""One-kernel generation step (decode_fused.cu) vs the oracle engine and vs the per-operator step.

zcu_engine_generate runs each token of a one-sequence, one-GPU generation as a single cooperative kernel when the
model's shapes fit it.  These tests check that the form actually ran (zcu_engine_step_kind) and that its greedy
tokens are the oracle's (LlmEngine.GenerateStreamAsync with greedy sampling, LlmSampler.cs:21-72) -- with and
without the repetition penalty, with grouped-query attention, head sizes 64 and 128, contexts spanning many pages,
a stop token, and the 12-layer d768 / 32000-token benchmark model -- and identical to the per-operator graph's.
The oracle rounds appended K/V to binary16 as the device cache stores them.
"""
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _engine(m, **kw):
    from zeroplatform_b200.engine import LlmEngine
    return LlmEngine(m, **kw)


def _fused_tokens(m, prompt, n_new, penalty=1.0, eos=-1, fused=True, **kw):
    old = os.environ.get("ZCU_FUSED_DECODE")
    if not fused:
        os.environ["ZCU_FUSED_DECODE"] = "0"
    try:
        e = _engine(m, **kw)
        toks, _, _ = e.generate_greedy(3, prompt, n_new, repetition_penalty=penalty, eos_token=eos)
        kind, why = e.step_kind()
        e.close()
    finally:
        if old is None:
            os.environ.pop("ZCU_FUSED_DECODE", None)
        else:
            os.environ["ZCU_FUSED_DECODE"] = old
    return list(int(t) for t in toks), kind, why


MODELS = {
    "d768_h12": dict(vocab=4096, dim=768, layers=3, heads=12, kv_heads=12, ffn=2048, seed=31),
    "d512_gqa4": dict(vocab=3000, dim=512, layers=4, heads=8, kv_heads=2, ffn=1024, seed=32),
    "d1024_hd128": dict(vocab=2048, dim=1024, layers=2, heads=8, kv_heads=4, ffn=2560, seed=33),
}


@pytest.mark.parametrize("name", sorted(MODELS))
@pytest.mark.parametrize("penalty", [1.0, 1.1])
def test_fused_generation_matches_oracle_tokens(name, penalty):
    cfg = MODELS[name]
    m = O.make_model(**cfg)
    prompt = np.random.default_rng(7).integers(0, cfg["vocab"], 45).astype(np.int32)
    toks, kind, why = _fused_tokens(m, prompt, 32, penalty=penalty)
    assert kind == 1, why
    ref = O.Engine(m, kv_fp16=True)
    want, _ = ref.generate_greedy(3, prompt, 32, penalty=penalty)
    ref.close()
    assert toks == want


def test_fused_and_per_operator_steps_agree_over_long_contexts():
    """300-token prompt (19 pages), 40 new tokens: the attention splits cover many pages; both step forms give the
    oracle's tokens."""
    cfg = MODELS["d512_gqa4"]
    m = O.make_model(**cfg)
    prompt = np.random.default_rng(8).integers(0, cfg["vocab"], 300).astype(np.int32)
    fused, kind, why = _fused_tokens(m, prompt, 40, total_pages=64)
    assert kind == 1, why
    plain, kind0, why0 = _fused_tokens(m, prompt, 40, fused=False, total_pages=64)
    assert kind0 == 0 and "ZCU_FUSED_DECODE" in why0
    ref = O.Engine(m, kv_fp16=True, total_pages=64)
    want, _ = ref.generate_greedy(3, prompt, 40)
    ref.close()
    assert fused == want and plain == want


def test_fused_generation_stops_at_the_stop_token():
    cfg = MODELS["d768_h12"]
    m = O.make_model(**cfg)
    prompt = np.random.default_rng(9).integers(0, cfg["vocab"], 20).astype(np.int32)
    ref = O.Engine(m, kv_fp16=True)
    want, _ = ref.generate_greedy(3, prompt, 12)
    ref.close()
    eos = want[5]
    stop = want.index(eos)  # the first occurrence ends generation; the stop token itself is not emitted
    toks, kind, _ = _fused_tokens(m, prompt, 12, eos=eos)
    assert kind == 1
    assert toks == want[:stop]


def test_fused_generation_at_the_benchmark_model():
    """12 layers, d_model 768, 12 heads x 64, SwiGLU 2048, vocabulary 32000 (the small-Llama decode workload):
    512-token prompt, 48 greedy tokens."""
    cfg = dict(vocab=32000, dim=768, layers=12, heads=12, kv_heads=12, ffn=2048, seed=11)
    m = O.make_model(**cfg)
    prompt = np.random.default_rng(5).integers(0, 32000, 512).astype(np.int32)
    toks, kind, why = _fused_tokens(m, prompt, 48, total_pages=64, max_pages_per_seq=64, max_prefill_tokens=512)
    assert kind == 1, why
    ref = O.Engine(m, kv_fp16=True, total_pages=64)
    want, _ = ref.generate_greedy(3, prompt, 48)
    ref.close()
    agree = next((i for i, (a, b) in enumerate(zip(toks, want)) if a != b), len(want))
    print(f"benchmark model: greedy agreement {agree}/{len(want)}")
    assert toks == want
