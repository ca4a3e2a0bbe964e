"""Pins the CPU oracle to the reference's own known-answer tests (no GPU needed).

Each test restates one reference xUnit test (cited) against the oracle, plus an independent numpy
restatement of the block quantizers so that the C++ oracle is checked by a second implementation.
"""
import numpy as np
import pytest

import oracle as O
from tests.conftest import rel_err


# ---- GEMV goldens: ZeroTensor/tests/ZeroTensor.Tests/NeuralOperatorsTests.cs:585-628 ------------------
def q8_golden_block():
    blk = np.zeros(34, np.uint8)
    blk[0], blk[1] = 0x00, 0x40  # fp16 2.0
    blk[2:] = 3
    return blk


def q4_golden_block():
    blk = np.zeros(18, np.uint8)
    blk[0], blk[1] = 0x00, 0x3C  # fp16 1.0
    blk[2:] = 0x9A               # low nibble 10 -> +2, high nibble 9 -> +1
    return blk


@pytest.mark.parametrize("path", [0, 1])
def test_gemv_q8_0_golden_192(path):
    x = np.ones(32, np.float32)
    assert abs(O.dot_q8_0(x, q8_golden_block(), path) - 192.0) < 1e-4
    assert abs(O.matvec(8, q8_golden_block(), x, 1, 32)[0] - 192.0) < 1e-4


@pytest.mark.parametrize("path", [0, 1])
def test_gemv_q4_0_golden_48(path):
    x = np.ones(32, np.float32)
    assert abs(O.dot_q4_0(x, q4_golden_block(), path) - 48.0) < 1e-4
    assert abs(O.matvec(4, q4_golden_block(), x, 1, 32)[0] - 48.0) < 1e-4


# ---- ZeroLlm/tests/ZeroLlm.Tests/QuantizedKernelsTests.cs ----------------------------------------------
def test_half_roundtrip_kat():  # :10-19
    for v in [0.0, 1.0, -1.0, 0.5, 2.5, -10.25, 100.0]:
        h = O.lib().orc_f32_to_f16(v)
        assert round(O.lib().orc_f16_to_f32(h), 2) == round(v, 2)


def test_half_matches_ieee_rne():
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(200_000) * 10.0 ** rng.integers(-9, 6, 200_000)).astype(np.float32)
    x = np.concatenate([x, np.float32([65504, 65519.99, 65520, -65520, 6.1e-5, 5.96e-8, 2.98e-8, 0.0, -0.0])])
    with np.errstate(over="ignore"):
        assert np.array_equal(O.f32_to_f16(x), x.astype(np.float16).view(np.uint16))


def test_q8_quantize_error_kat():  # :22-39
    src = np.array([(i - 16) * 1.5 for i in range(32)], np.float32)
    rec = O.dequantize_q8_0(O.quantize_q8_0(src[None]), 32)[0]
    assert np.all(np.abs(src - rec) <= 0.2)


def test_q4_quantize_error_kat():  # :41-59
    src = np.array([(i - 16) * 0.5 for i in range(32)], np.float32)
    rec = O.dequantize_q4_0(O.quantize_q4_0(src[None]), 32)[0]
    assert np.all(np.abs(src - rec) <= 0.75)


@pytest.mark.parametrize("path", [0, 1])
def test_dot_q8_matches_dequantized_kat(path):  # :62-90
    i = np.arange(64)
    x = ((i % 5) * np.float32(0.2)).astype(np.float32)
    w = (((i % 7) - 3) * np.float32(0.5)).astype(np.float32)
    blocks = O.quantize_q8_0(w[None])[0]
    deq = O.dequantize_q8_0(blocks, 64)[0]
    expected = np.float32(0)
    for a, b in zip(x, deq):
        expected = np.float32(expected + np.float32(a * b))
    assert round(O.dot_q8_0(x, blocks, path), 3) == round(float(expected), 3)


@pytest.mark.parametrize("path", [0, 1])
def test_dot_q4_matches_dequantized_kat(path):  # :92-121
    i = np.arange(64)
    x = ((i % 3) * np.float32(0.4)).astype(np.float32)
    w = (((i % 5) - 2) * np.float32(0.8)).astype(np.float32)
    blocks = O.quantize_q4_0(w[None])[0]
    deq = O.dequantize_q4_0(blocks, 64)[0]
    expected = np.float32(0)
    for a, b in zip(x, deq):
        expected = np.float32(expected + np.float32(a * b))
    assert round(O.dot_q4_0(x, blocks, path), 3) == round(float(expected), 3)


def test_matvec_q8_row_sums_kat():  # :123-149
    rows = np.stack([np.full(32, (r + 1) * np.float32(0.1), np.float32) for r in range(3)])
    y = O.matvec(8, O.quantize_q8_0(rows), np.ones(32, np.float32), 3, 32)
    assert 3.1 <= y[0] <= 3.3 and 6.2 <= y[1] <= 6.6 and 9.4 <= y[2] <= 9.8


def test_multiblock_avx2_kat():  # :151-190
    i = np.arange(8 * 32)
    x = (((i % 13) - 6) * np.float32(0.15)).astype(np.float32)
    w = (((i % 11) - 5) * np.float32(0.35)).astype(np.float32)
    q8 = O.quantize_q8_0(w[None])[0]
    q4 = O.quantize_q4_0(w[None])[0]
    e8 = float(np.dot(x.astype(np.float64), O.dequantize_q8_0(q8, 256)[0].astype(np.float64)))
    e4 = float(np.dot(x.astype(np.float64), O.dequantize_q4_0(q4, 256)[0].astype(np.float64)))
    assert round(O.dot_q8_0(x, q8, 0), 2) == round(e8, 2)
    assert round(O.dot_q4_0(x, q4, 0), 2) == round(e4, 2)


# ---- independent numpy restatement of the quantizers (BlockQ8_0.cs:43-71, BlockQ4_0.cs:120-150) --------
def np_quantize_q8_0(w):
    b = w.reshape(-1, 32).astype(np.float32)
    amax = np.max(np.abs(b), axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d > np.float32(1e-15), np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.clip(np.rint((b * idv[:, None]).astype(np.float32).astype(np.float64)), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def np_quantize_q4_0(w):
    b = w.reshape(-1, 32).astype(np.float32)
    amax = np.max(np.abs(b), axis=1)
    d = (amax / np.float32(8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.clip(np.rint((b * idv[:, None]).astype(np.float32).astype(np.float64)) + 8, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 18), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = (q[:, :16] & 0x0F) | ((q[:, 16:] & 0x0F) << 4)
    return out.reshape(-1)


@pytest.mark.parametrize("scale", [0.02, 1.0, 1e-6, 300.0])
def test_quantizers_match_numpy_restatement(scale):
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((64, 256)) * scale).astype(np.float32)
    w[0, :32] = 0.0          # all-zero block
    w[1, 5] = 7 * scale      # isolated outlier
    assert np.array_equal(O.quantize_q8_0(w).reshape(-1), np_quantize_q8_0(w))
    assert np.array_equal(O.quantize_q4_0(w).reshape(-1), np_quantize_q4_0(w))


def test_matvec_q8_matches_float64_dequantized():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((300, 512)) * 0.02).astype(np.float32)
    x = rng.standard_normal(512).astype(np.float32)
    blocks = O.quantize_q8_0(w)
    ref = O.dequantize_q8_0(blocks, 512).astype(np.float64) @ x.astype(np.float64)
    assert rel_err(O.matvec(8, blocks, x, 300, 512), ref) < 1e-5
    y0 = rng.standard_normal(300).astype(np.float32)
    y = O.matvec(8, blocks, x, 300, 512, y=y0.copy())
    assert rel_err(y, ref + y0) < 1e-5


# ---- int8 x int8 -> int32: ZeroTensor/tests/ZeroTensor.Tests/TensorBFloat16AndInt4Tests.cs:108-145 ------
def test_gemm_i8_exact_kat():
    m, k, n = 5, 19, 27
    a = np.array([[((i * 7 + p * 3) % 21) - 10 for p in range(k)] for i in range(m)], np.int8)
    b = np.array([[((p * 5 + j * 11) % 31) - 15 for j in range(n)] for p in range(k)], np.int8)
    c = O.gemm_i8(a, b)
    assert np.array_equal(c, a.astype(np.int32) @ b.astype(np.int32))
    assert O.dot_i8(a[0], b[:, 0].copy()) == int(c[0, 0])


# ---- PagedKvCache: ZeroLlm/tests/ZeroLlm.Tests/PagedKvCacheTests.cs:10-51 ----------------------------
def _tiny_model(layers=2, vocab=64, seed=0):
    # kv_heads 2 x head_dim 8 as in the reference test; dim 32 (4 query heads) keeps Q8_0 rows whole blocks
    return O.make_model(vocab=vocab, dim=32, layers=layers, heads=4, kv_heads=2, ffn=64, seed=seed)


def test_paged_kv_cache_accounting_kat():
    m = _tiny_model()
    e = O.Engine(m, total_pages=16, page_size=4)
    assert e.free_blocks() == 16
    key = np.zeros(16, np.float32)
    val = np.zeros(16, np.float32)
    for t in range(10):
        key[0], val[0] = t * 1.5, t * 2.5
        e.append_token(101, 0, key, val)
        e.append_token(101, 1, key, val)
    assert e.seq_len(101) == 10
    assert e.free_blocks() == 16 - 3
    assert e.get_kv(101, 0, 7)[0] == np.float32(7 * 1.5)
    assert e.get_kv(101, 1, 7, value=True)[0] == np.float32(7 * 2.5)
    # Stack<int> pops the most recently pushed page first: 15, 14, 13
    assert list(e.page_table(101)) == [15, 14, 13]
    e.free_sequence(101)
    assert e.seq_len(101) == 0 and e.free_blocks() == 16
    e.close()


# ---- PagedAttention: NeuralOperatorsTests.cs:950-971 (setup), TensorOps.Neural.cs:2418-2473 ----------
def _float64_paged_reference(q, k, v, bt, ctx, hkv):
    hq, hd = q.shape
    bs = k.shape[1]
    g = hq // hkv
    out = np.zeros((hq, hd))
    for h in range(hq):
        rows_k = np.stack([k[bt[t // bs], t % bs, h // g] for t in range(ctx)]).astype(np.float64)
        rows_v = np.stack([v[bt[t // bs], t % bs, h // g] for t in range(ctx)]).astype(np.float64)
        s = rows_k @ q[h].astype(np.float64) / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ rows_v
    return out


def test_paged_attention_setup_kat():
    rng = np.random.default_rng(42)
    hq, hkv, hd, bs, ctx = 4, 2, 8, 4, 10
    q = rng.standard_normal((hq, hd)).astype(np.float32)
    k = rng.standard_normal((3, bs, hkv, hd)).astype(np.float32)
    v = rng.standard_normal((3, bs, hkv, hd)).astype(np.float32)
    bt = np.array([2, 0, 1], np.int32)
    online = O.paged_attention(q, k, v, bt, ctx)
    ref = _float64_paged_reference(q, k, v, bt, ctx, hkv)
    assert np.max(np.abs(online - ref)) < 1e-5
    # GqaAttention's two-pass softmax over the same pages agrees with the online form (both within 1e-3,
    # the reference test's tolerance; in practice to ~1e-6).
    two_pass = O.gqa_attention(q.reshape(-1), k, v, bt, bs, ctx, hq, hkv, hd).reshape(hq, hd)
    assert np.max(np.abs(two_pass - online)) < 1e-5


# ---- LlmEngine: ZeroLlm/tests/ZeroLlm.Tests/LlmEngineTests.cs:92-135 ----------------------------------
def test_batched_prefill_equals_sequential_kat():
    m = O.make_model(vocab=128, dim=32, layers=2, heads=2, kv_heads=2, ffn=64, seed=777)
    e = O.Engine(m)
    prompt = np.array([5, 12, 23, 34, 45, 56], np.int32)
    batched = e.prefill(42, prompt, 0)
    assert e.seq_len(42) == len(prompt)
    assert np.all(np.isfinite(batched))
    seq = None
    for t in range(len(prompt)):
        seq = e.prefill(43, prompt[t:t + 1], t)
    assert np.all(np.round(seq, 4) == np.round(batched, 4)) or np.max(np.abs(seq - batched)) < 5e-5
    e.close()


def test_causal_quirk_first_token_non_final_layers_see_nothing():
    """At pos 0 every layer but the last attends to an empty context (PagedKvCache.cs:139-142)."""
    m = O.make_model(vocab=64, dim=32, layers=3, heads=2, kv_heads=2, ffn=64, seed=5)
    e = O.Engine(m)
    e.forward_token(1, 3, 0)
    assert e.seq_len(1) == 1
    e.close()


def test_sampler_reference_known_answers():
    """LlmSamplerTests (ZeroLlm/tests/ZeroLlm.Tests/LlmSamplerTests.cs:9-61): greedy picks the maximum (:10-17);
    a penalty of 2 on past token 1 turns {2.0, 2.1} into a win for token 0 (:20-31); a token masked to -inf loses
    (:34-46, the mask applied to the input); Min-P 0.1 keeps only token 0 of {10, 5, 0.1} whatever the draw
    (:49-61, SamplingConfig defaults otherwise: Top-K 40, penalty 1.1)."""
    greedy = dict(temperature=0.0, top_p=1.0, top_k=1, penalty=1.0)
    assert O.sample([1.2, 5.8, 0.4, 3.1], **greedy)[0] == 1
    assert O.sample([2.0, 2.1], past=[1], temperature=0.0, penalty=2.0)[0] == 0
    assert O.sample([2.0, -np.inf, 4.0], **greedy)[0] == 2
    for u in (0.0, 0.3, 0.999999):
        tok, ids, ps, _ = O.sample([10.0, 5.0, 0.1], temperature=1.0, top_p=1.0, min_p=0.1, u=u)
        assert tok == 0 and list(ids) == [0] and ps[0] == 1.0


def test_sampler_restatement_against_numpy():
    """The oracle's stochastic branch against an independent numpy restatement of LlmSampler.cs:75-171 (float32
    arithmetic in the reference's order): the same candidates, probabilities and token for a grid of draws."""
    rng = np.random.default_rng(3)
    for trial in range(6):
        V = 500
        logits = (rng.standard_normal(V) * 3).astype(np.float32)
        past = rng.integers(0, V, 20).astype(np.int32)
        T, top_p, min_p, top_k, pen = [(0.7, 0.9, 0.0, 40, 1.1), (1.3, 0.95, 0.02, 0, 1.0), (0.5, 0.8, 0.0, 5, 1.3),
                                       (1.0, 1.0, 0.05, 100, 1.05), (2.0, 0.5, 0.0, 0, 1.0),
                                       (0.9, 0.99, 0.01, 300, 1.2)][trial]
        lg = logits.copy()
        for t in past:  # penalty, occurrence by occurrence
            lg[t] = lg[t] / np.float32(pen) if lg[t] > 0 else lg[t] * np.float32(pen)
        lg = lg * (np.float32(1.0) / np.float32(T))
        m = lg.max()
        e = np.array([np.float32(np.exp(np.float64(v - m))) for v in lg], np.float32)
        s = np.float32(0)
        for v in e:
            s = np.float32(s + v)
        p = e * (np.float32(1.0) / s)
        cand = sorted([(i, p[i]) for i in range(V) if p[i] > np.float32(1e-6)], key=lambda c: (-c[1], c[0]))
        if top_k > 0:
            cand = cand[:top_k]
        if min_p > 0:
            thr = np.float32(cand[0][1] * np.float32(min_p))
            cand = [cand[0]] + [c for c in cand[1:] if not c[1] < thr]
        cum, cut = np.float32(0), len(cand)
        for i, (_, v) in enumerate(cand):
            cum = np.float32(cum + v)
            if cum >= np.float32(top_p):
                cut = i + 1
                break
        cand = cand[:cut]
        tot = np.float32(0)
        for _, v in cand:
            tot = np.float32(tot + v)
        inv = np.float32(1.0) / tot
        for u in np.linspace(0.0, 1.0, 23, dtype=np.float32):
            tok, ids, ps, _ = O.sample(logits, past, T, top_p, min_p, top_k, pen, float(u))
            assert list(ids) == [c[0] for c in cand]
            assert np.array_equal(ps, np.array([np.float32(v * inv) for _, v in cand], np.float32))
            run, want = np.float32(0), cand[0][0]
            for i, v in cand:
                run = np.float32(run + np.float32(v * inv))
                if u <= run:
                    want = i
                    break
            assert tok == want


def test_flash_attention_restatement_on_the_reference_inputs():
    """FlashAttentionCpu_MatchesStandardAttention and _GroupedQueryAttention_MatchesExpanded
    (ZeroTensor/tests/ZeroTensor.Tests/NeuralOperatorsTests.cs:390-427, 660-723): the restatement agrees with plain
    softmax attention within the tests' 1e-4, for a masked form too (mask batch broadcast b % mask batches), and a
    row whose keys are all masked gives zeros."""
    i = np.arange(8, dtype=np.float32)[:, None]
    d = np.arange(16, dtype=np.float32)[None, :]
    q = np.stack([(i + d) * np.float32(0.1), (i - d) * np.float32(0.1)])[None]
    k = np.stack([(i - d) * np.float32(0.05), (i + d) * np.float32(0.05)])[None]
    v = np.stack([(i * 2 + d) * np.float32(0.1), (d - i) * np.float32(0.1)])[None]

    def sdpa(q, k, v, mask=None):
        if k.shape[1] != q.shape[1]:
            g = q.shape[1] // k.shape[1]
            k, v = np.repeat(k, g, axis=1), np.repeat(v, g, axis=1)
        s = q.astype(np.float64) @ np.swapaxes(k.astype(np.float64), -1, -2) / np.sqrt(q.shape[-1])
        if mask is not None:
            s = s + mask
        m = s.max(-1, keepdims=True)
        p = np.where(np.isneginf(s), 0.0, np.exp(s - np.where(np.isneginf(m), 0.0, m)))
        den = p.sum(-1, keepdims=True)
        return np.where(den > 0, p / np.where(den > 0, den, 1.0), 0.0) @ v.astype(np.float64)

    assert np.max(np.abs(O.flash_attention(q, k, v) - sdpa(q, k, v))) < 1e-4
    h = np.arange(4, dtype=np.float64)[:, None, None]
    s = np.arange(8, dtype=np.float64)[None, :, None]
    dd = np.arange(16, dtype=np.float64)[None, None, :]
    qg = np.sin(h * 10 + s + dd * 0.1).astype(np.float32)[None]
    hk = np.arange(2, dtype=np.float64)[:, None, None]
    kg = np.cos(hk * 5 + s * 0.5 + dd * 0.2).astype(np.float32)[None]
    vg = np.sin(hk * 3 + s * 0.2 + dd * 0.3).astype(np.float32)[None]
    assert np.max(np.abs(O.flash_attention(qg, kg, vg) - sdpa(qg, kg, vg))) < 1e-4
    causal = np.triu(np.full((8, 8), -np.inf, np.float32), 1)
    causal[0, 0] = -np.inf                                     # row 0 attends to nothing
    got = O.flash_attention(qg, kg, vg, mask=causal)
    assert np.all(got[:, :, 0] == 0.0)
    assert np.max(np.abs(got - sdpa(qg, kg, vg, causal))) < 1e-4
