"""Device sampler (zcu_sample, zcu_engine_generate_sampled) vs the oracle's LlmSampler.Sample restatement.

The deterministic parts are compared with the random draw supplied to both sides: the kept candidates (ids in
order, after Top-K, Min-P and Top-P) exactly, their renormalised probabilities within 1e-5 max-rel (the device sums
the softmax as a tree, the reference left to right), and the sampled token exactly for every draw that does not fall
within 1e-5 of a boundary of the oracle's cumulative distribution.  .NET's System.Random draws cannot be replayed,
so generation is checked step by step against the oracle fed the device's own tokens and the same draws.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
CAP = 4096


def _lib():
    from zeroplatform_b200 import _lib
    return _lib.lib()


def _cfg(temperature, top_p, min_p, top_k, penalty):
    from zeroplatform_b200._lib import SamplingConfig
    return SamplingConfig(temperature, top_p, min_p, top_k, penalty)


def _device(logits, pasts, cfg, us):
    """zcu_sample on rows of logits; returns (tokens, [candidate ids], [candidate probabilities], logits after)."""
    L = _lib()
    rows, vocab = logits.shape
    lg = torch.from_numpy(logits.astype(np.float32)).cuda()
    pcap = max(1, max(len(p) for p in pasts))
    past = np.zeros((rows, pcap), np.int32)
    plen = np.zeros(rows, np.int32)
    for r, p in enumerate(pasts):
        past[r, :len(p)] = p
        plen[r] = len(p)
    past_d, plen_d = torch.from_numpy(past).cuda(), torch.from_numpy(plen).cuda()
    u = torch.tensor(us, dtype=torch.float32).cuda()
    out = torch.zeros(rows, dtype=torch.int32).cuda()
    ci = torch.zeros((rows, CAP), dtype=torch.int32).cuda()
    cp = torch.zeros((rows, CAP), dtype=torch.float32).cuda()
    nc = torch.zeros(rows, dtype=torch.int32).cuda()
    rc = L.zcu_sample(lg.data_ptr(), rows, vocab, past_d.data_ptr(), plen_d.data_ptr(), pcap, ctypes.byref(cfg),
                      u.data_ptr(), out.data_ptr(), ci.data_ptr(), cp.data_ptr(), nc.data_ptr(), CAP,
                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.zc_cuda_last_error()
    torch.cuda.synchronize()
    n = nc.cpu().numpy()
    ids = [ci[r, :max(n[r], 0)].cpu().numpy() for r in range(rows)]
    ps = [cp[r, :max(n[r], 0)].cpu().numpy() for r in range(rows)]
    return out.cpu().numpy(), ids, ps, lg.cpu().numpy()


def test_reference_known_answers_on_the_device():
    """LlmSamplerTests.cs:9-61 through the device sampler (see the oracle's golden test for each)."""
    g = _cfg(0.0, 1.0, 0.0, 1, 1.0)
    assert _device(np.array([[1.2, 5.8, 0.4, 3.1]]), [[]], g, [0.5])[0][0] == 1
    assert _device(np.array([[2.0, 2.1]]), [[1]], _cfg(0.0, 0.9, 0.0, 40, 2.0), [0.5])[0][0] == 0
    assert _device(np.array([[2.0, -np.inf, 4.0]]), [[]], g, [0.5])[0][0] == 2
    for u in (0.0, 0.3, 0.999999):
        tok, ids, ps, _ = _device(np.array([[10.0, 5.0, 0.1]]), [[]], _cfg(1.0, 1.0, 0.1, 40, 1.1), [u])
        assert tok[0] == 0 and list(ids[0]) == [0] and ps[0][0] == 1.0


# (temperature, top_p, min_p, top_k, penalty, logit scale): Top-K 0 keeps every candidate above 1e-6, so those rows
# use peaked logits (about 1,000-2,000 candidates; a flat row is the refusal test below)
CONFIGS = [(0.7, 0.9, 0.0, 40, 1.1, 2.5), (1.3, 0.95, 0.02, 0, 1.0, 6.0), (0.5, 0.8, 0.0, 5, 1.3, 2.5),
           (1.0, 1.0, 0.05, 100, 1.05, 2.5), (2.0, 0.5, 0.0, 0, 1.0, 10.0), (0.9, 0.99, 0.0, 1000, 1.2, 2.5)]


@pytest.mark.parametrize("temperature,top_p,min_p,top_k,penalty,scale", CONFIGS)
def test_sampler_matches_oracle(temperature, top_p, min_p, top_k, penalty, scale):
    rng = np.random.default_rng(int(temperature * 100 + top_k))
    rows, vocab = 4, 32000
    logits = (rng.standard_normal((rows, vocab)) * scale).astype(np.float32)
    pasts = [rng.integers(0, vocab, n).astype(np.int32) for n in (0, 7, 40, 200)]
    us = [0.05, 0.37, 0.71, 0.993]
    cfg = _cfg(temperature, top_p, min_p, top_k, penalty)
    tok, ids, ps, after = _device(logits, pasts, cfg, us)
    for r in range(rows):
        want, wid, wp, wlg = O.sample(logits[r], pasts[r], temperature, top_p, min_p, top_k, penalty, us[r], cap=CAP)
        assert np.array_equal(ids[r], wid), (r, len(ids[r]), len(wid))
        assert np.max(np.abs(ps[r] - wp)) <= 1e-5 * max(1.0, float(np.max(wp)))
        cdf = np.cumsum(wp.astype(np.float64))
        if np.min(np.abs(cdf - us[r])) > 1e-5:
            assert tok[r] == want
        # the probabilities left in place: the reference's left-to-right float sum over 32,000 terms drifts by about
        # sqrt(V) * 2^-24 relative, the tree sum does not (the renormalised candidates above cancel that factor)
        assert np.max(np.abs(after[r] - wlg)) <= 1e-4 * max(float(np.max(np.abs(wlg))), 1e-30)


def test_ties_keep_the_lower_token_first_and_greedy_edges():
    logits = np.zeros((1, 5000), np.float32)
    logits[0, [17, 3, 4000, 250]] = 4.0  # four equal maxima
    tok, ids, ps, _ = _device(logits, [[]], _cfg(1.0, 1.0, 0.0, 6, 1.0), [0.999])
    w, wid, wp, _ = O.sample(logits[0], [], 1.0, 1.0, 0.0, 6, 1.0, 0.999)
    assert list(ids[0]) == list(wid) == [3, 17, 250, 4000, 0, 1] and tok[0] == w
    # greedy: a NaN at index 0 keeps 0 (every comparison against it is false); all -inf gives 0; ties: first index
    g = _cfg(0.0, 1.0, 0.0, 1, 1.0)
    assert _device(np.array([[np.nan, 5.0, 7.0]]), [[]], g, [0.5])[0][0] == 0
    assert _device(np.array([[1.0, np.nan, 7.0]]), [[]], g, [0.5])[0][0] == 2
    assert _device(np.full((1, 9), -np.inf, np.float32), [[]], g, [0.5])[0][0] == 0
    assert _device(np.array([[1.0, 7.0, 7.0]]), [[]], g, [0.5])[0][0] == 1


def test_top_k_zero_over_a_flat_distribution_is_refused_per_row():
    """More than 4096 candidates after Top-K cannot be sorted in one row's shared memory: the row's token is -1."""
    logits = np.zeros((2, 20000), np.float32)
    logits[1, :10] = 30.0  # the second row has 10 candidates
    tok, ids, _, _ = _device(logits, [[], []], _cfg(1.0, 0.9, 0.0, 0, 1.0), [0.5, 0.5])
    want, wid, _, _ = O.sample(logits[1], [], 1.0, 0.9, 0.0, 0, 1.0, 0.5)
    assert tok[0] == -1 and tok[1] == want and list(ids[1]) == list(wid)  # Top-P 0.9 keeps 9 of the 10


def test_sampled_generation_matches_oracle_step_by_step():
    """zcu_engine_generate_sampled (T 0.8, Top-P 0.9, Top-K 40, penalty 1.1): each device token is the oracle's for
    the same history and the same draw, except draws within 2e-3 of a boundary of the oracle's distribution (the
    device logits differ from the oracle's by up to 1e-3)."""
    from zeroplatform_b200.engine import LlmEngine
    L = _lib()
    m = O.make_model(vocab=2048, dim=256, layers=3, heads=4, kv_heads=4, ffn=512, seed=41)
    prompt = np.random.default_rng(3).integers(0, 2048, 30).astype(np.int32)
    seed, n = 1234567, 40
    e = LlmEngine(m)
    toks, _, _ = e.generate_sampled(1, prompt, n, temperature=0.8, top_p=0.9, top_k=40, repetition_penalty=1.1,
                                    seed=seed)
    e.close()
    assert len(toks) == n
    ref = O.Engine(m, kv_fp16=True)
    logits = ref.prefill(1, prompt, 0)
    past = list(int(t) for t in prompt)
    checked = 0
    for i, t in enumerate(toks):
        u = L.zcu_sample_uniform(seed, i)
        want, _, wp, _ = O.sample(logits, past, 0.8, 0.9, 0.0, 40, 1.1, u)
        if np.min(np.abs(np.cumsum(wp.astype(np.float64)) - u)) > 2e-3:
            assert int(t) == want, (i, int(t), want)
            checked += 1
        past.append(int(t))
        logits = ref.forward_token(1, int(t), len(prompt) + i)
    ref.close()
    assert checked >= n // 2


def test_host_mirror_samples_like_the_entry_point():
    """ops.LlmSampler.sample (the host-facing mirror of LlmSampler.Sample) on the same rows as the oracle."""
    from zeroplatform_b200.ops import LlmSampler
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal((3, 1000)) * 3).astype(np.float32)
    past = [[1, 2, 3], [], [999, 999]]
    us = [0.2, 0.6, 0.9]
    out = LlmSampler.sample(torch.from_numpy(logits.copy()).cuda(), past, u=us).cpu().numpy()
    for r in range(3):
        want, _, wp, _ = O.sample(logits[r], past[r], u=us[r])
        if np.min(np.abs(np.cumsum(wp.astype(np.float64)) - us[r])) > 1e-5:
            assert out[r] == want
