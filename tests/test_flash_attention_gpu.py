"""zc_flash_attention_f32 (the bridge's FlashAttention entry) and the engine's tiled prefill attention vs the oracle.

The bridge entry runs TensorOps.FlashAttentionCpu's contract (TensorOps.Neural.cs:983-1180) on the device: q
[batch][sq][d], k / v [kv batch][sk][d], grouped-query kv batch (b / hq) * hkv + (b % hq) / group.  Outputs are
compared with the oracle's restatement of FlashAttentionCpu, max abs difference <= 1e-4 (the reference's own bound in
NeuralOperatorsTests.cs:423,719; the device's exp2 online softmax and the oracle's double exp differ by about 1e-6).
A mask, dv != d or a head size outside 16/32/64/128 returns -1 (not handled) and leaves the output untouched.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _lib():
    from zeroplatform_b200 import _lib
    return _lib.lib()


def _vp(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _device(q, k, v, mask=None, scale=None, out=None):
    """Calls the bridge entry the way TensorOps.FlashAttentionCpu does; returns (status, out)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    sq, d = q.shape[-2:]
    sk, dv = k.shape[-2], v.shape[-1]
    hq = hkv = 1
    if q.ndim == 4 and k.ndim == 4:
        hq, hkv = q.shape[1], k.shape[1]
    group = hq // hkv
    batch = int(np.prod(q.shape[:-2]))
    if out is None:
        out = np.full(q.shape[:-1] + (dv,), 7.0, np.float32)
    sc = np.float32(1.0) / np.float32(np.sqrt(np.float64(d))) if scale is None else np.float32(scale)
    m = None if mask is None else np.ascontiguousarray(mask, np.float32)
    rc = _lib().zc_flash_attention_f32(batch, sq, sk, d, dv, float(sc), int(group > 1), hq, hkv, group, _vp(q),
                                        _vp(k), _vp(v), _vp(m), _vp(out))
    return rc, out


def _sdpa(q, k, v):
    """Plain softmax(q k^T / sqrt(d)) v in float64 (TensorOps.ScaledDotProductAttention), k / v expanded per group."""
    if q.ndim == 4 and k.shape[1] != q.shape[1]:
        g = q.shape[1] // k.shape[1]
        k, v = np.repeat(k, g, axis=1), np.repeat(v, g, axis=1)
    s = q.astype(np.float64) @ np.swapaxes(k.astype(np.float64), -1, -2) / np.sqrt(q.shape[-1])
    p = np.exp(s - s.max(-1, keepdims=True))
    return (p / p.sum(-1, keepdims=True)) @ v.astype(np.float64)


def test_reference_flash_matches_standard_attention_inputs():
    """FlashAttentionCpu_MatchesStandardAttention (NeuralOperatorsTests.cs:390-427): batch 1, 2 heads, 8 x 16."""
    i = np.arange(8, dtype=np.float32)[:, None]
    d = np.arange(16, dtype=np.float32)[None, :]
    q = np.stack([(i + d) * np.float32(0.1), (i - d) * np.float32(0.1)])[None]
    k = np.stack([(i - d) * np.float32(0.05), (i + d) * np.float32(0.05)])[None]
    v = np.stack([(i * 2 + d) * np.float32(0.1), (d - i) * np.float32(0.1)])[None]
    rc, out = _device(q, k, v)
    assert rc == 0
    assert np.max(np.abs(out - _sdpa(q, k, v))) < TOL
    assert np.max(np.abs(out - O.flash_attention(q, k, v))) < TOL


def test_reference_grouped_query_inputs():
    """FlashAttentionCpu_GroupedQueryAttention_MatchesExpanded (NeuralOperatorsTests.cs:660-723): 4 q heads over 2
    kv heads, 8 x 16."""
    h = np.arange(4, dtype=np.float64)[:, None, None]
    s = np.arange(8, dtype=np.float64)[None, :, None]
    d = np.arange(16, dtype=np.float64)[None, None, :]
    q = np.sin(h * 10 + s + d * 0.1).astype(np.float32)[None]
    hk = np.arange(2, dtype=np.float64)[:, None, None]
    k = np.cos(hk * 5 + s * 0.5 + d * 0.2).astype(np.float32)[None]
    v = np.sin(hk * 3 + s * 0.2 + d * 0.3).astype(np.float32)[None]
    rc, out = _device(q, k, v)
    assert rc == 0
    assert np.max(np.abs(out - _sdpa(q, k, v))) < TOL
    assert np.max(np.abs(out - O.flash_attention(q, k, v))) < TOL


# (batch, hq, hkv, sq, sk, d): single rows, ragged tiles and key blocks, GQA and MQA, every head size
SHAPES = [(1, 8, 2, 1, 1, 64), (2, 8, 2, 37, 300, 64), (1, 4, 4, 130, 70, 128), (1, 32, 8, 96, 1000, 128),
          (2, 6, 1, 33, 17, 32), (1, 2, 2, 65, 129, 16), (1, 12, 12, 512, 512, 64)]


@pytest.mark.parametrize("shape", SHAPES)
def test_grouped_shapes_match_oracle(shape):
    b, hq, hkv, sq, sk, d = shape
    rng = np.random.default_rng(sum(shape))
    q = rng.standard_normal((b, hq, sq, d)).astype(np.float32)
    k = rng.standard_normal((b, hkv, sk, d)).astype(np.float32)
    v = rng.standard_normal((b, hkv, sk, d)).astype(np.float32)
    rc, out = _device(q, k, v)
    assert rc == 0
    assert np.max(np.abs(out - O.flash_attention(q, k, v))) < TOL


def test_flattened_batch_and_peaked_scores():
    """Rank-3 tensors (the batch is every leading dimension, kv batch = batch) and scores in the hundreds, where the
    running maximum moves by large steps between key blocks.  At scale 0.5 the scores reach ~600: a 64-term fp32 dot
    product of that size is only defined to ~3e-4 in any summation order, which moves a softmax weight by as much
    relatively, so that case is checked at 1e-3."""
    rng = np.random.default_rng(9)
    q = (rng.standard_normal((5, 70, 64)) * 6).astype(np.float32)
    k = (rng.standard_normal((5, 200, 64)) * 6).astype(np.float32)
    v = rng.standard_normal((5, 200, 64)).astype(np.float32)
    rc, out = _device(q, k, v)
    assert rc == 0
    assert np.max(np.abs(out - O.flash_attention(q, k, v))) < TOL
    rc, out = _device(q, k, v, scale=0.5)
    assert rc == 0 and np.max(np.abs(out - O.flash_attention(q, k, v, scale=0.5))) < 1e-3


def test_unhandled_forms_return_minus_one_and_edges():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 2, 8, 64)).astype(np.float32)
    k = rng.standard_normal((1, 2, 12, 64)).astype(np.float32)
    v = rng.standard_normal((1, 2, 12, 64)).astype(np.float32)
    rc, out = _device(q, k, v, mask=np.zeros((8, 12), np.float32))
    assert rc == -1 and np.all(out == 7.0)                            # a mask: the managed path runs
    rc, out = _device(q, k, rng.standard_normal((1, 2, 12, 32)).astype(np.float32))
    assert rc == -1 and np.all(out == 7.0)                            # dv != d
    rc, out = _device(q[..., :8], k[..., :8], v[..., :8])
    assert rc == -1                                                   # d = 8
    rc, out = _device(q, k[:, :, :0], v[:, :, :0])
    assert rc == 0 and np.all(out == 0.0)                             # no keys: zeros (sum 0)
    assert np.all(O.flash_attention(q, k[:, :, :0], v[:, :, :0]) == 0.0)


@pytest.mark.parametrize("page_size", [8, 16, 32])
@pytest.mark.parametrize("heads,kv_heads,dim", [(12, 12, 768), (8, 2, 1024)])
def test_engine_long_prefill_matches_oracle(page_size, heads, kv_heads, dim):
    """A prompt long enough for the tiled prefill kernel (at least 64 rows): 290 tokens at once, then 200 tokens and
    a 90-token chunk at position 200 whose rows see the first chunk's keys; logits vs the oracle within 1e-3
    max-rel (the engine's tolerance)."""
    from zeroplatform_b200.engine import LlmEngine
    m = O.make_model(vocab=2048, dim=dim, layers=2, heads=heads, kv_heads=kv_heads, ffn=1024, seed=page_size)
    rng = np.random.default_rng(page_size)
    prompt = rng.integers(0, 2048, 290).astype(np.int32)
    pages = 2 * (290 // page_size + 2)
    e = LlmEngine(m, total_pages=pages, page_size=page_size, max_pages_per_seq=pages // 2)
    ref = O.Engine(m, total_pages=pages, page_size=page_size, kv_fp16=True)
    assert rel_err(e.prefill(1, prompt, 0), ref.prefill(1, prompt, 0)) <= 1e-3
    assert rel_err(e.prefill(2, prompt[:200], 0), ref.prefill(2, prompt[:200], 0)) <= 1e-3
    assert rel_err(e.prefill(2, prompt[200:], 200), ref.prefill(2, prompt[200:], 200)) <= 1e-3
    assert rel_err(e.forward_token(2, 7, 290), ref.forward_token(2, 7, 290)) <= 1e-3
    e.close()
    ref.close()
