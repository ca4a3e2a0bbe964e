"""Decode GEMV parity: CUDA (libzero_tensor.so) vs the CPU oracle on identical seeded inputs.

Tolerance: max|y - y_oracle| / max|y_oracle| <= 3e-4 (the parity bound for fp32 outputs is 1e-3).  GEMVs below 64 MB of
weights keep x in fp32 (only the summation order differs: ~1e-6).  The streaming form for large weights
re-expresses x per 32-value block as int16 (scale max|x| / 32767, so each value is within 2^-16 of the block
maximum) and sums int16 x int8 products exactly in int32 (DP2A): for N(0,1) activations and N(0,0.02) weights
at K = 4096 that error has a standard deviation of about 2.4e-5 per output against max|y| of about 4.5
(max-rel ~2e-5).  The oracle keeps x in fp32, as the reference does.
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 3e-4

# (32768, 4096) is large enough (>= 64 MB of weights) for the streaming form (int16 activations, DP2A, L2
# prefetch); the others run the fp32-activation forms: Q8_0 rows of K = 4096 the slab form (7 rows a CTA, 4 in
# registers and 3 bulk-copied: 10 and 13 rows leave partial CTAs), K > 8192 in segments.
SHAPES = [(1, 32), (3, 64), (17, 96), (1023, 768), (2304, 768), (4096, 4096), (768, 2048), (4096, 11008),
          (11008, 4096), (257, 14336), (33, 20480), (64, 1056), (40, 2080), (150, 256), (149, 512), (2, 4096),
          (10, 4096), (13, 4096), (32768, 4096)]


def _case(qtype, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal(cols, dtype=np.float32)
    blocks = O.quantize_q8_0(w) if qtype == 8 else O.quantize_q4_0(w)
    return blocks, x, rng


@pytest.mark.parametrize("qtype", [8, 4])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_device_gemv_matches_oracle(qtype, rows, cols):
    from zeroplatform_b200.ops import QuantizedWeight
    blocks, x, rng = _case(qtype, rows, cols, rows * 131 + cols + qtype)
    ref = O.matvec(qtype, blocks, x, rows, cols)
    qw = QuantizedWeight.upload(qtype, blocks, rows, cols)
    xd = torch.from_numpy(x).cuda()
    y = qw.gemv(xd)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), ref) <= TOL
    # MatVecAdd: y += W x
    y0 = rng.standard_normal(rows, dtype=np.float32)
    yt = torch.from_numpy(y0.copy()).cuda()
    qw.gemv(xd, yt, accumulate=True)
    ref_acc = O.matvec(qtype, blocks, x, rows, cols, y=y0.copy())
    assert rel_err(yt.cpu().numpy(), ref_acc) <= TOL


def test_repack_is_a_pure_relayout():
    from zeroplatform_b200.ops import QuantizedWeight
    blocks, _, _ = _case(8, 64, 256, 1)
    qw = QuantizedWeight.upload(8, blocks, 64, 256)
    b = blocks.reshape(64, 8, 34)
    assert np.array_equal(qw.qs.cpu().numpy().view(np.uint8).reshape(64, 8, 32), b[:, :, 2:])
    assert np.array_equal(qw.d.cpu().numpy().view(np.uint8).reshape(64, 8, 2), b[:, :, :2])
    b4, _, _ = _case(4, 64, 256, 2)
    q4 = QuantizedWeight.upload(4, b4, 64, 256)
    b4 = b4.reshape(64, 8, 18)
    assert np.array_equal(q4.qs.cpu().numpy().reshape(64, 8, 16), b4[:, :, 2:])
    assert np.array_equal(q4.d.cpu().numpy().view(np.uint8).reshape(64, 8, 2), b4[:, :, :2])


# ---- the reference bridge ABI with host buffers (NeuralOperatorsTests.cs:584-628 goldens) ---------------
def test_bridge_gemv_q8_0_golden_192():
    from zeroplatform_b200.ops import TensorBlas
    blk = np.zeros(34, np.uint8)
    blk[1] = 0x40
    blk[2:] = 3
    y = TensorBlas.gemv_q8_0(np.ones(32, np.float32), blk, 1, 32)
    assert abs(y[0] - 192.0) < 1e-4


def test_bridge_gemv_q4_0_golden_48():
    from zeroplatform_b200.ops import TensorBlas
    blk = np.zeros(18, np.uint8)
    blk[1] = 0x3C
    blk[2:] = 0x9A
    y = TensorBlas.gemv_q4_0(np.ones(32, np.float32), blk, 1, 32)
    assert abs(y[0] - 48.0) < 1e-4


@pytest.mark.parametrize("qtype", [8, 4])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (300, 11008), (5, 64)])
def test_bridge_gemv_matches_oracle(qtype, rows, cols):
    from zeroplatform_b200.ops import TensorBlas
    blocks, x, _ = _case(qtype, rows, cols, 99 + rows)
    ref = O.matvec(qtype, blocks, x, rows, cols)
    fn = TensorBlas.gemv_q8_0 if qtype == 8 else TensorBlas.gemv_q4_0
    assert rel_err(fn(x, blocks, rows, cols), ref) <= TOL


def test_bridge_rejects_bad_k():
    from zeroplatform_b200 import _lib
    from zeroplatform_b200.ops import _np_ptr
    x = np.ones(48, np.float32)
    y = np.zeros(1, np.float32)
    w = np.zeros(64, np.uint8)
    assert _lib.lib().zc_gemv_q8_0(_np_ptr(w), _np_ptr(x), _np_ptr(y), 1, 48) == -2


def test_bridge_is_reentrant_across_threads():
    """LlmEngine.PrefillPrompt calls the kernels from Parallel.For workers (LlmEngine.cs:208)."""
    import concurrent.futures as cf
    from zeroplatform_b200.ops import TensorBlas
    cases = [_case(8, 512, 768, s) for s in range(8)]
    refs = [O.matvec(8, b, x, 512, 768) for b, x, _ in cases]
    with cf.ThreadPoolExecutor(8) as ex:
        outs = list(ex.map(lambda c: TensorBlas.gemv_q8_0(c[1], c[0], 512, 768), cases))
    for o, r in zip(outs, refs):
        assert rel_err(o, r) <= TOL


@pytest.mark.parametrize("qtype", [8, 4])
@pytest.mark.parametrize("scale", [0.02, 1.0, 1e-6, 300.0])
def test_device_quantizer_bit_exact(qtype, scale):
    """zcu_quantize_q*_0 vs LlmQuantizer (oracle): identical bytes, including all-zero and outlier blocks."""
    from zeroplatform_b200.ops import quantize
    rng = np.random.default_rng(int(scale * 1000) + qtype)
    w = (rng.standard_normal((96, 512)) * scale).astype(np.float32)
    w[0, :32] = 0.0
    w[1, 7] = 9 * scale
    w[2, 40] = -9 * scale
    ref = O.quantize_q8_0(w) if qtype == 8 else O.quantize_q4_0(w)
    got = quantize(qtype, torch.from_numpy(w).cuda()).cpu().numpy()
    assert np.array_equal(got, ref)


def test_registered_weights_are_used_and_released():
    """zc_register_weights keeps a device copy: results match, and re-registering picks up new bytes."""
    from zeroplatform_b200 import _lib
    from zeroplatform_b200.ops import TensorBlas, _np_ptr
    L = _lib.lib()
    blocks, x, _ = _case(8, 1024, 768, 5)
    ref = O.matvec(8, blocks, x, 1024, 768)
    assert L.zc_register_weights(8, _np_ptr(blocks), 1024, 768) == 0
    assert rel_err(TensorBlas.gemv_q8_0(x, blocks, 1024, 768), ref) <= TOL
    other, _, _ = _case(8, 1024, 768, 6)
    blocks[...] = other                      # caller broke the promise: the resident copy is still used
    assert rel_err(TensorBlas.gemv_q8_0(x, blocks, 1024, 768), ref) <= TOL
    assert L.zc_register_weights(8, _np_ptr(blocks), 1024, 768) == 0   # re-registration refreshes the copy
    assert rel_err(TensorBlas.gemv_q8_0(x, blocks, 1024, 768), O.matvec(8, other, x, 1024, 768)) <= TOL
    assert L.zc_unregister_weights(_np_ptr(blocks)) == 0
    assert L.zc_unregister_weights(_np_ptr(blocks)) == -1
    assert rel_err(TensorBlas.gemv_q8_0(x, blocks, 1024, 768), O.matvec(8, other, x, 1024, 768)) <= TOL
    b4, x4, _ = _case(4, 300, 2048, 7)
    assert L.zc_register_weights(2, _np_ptr(b4), 300, 2048) == 0
    assert rel_err(TensorBlas.gemv_q4_0(x4, b4, 300, 2048), O.matvec(4, b4, x4, 300, 2048)) <= TOL
    assert L.zc_unregister_weights(_np_ptr(b4)) == 0


def test_registered_weights_replayed_calls_track_new_activations():
    """Calls on registered weights after the first replay one recorded graph (zero-copy x / y through pinned
    buffers): every call must see its own x, including a row count whose y is not a whole number of 16 bytes."""
    from zeroplatform_b200 import _lib
    from zeroplatform_b200.ops import TensorBlas, _np_ptr
    L = _lib.lib()
    for qtype, ggml, n, k in ((8, 8, 301, 512), (4, 2, 77, 1024)):
        blocks, _, _ = _case(qtype, n, k, 11)
        assert L.zc_register_weights(ggml, _np_ptr(blocks), n, k) == 0
        rng = np.random.default_rng(12)
        gemv = TensorBlas.gemv_q8_0 if qtype == 8 else TensorBlas.gemv_q4_0
        for _ in range(4):
            x = rng.standard_normal(k, dtype=np.float32)
            assert rel_err(gemv(x, blocks, n, k), O.matvec(qtype, blocks, x, n, k)) <= TOL
        assert L.zc_unregister_weights(_np_ptr(blocks)) == 0
