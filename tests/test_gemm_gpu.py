"""Prefill / batched Q8_0 GEMM on tcgen05 vs the oracle's token-parallel MatVecMulQ8_0 (LlmEngine.PrefillPrompt).

Tolerance: max|Y - Y_oracle| / max|Y_oracle| <= 1e-3 -- the parity bound for fp32 outputs.  The tensor
core consumes both operands as fp16 pairs (weights hi = fp16(q*d), lo = fp16(q*d - hi); activations hi = fp16(x),
lo = fp16(x - hi)) with fp32 accumulation, so the products carry ~2^-22 and the result differs from the fp32
restatement by summation order; the measured error is printed.
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _lib():
    from zeroplatform_b200 import _lib
    return _lib.lib()


def _run(qw, x, y, accumulate=False):
    fn = _lib().zcu_gemm_q8_0 if qw.qtype == 8 else _lib().zcu_gemm_q4_0
    rc = fn(qw.qs.data_ptr(), qw.d.data_ptr(), x.data_ptr(), y.data_ptr(), x.shape[0], qw.rows, qw.cols,
            int(accumulate), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert _lib().zcu_device_status(1) == 0  # no bounded wait expired


@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (5, 200, 96), (64, 256, 768), (100, 384, 2048), (130, 1000, 4096),
                                   (257, 128, 128), (512, 11008, 4096), (32, 4096, 4096), (32, 4096, 11008),
                                   (9, 2304, 768), (128, 11008, 4096), (33, 96, 4096)])
def test_gemm_matches_oracle(m, n, k):
    from zeroplatform_b200.ops import QuantizedWeight
    rng = np.random.default_rng(m * 7 + n + k)
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal((m, k), dtype=np.float32)
    blocks = O.quantize_q8_0(w)
    ref = O.matmul(8, blocks, x, n, k)
    qw = QuantizedWeight.upload(8, blocks, n, k)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((m, n), float("nan"), device="cuda")
    _run(qw, xd, y)
    err = rel_err(y.cpu().numpy(), ref)
    print(f"gemm {m}x{n}x{k}: max-rel err {err:.3e}")
    assert err <= TOL
    # MatVecAdd form (Wo / Wdown residual adds): Y += W X
    y0 = rng.standard_normal((m, n), dtype=np.float32)
    yt = torch.from_numpy(y0.copy()).cuda()
    _run(qw, xd, yt, accumulate=True)
    assert rel_err(yt.cpu().numpy() - y0, ref) <= TOL


def test_gemm_is_deterministic_and_repeatable():
    from zeroplatform_b200.ops import QuantizedWeight
    rng = np.random.default_rng(1)
    n, k, m = 512, 1024, 300
    qw = QuantizedWeight.upload(8, O.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)),
                                n, k)
    xd = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).cuda()
    y1 = torch.empty((m, n), device="cuda")
    y2 = torch.empty((m, n), device="cuda")
    _run(qw, xd, y1)
    _run(qw, xd, y2)
    assert torch.equal(y1, y2)


def test_gemm_matches_exact_products_tightly():
    """The weight and activation hi / lo pairs carry q*d and x to ~2^-22: against float64 sums of the exact
    products only fp32 summation order differs."""
    from zeroplatform_b200.ops import QuantizedWeight
    rng = np.random.default_rng(2)
    n, k, m = 256, 512, 96
    blocks = O.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal((m, k), dtype=np.float32)
    b = blocks.reshape(n, k // 32, 34)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32)          # [n, k/32, 1]
    q = b[:, :, 2:].view(np.int8).astype(np.float32)                   # [n, k/32, 32]
    w = (q.astype(np.float64) * d).reshape(n, k)                       # exact q*d
    ref = x.astype(np.float64) @ w.T
    qw = QuantizedWeight.upload(8, blocks, n, k)
    y = torch.empty((m, n), device="cuda")
    _run(qw, torch.from_numpy(x).cuda(), y)
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (64, 256, 768), (130, 1000, 4096), (64, 28672, 4096),
                                   (64, 4096, 14336), (9, 2304, 96)])
def test_gemm_q4_0_matches_oracle(m, n, k):
    """Q4_0 weights (the MoE experts' format) on the tensor cores vs the oracle's token-parallel MatVecMulQ4_0."""
    from zeroplatform_b200.ops import QuantizedWeight
    rng = np.random.default_rng(m * 13 + n + k)
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal((m, k), dtype=np.float32)
    blocks = O.quantize_q4_0(w)
    ref = O.matmul(4, blocks, x, n, k)
    qw = QuantizedWeight.upload(4, blocks, n, k)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((m, n), float("nan"), device="cuda")
    _run(qw, xd, y)
    err = rel_err(y.cpu().numpy(), ref)
    print(f"gemm q4_0 {m}x{n}x{k}: max-rel err {err:.3e}")
    assert err <= TOL
    y0 = rng.standard_normal((m, n), dtype=np.float32)
    yt = torch.from_numpy(y0.copy()).cuda()
    _run(qw, xd, yt, accumulate=True)
    assert rel_err(yt.cpu().numpy() - y0, ref) <= TOL
