"""Decode-step operators and the remaining bridge entry points vs the oracle / numpy restatements."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data


def L():
    from zeroplatform_b200 import _lib
    return _lib.lib()


def _s():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("rows,n", [(1, 768), (7, 4096), (3, 32), (2, 11008)])
def test_rmsnorm_matches_oracle(rows, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((rows, n), dtype=np.float32)
    w = rng.standard_normal(n, dtype=np.float32)
    ref = np.stack([O.rmsnorm(x[r], w) for r in range(rows)])
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.empty_like(xd)
    assert L().zcu_rmsnorm(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), rows, n, 1e-5, _s()) == 0
    assert rel_err(out.cpu().numpy(), ref) <= 1e-6
    host = np.empty(n, np.float32)
    assert L().zc_rmsnorm_f32(n, _p(x[0]), _p(w), _p(host), 1e-5) == 0
    assert rel_err(host, ref[0]) <= 1e-6


def test_swiglu_and_silu():
    rng = np.random.default_rng(1)
    g = (rng.standard_normal(11008, dtype=np.float32) * 4).astype(np.float32)
    u = rng.standard_normal(11008, dtype=np.float32)
    ref = O.swiglu(g, u)
    gd, ud = torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()
    out = torch.empty_like(gd)
    assert L().zcu_swiglu(gd.data_ptr(), ud.data_ptr(), out.data_ptr(), g.size, _s()) == 0
    assert rel_err(out.cpu().numpy(), ref) <= 1e-6
    host = np.empty_like(g)
    assert L().zc_swiglu_f32(g.size, _p(g), _p(u), _p(host)) == 0
    assert rel_err(host, ref) <= 1e-6
    assert L().zc_silu_f32(g.size, _p(g), _p(host)) == 0
    assert rel_err(host, g / (1 + np.exp(-g.astype(np.float64)))) <= 1e-6


@pytest.mark.parametrize("hd,heads,rows,pos0", [(64, 12, 1, 0), (64, 12, 5, 1000), (128, 32, 3, 2047), (8, 2, 4, 3)])
def test_rope_matches_oracle_table(hd, heads, rows, pos0):
    rng = np.random.default_rng(hd + pos0)
    max_pos = max(1024, pos0 + rows + 1)
    cos_t, sin_t = O.rope_table(max_pos, hd)
    x = rng.standard_normal((rows, heads, hd), dtype=np.float32)
    ref = np.stack([np.stack([O.rope_apply(x[r, h], pos0 + r, hd, cos_t, sin_t) for h in range(heads)])
                    for r in range(rows)])
    xd = torch.from_numpy(x).cuda()
    ct, st = torch.from_numpy(cos_t).cuda(), torch.from_numpy(sin_t).cuda()
    assert L().zcu_rope(xd.data_ptr(), rows, heads, hd, None, pos0, ct.data_ptr(), st.data_ptr(), max_pos, _s()) == 0
    assert np.array_equal(xd.cpu().numpy(), ref)  # identical table, identical float ops


def test_bridge_rope_tensorops_formula():
    """zc_rope_f32 follows TensorOps.ApplyRoPEInPlace's interleaved branch (TensorOps.Neural.cs:1246-1366)."""
    rng = np.random.default_rng(2)
    heads, seq, hd, pos0, theta = 3, 5, 16, 7, np.float32(10000.0)
    x = rng.standard_normal((heads, seq, hd), dtype=np.float32)
    ref = x.copy()
    for s in range(seq):
        for i in range(hd // 2):
            inv = np.float32(np.float32(1.0) / np.float32(np.power(np.float64(theta), (2.0 * i) / hd)))
            ang = np.float32(np.float32(pos0 + s) * inv)
            c, sn = np.float32(np.cos(np.float64(ang))), np.float32(np.sin(np.float64(ang)))
            a, b = x[:, s, 2 * i].copy(), x[:, s, 2 * i + 1].copy()
            ref[:, s, 2 * i] = a * c - b * sn
            ref[:, s, 2 * i + 1] = b * c + a * sn
    out = x.copy()
    assert L().zc_rope_f32(heads, seq, hd, pos0, float(theta), _p(out)) == 0
    assert np.max(np.abs(out - ref)) <= 1e-6


def test_embed_q8_0_matches_dequantized_rows():
    from zeroplatform_b200.ops import QuantizedWeight
    rng = np.random.default_rng(3)
    vocab, dim = 100, 96
    table = O.quantize_q8_0(rng.standard_normal((vocab, dim), dtype=np.float32) * np.float32(0.02))
    deq = O.dequantize_q8_0(table, dim)
    qw = QuantizedWeight.upload(8, table, vocab, dim)
    toks = np.array([5, 0, 99, -3, 100, 42], np.int32)   # unknown ids read row 0 (LlmEngine.cs:321)
    td = torch.from_numpy(toks).cuda()
    out = torch.empty((len(toks), dim), dtype=torch.float32, device="cuda")
    assert L().zcu_embed_q8_0(qw.qs.data_ptr(), qw.d.data_ptr(), td.data_ptr(), len(toks), vocab, dim,
                              out.data_ptr(), _s()) == 0
    exp = deq[[5, 0, 99, 0, 0, 42]]
    assert np.array_equal(out.cpu().numpy(), exp)


def test_bridge_dot_i8_exact():
    rng = np.random.default_rng(4)
    for n in [0, 1, 19, 4096, 1_000_003]:
        a = rng.integers(-128, 128, n).astype(np.int8)
        b = rng.integers(-128, 128, n).astype(np.int8)
        out = np.zeros(1, np.int32)
        assert L().zc_dot_i8(n, _p(a) if n else 0, _p(b) if n else 0, _p(out)) == 0
        assert int(out[0]) == O.dot_i8(a, b) == int(a.astype(np.int64) @ b.astype(np.int64))


@pytest.mark.parametrize("m,n,k,trans", [(5, 7, 3, False), (64, 96, 130, True), (1, 1000, 64, False)])
def test_bridge_gemm_f32_strided(m, n, k, trans):
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k), dtype=np.float32)
    bmat = rng.standard_normal((k, n), dtype=np.float32)
    c = rng.standard_normal((m, n), dtype=np.float32)
    alpha, beta = np.float32(0.5), np.float32(1.5)
    ref = alpha * (a.astype(np.float64) @ bmat.astype(np.float64)) + beta * c.astype(np.float64)
    if trans:  # B given as its transpose in memory (row stride 1, column stride k)
        bt = np.ascontiguousarray(bmat.T)
        rc = L().zc_gemm_f32(m, n, k, alpha, _p(a), k, 1, _p(bt), 1, k, beta, _p(c), n, 1, 1)
    else:
        rc = L().zc_gemm_f32(m, n, k, alpha, _p(a), k, 1, _p(bmat), n, 1, beta, _p(c), n, 1, 1)
    assert rc == 0
    assert rel_err(c, ref) <= 1e-5


def test_flash_attention_declines_what_it_does_not_run():
    """zc_flash_attention_f32 answers -1 (the managed FlashAttention runs) for head size 8 and for a mask; null
    buffers are a bad argument (-2).  The handled forms are in test_flash_attention_gpu.py."""
    q = np.zeros(8, np.float32)
    p = q.ctypes.data_as(ctypes.c_void_p)
    assert L().zc_flash_attention_f32(1, 1, 1, 8, 8, 1.0, 0, 1, 1, 1, p, p, p, None, p) == -1
    assert L().zc_flash_attention_f32(1, 1, 1, 8, 8, 1.0, 0, 1, 1, 1, p, p, p, p, p) == -1
    assert L().zc_flash_attention_f32(1, 1, 1, 64, 64, 1.0, 0, 1, 1, 1, None, None, None, None, None) == -2


def test_bounded_peer_wait_runs_out_and_reports():
    """The tensor-parallel all-reduce's reduce kernel waits (bounded) until every peer's words carry the current
    epoch.  Here it runs on one GPU against a receive area of 2 (and 8) ranks where no peer ever pushes: the wait
    must give up after the shortened limit, record code 21 with what it saw (it needed epoch 1; rank 0's words
    carry 1, the others 0), and return -- and the context must stay usable for the next kernel."""
    import time
    from zeroplatform_b200 import _lib
    from zeroplatform_b200.ops import QuantizedWeight
    L = _lib.lib()
    for ranks in (2, 8):
        seen = (ctypes.c_uint32 * 16)()
        t0 = time.perf_counter()
        rc = L.zcu_peer_wait_selftest(ranks, 200, seen)
        el = time.perf_counter() - t0
        assert rc == 21, rc
        assert 0.15 < el < 5.0, el
        assert seen[4] == 1 and seen[5] == 1 and all(seen[5 + q] == 0 for q in range(1, ranks))
    assert L.zcu_peer_wait_selftest(1, 200, None) == -2 and L.zcu_peer_wait_selftest(2, 0, None) == -2
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 256), dtype=np.float32) * np.float32(0.02)
    blocks = O.quantize_q8_0(w)
    x = rng.standard_normal(256, dtype=np.float32)
    y = QuantizedWeight.upload(8, blocks, 64, 256).gemv(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), O.matvec(8, blocks, x, 64, 256)) <= 1e-5
    assert L.zcu_device_status(1) == 0  # the self-test used its own status word
