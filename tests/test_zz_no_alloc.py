"""zcu_paged_attention_noalloc: paged decode attention that allocates no device memory.

Some users of this library cannot call cudaMalloc at the moment they run attention: a serving process that
has already handed all free HBM to its KV page pool (a late allocation would fail or fragment it), or a host
runtime whose decode loop forbids device allocation after start-up because cudaMalloc and cudaFree can
synchronise the whole device and stall every stream on it.  For them the library keeps the split-K scratch of
the attention kernel in a fixed 1 MiB array compiled into libzero_tensor.so instead of a workspace it allocates
on demand.

These tests call the entry point through the C ABI and check it against zcu_paged_attention (the allocating
entry point) and against the oracle, with the tolerance of the other attention tests, on two calls in a row, so
that scratch left behind by the first call cannot leak into the second.  This file is collected last.
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _lib():
    from zeroplatform_b200 import _lib
    return _lib.lib()


def _case(seed, batch, hq, hkv, hd, max_ctx, ps=16):
    """Head-major fp16 pools [page][kv head][slot][hd], a random page table, per-sequence context lengths."""
    rng = np.random.default_rng(seed)
    max_pages = (max_ctx + ps - 1) // ps
    num_pages = batch * max_pages + 2
    k = torch.from_numpy(rng.standard_normal((num_pages, hkv, ps, hd), dtype=np.float32)).half().cuda()
    v = torch.from_numpy(rng.standard_normal((num_pages, hkv, ps, hd), dtype=np.float32)).half().cuda()
    pt = torch.from_numpy(rng.permutation(num_pages)[:batch * max_pages].astype(np.int32).reshape(batch, max_pages)).cuda()
    ctx = rng.integers(1, max_ctx + 1, batch).astype(np.int32)
    ctx[0] = max_ctx
    q = torch.from_numpy(rng.standard_normal((batch, hq, hd), dtype=np.float32)).cuda()
    return dict(q=q, k=k, v=v, pt=pt, ctx=torch.from_numpy(ctx).cuda(), batch=batch, hq=hq, hkv=hkv, hd=hd, ps=ps,
                max_pages=max_pages, num_pages=num_pages, max_ctx=max_ctx)


def _call(fn, c, out):
    return fn(c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(), 1, c["pt"].data_ptr(), c["ctx"].data_ptr(),
              out.data_ptr(), c["batch"], c["hq"], c["hkv"], c["hd"], c["ps"], c["max_pages"], c["num_pages"],
              c["hkv"] * c["ps"] * c["hd"], c["hd"], c["ps"] * c["hd"],
              float(np.float32(1.0) / np.float32(np.sqrt(c["hd"]))), c["max_ctx"],
              torch.cuda.current_stream().cuda_stream)


def test_no_alloc_matches_allocating_entry_point_on_two_calls_in_a_row():
    L = _lib()
    # Two different shapes, both with several splits per sequence, so the shared scratch is used twice.
    cases = [_case(1, batch=2, hq=12, hkv=12, hd=64, max_ctx=640), _case(2, batch=1, hq=8, hkv=2, hd=128, max_ctx=1000)]
    for c in cases:
        ref = torch.empty_like(c["q"])
        got = torch.full_like(c["q"], float("nan"))
        assert _call(L.zcu_paged_attention, c, ref) == 0
        assert _call(L.zcu_paged_attention_noalloc, c, got) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= TOL
        # and against the oracle (TensorOps.PagedAttention, slot-major fp32 pools) sequence by sequence
        kf = c["k"].float().permute(0, 2, 1, 3).contiguous().cpu().numpy()
        vf = c["v"].float().permute(0, 2, 1, 3).contiguous().cpu().numpy()
        pt, ctx, q = c["pt"].cpu().numpy(), c["ctx"].cpu().numpy(), c["q"].cpu().numpy()
        g = got.cpu().numpy()
        for b in range(c["batch"]):
            want = O.paged_attention(q[b], kf, vf, pt[b], int(ctx[b]))
            assert rel_err(g[b], want) <= TOL


def test_no_alloc_rejects_shapes_beyond_its_fixed_scratch():
    """64 query heads x 64 splits x (128 + 2) floats exceed the 1 MiB array: refused before any launch."""
    L = _lib()
    c = _case(3, batch=1, hq=64, hkv=4, hd=128, max_ctx=4096)
    out = torch.zeros_like(c["q"])
    rc = _call(L.zcu_paged_attention_noalloc, c, out)
    assert rc == -6
    assert b"scratch" in L.zc_cuda_last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing was launched
