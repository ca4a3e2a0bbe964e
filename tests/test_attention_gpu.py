"""Paged decode attention parity: CUDA vs the CPU oracle (GqaAttention two-pass softmax and
TensorOps.PagedAttention online softmax), fp32 and fp16 page pools.

Tolerance: max|out - out_oracle| / max|out_oracle| <= 1e-5 (fp32 math on identical K/V values; for fp16
pools the oracle reads the same fp16-rounded K/V).
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _pools(rng, num_pages, page_size, hkv, hd):
    k = rng.standard_normal((num_pages, page_size, hkv, hd), dtype=np.float32)
    v = rng.standard_normal((num_pages, page_size, hkv, hd), dtype=np.float32)
    return k, v


def test_reference_setup_blocktable_201_ctx10():
    """TensorOps.PagedAttention setup of NeuralOperatorsTests.cs:950-971 (hq 4, hkv 2, hd 8, bs 4, ctx 10)."""
    from zeroplatform_b200.ops import TensorOps
    rng = np.random.default_rng(42)
    q = rng.standard_normal((4, 8), dtype=np.float32)
    k, v = _pools(rng, 3, 4, 2, 8)
    bt = np.array([2, 0, 1], np.int32)
    ref = O.paged_attention(q, k, v, bt, 10)
    host = TensorOps.paged_attention(q, k, v, bt, 10)          # bridge ABI, host buffers
    assert np.max(np.abs(host - ref)) < 1e-3 and rel_err(host, ref) <= TOL
    dev = TensorOps.paged_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                                    torch.from_numpy(v).cuda(), bt, 10)
    assert rel_err(dev.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("hq,hkv,hd", [(4, 2, 8), (12, 12, 64), (32, 32, 128), (8, 1, 64), (6, 2, 32), (4, 4, 256),
                                       (3, 1, 16)])
@pytest.mark.parametrize("ctx", [0, 1, 15, 16, 17, 100, 640, 2048])
def test_bridge_paged_attention_matches_oracle(hq, hkv, hd, ctx):
    from zeroplatform_b200.ops import TensorOps
    rng = np.random.default_rng(hq * 1000 + hd * 7 + ctx)
    bs = 16
    nlb = max(1, (ctx + bs - 1) // bs)
    num_pages = nlb + 5
    q = rng.standard_normal((hq, hd), dtype=np.float32)
    k, v = _pools(rng, num_pages, bs, hkv, hd)
    bt = rng.permutation(num_pages)[:nlb].astype(np.int32)
    ref = O.paged_attention(q, k, v, bt, ctx)
    two_pass = O.gqa_attention(q.reshape(-1), k, v, bt, bs, ctx, hq, hkv, hd).reshape(hq, hd)
    out = TensorOps.paged_attention(q, k, v, bt, ctx)
    if ctx == 0:
        assert np.all(out == 0)
        return
    assert rel_err(out, ref) <= TOL
    assert rel_err(out, two_pass) <= TOL


@pytest.mark.parametrize("kv_half", [False, True])
@pytest.mark.parametrize("batch,hq,hkv,hd,max_ctx", [(1, 12, 12, 64, 640), (32, 32, 32, 128, 300), (4, 8, 2, 64, 1000),
                                                     (3, 16, 16, 128, 33)])
def test_batched_head_major_pools(kv_half, batch, hq, hkv, hd, max_ctx):
    """The engine's layout: pool [page][kv head][slot][hd], per-sequence ctx_len, shared page pool."""
    from zeroplatform_b200.ops import paged_attention_batched
    rng = np.random.default_rng(batch * 17 + hd + int(kv_half))
    ps = 16
    max_pages = (max_ctx + ps - 1) // ps
    num_pages = batch * max_pages + 3
    k = rng.standard_normal((num_pages, hkv, ps, hd), dtype=np.float32)
    v = rng.standard_normal((num_pages, hkv, ps, hd), dtype=np.float32)
    if kv_half:
        k = k.astype(np.float16).astype(np.float32)
        v = v.astype(np.float16).astype(np.float32)
    perm = rng.permutation(num_pages)[:batch * max_pages].astype(np.int32).reshape(batch, max_pages)
    ctx = rng.integers(0, max_ctx + 1, batch).astype(np.int32)
    ctx[0] = max_ctx
    q = rng.standard_normal((batch, hq, hd), dtype=np.float32)
    # oracle wants [page][slot][hkv][hd]
    k_ref = np.ascontiguousarray(k.transpose(0, 2, 1, 3))
    v_ref = np.ascontiguousarray(v.transpose(0, 2, 1, 3))
    dt = torch.float16 if kv_half else torch.float32
    kd = torch.from_numpy(k).to(dt).cuda()
    vd = torch.from_numpy(v).to(dt).cuda()
    out = paged_attention_batched(torch.from_numpy(q).cuda(), kd, vd, torch.from_numpy(perm).cuda(),
                                  torch.from_numpy(ctx).cuda(), hkv, ps, num_pages, hkv * ps * hd, hd, ps * hd,
                                  float(np.float32(1) / np.float32(np.sqrt(hd))), max_ctx)
    out = out.cpu().numpy()
    for b in range(batch):
        ref = O.gqa_attention(q[b].reshape(-1), k_ref, v_ref, perm[b], ps, int(ctx[b]), hq, hkv, hd).reshape(hq, hd)
        if ctx[b] == 0:
            assert np.all(out[b] == 0)
        else:
            assert rel_err(out[b], ref) <= TOL, b


def test_invalid_page_ids_are_skipped_not_dereferenced():
    from zeroplatform_b200.ops import paged_attention_batched
    rng = np.random.default_rng(5)
    hq = hkv = 2
    hd, ps = 64, 16
    k = torch.from_numpy(rng.standard_normal((4, hkv, ps, hd), dtype=np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((4, hkv, ps, hd), dtype=np.float32)).cuda()
    pt = torch.tensor([[0, 1_000_000, -5, 3]], dtype=torch.int32, device="cuda")
    ctx = torch.tensor([64], dtype=torch.int32, device="cuda")
    q = torch.from_numpy(rng.standard_normal((1, hq, hd), dtype=np.float32)).cuda()
    out = paged_attention_batched(q, k, v, pt, ctx, hkv, ps, 4, hkv * ps * hd, hd, ps * hd, 0.125, 64)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    # equals attention over the two valid pages only
    valid = torch.tensor([[0, 3]], dtype=torch.int32, device="cuda")
    ref = paged_attention_batched(q, k, v, valid, torch.tensor([32], dtype=torch.int32, device="cuda"), hkv, ps, 4,
                                  hkv * ps * hd, hd, ps * hd, 0.125, 32)
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= TOL
