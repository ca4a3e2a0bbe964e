"""Tensor-parallel host logic on CPU: the shard plan (zcu_tp_plan), the NCCL unique-id hand-off over a
torch.distributed group (gloo ranks here), and the algebra the engine relies on -- row-split Wq|Wk|Wv and
Wgate|Wup, column-split Wo / Wdown on 32-block boundaries, whose per-rank partial products sum to the full
MatVecMulQ8_0 (QuantizedKernels.cs:190-226) result.  No GPU is used: zcu_tp_plan and zcu_nccl_unique_id are
host functions of libzero_tensor.so.
"""
import json
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

SEVEN_B = dict(vocab=32000, dim=4096, layers=32, heads=32, kv_heads=32, ffn=11008)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, model, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from zeroplatform_b200.engine import broadcast_unique_id, make_config, tp_plan
        uid = broadcast_unique_id(rank)
        plan = tp_plan(make_config(model), world, rank)
        got = [None] * world
        dist.all_gather_object(got, (plan, uid.hex()))
        if rank == 0:
            with open(os.path.join(out_dir, "plans.json"), "w") as f:
                json.dump(got, f)
    finally:
        dist.destroy_process_group()


def _tiles(plans, begin, count, total, multiple=1):
    pos = 0
    for p in plans:
        assert p[begin] == pos, (begin, plans)
        assert p[count] > 0 and p[count] % multiple == 0
        pos += p[count]
    assert pos == total


@pytest.mark.parametrize("world,model", [(2, SEVEN_B), (4, SEVEN_B), (8, SEVEN_B),
                                         (2, dict(vocab=1001, dim=256, layers=2, heads=8, kv_heads=4, ffn=544))])
def test_plan_tiles_the_model_and_every_rank_gets_rank0s_nccl_id(world, model):
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, port, model, d), nprocs=world, join=True, start_method="spawn")
        with open(os.path.join(d, "plans.json")) as f:
            got = json.load(f)
    plans = [p for p, _ in got]
    ids = {u for _, u in got}
    assert len(ids) == 1 and len(bytes.fromhex(ids.pop())) == 128
    _tiles(plans, "head_begin", "heads", model["heads"])
    _tiles(plans, "kv_head_begin", "kv_heads", model["kv_heads"])
    _tiles(plans, "ffn_begin", "ffn", model["ffn"], multiple=32)
    _tiles(plans, "vocab_begin", "vocab", model["vocab"])
    hd = model["dim"] // model["heads"]
    for p in plans:  # GQA groups stay whole on a rank; Wo column slices are whole 32-blocks
        assert p["heads"] * model["kv_heads"] == p["kv_heads"] * model["heads"]
        assert (p["heads"] * hd) % 32 == 0 and (p["head_begin"] * hd) % 32 == 0


def test_plan_rejects_unsplittable_models():
    from zeroplatform_b200 import _lib
    from zeroplatform_b200.engine import make_config, tp_plan
    with pytest.raises(_lib.ZcError):   # 2 K/V heads over 4 ranks
        tp_plan(make_config(dict(vocab=100, dim=256, layers=1, heads=8, kv_heads=2, ffn=512)), 4, 0)
    with pytest.raises(_lib.ZcError):   # a rank's Wo slice of 1 head x 8 dims is not a 32-block
        tp_plan(make_config(dict(vocab=100, dim=64, layers=1, heads=8, kv_heads=8, ffn=512)), 8, 0)
    with pytest.raises(_lib.ZcError):   # 2 FFN blocks over 4 ranks
        tp_plan(make_config(dict(vocab=100, dim=256, layers=1, heads=4, kv_heads=4, ffn=64)), 4, 0)


def test_column_split_partials_sum_to_the_full_matvec():
    """sum over ranks of MatVec(W[:, slice_r], x[slice_r]) == MatVec(W, x) within fp32 summation order, for
    the Wdown slices the plan gives (uneven 32-block split)."""
    from zeroplatform_b200.engine import make_config, tp_plan
    model = dict(vocab=1001, dim=256, layers=2, heads=8, kv_heads=4, ffn=544)
    rng = np.random.default_rng(3)
    n, k = model["dim"], model["ffn"]
    blocks = O.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).reshape(n, k // 32, 34)
    x = rng.standard_normal(k, dtype=np.float32)
    full = O.matvec(8, blocks.reshape(-1), x, n, k)
    acc = np.zeros(n, np.float64)
    cfg = make_config(model)
    for r in range(2):
        p = tp_plan(cfg, 2, r)
        b0, nb = p["ffn_begin"] // 32, p["ffn"] // 32
        part = np.ascontiguousarray(blocks[:, b0:b0 + nb, :]).reshape(-1)
        acc += O.matvec(8, part, x[p["ffn_begin"]:p["ffn_begin"] + p["ffn"]], n, p["ffn"])
    assert np.max(np.abs(acc - full)) / np.max(np.abs(full)) < 1e-6
