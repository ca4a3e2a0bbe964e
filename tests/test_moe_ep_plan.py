"""Expert-parallel dispatch on CPU ranks (gloo, world sizes 2 and 4): the exchange plan zcu_moe_forward follows,
driven through the library's host-only zcu_moe_ep_plan, with real all-to-all exchanges between processes.

Each rank routes its own tokens (SelectTopK of SparseMoeLayer.cs:159-182: repeated arg-max with a strict '>', so
ties keep the lowest expert), sends its (token, slot) rows in expert order to the experts' ranks after an
all-gather of the per-expert counts, reorders what it received into the [local expert][source] order the expert
GEMMs read, "runs" the experts (a tag transform that names the expert), and returns the results along the same
routes.  Checked: send and receive sizes, that every received row belongs to one of the rank's experts and sits
in its expert's contiguous block in source order, and that each rank gets back exactly the results of its own
rows, in its own expert order.  No GPU is involved.
"""
import ctypes
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _select_top_k(logits, k):
    """SelectTopK: k rounds of arg-max over the experts not yet picked, strict '>' (ties keep the lowest index)."""
    picked = np.zeros(logits.shape[0], bool)
    out = []
    for _ in range(k):
        best, bi = -np.inf, 0
        for j, v in enumerate(logits):
            if not picked[j] and v > best:
                best, bi = v, j
        picked[bi] = True
        out.append(bi)
    return out


def _tag(src, token, slot, expert):
    return ((src * 100000 + token) * 16 + slot) * 1000 + expert


def _worker(rank, world, port, n_experts, top_k, tokens, ties, errs):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        from zeroplatform_b200 import _lib
        L = _lib.lib()
        rng = np.random.default_rng(1000 + rank)
        T = tokens + rank  # ranks route different numbers of tokens
        logits = rng.standard_normal((T, n_experts)).astype(np.float32)
        if ties:  # many equal logits: the lowest expert index must win
            logits = np.round(logits).astype(np.float32)
        sel = [_select_top_k(logits[t], top_k) for t in range(T)]
        pairs = sorted((e, t, s) for t in range(T) for s, e in enumerate(sel[t]))  # expert order
        cnt = np.bincount([p[0] for p in pairs], minlength=n_experts).astype(np.int32)
        gathered = [torch.zeros(n_experts, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(cnt))
        counts_all = np.ascontiguousarray(torch.stack(gathered).numpy())
        epr = n_experts // world
        send_rows = np.zeros(world, np.int32)
        recv_rows = np.zeros(world, np.int32)
        recv_cnt = np.zeros((world, epr), np.int32)
        cap = int(counts_all[:, rank * epr:(rank + 1) * epr].sum())
        perm = np.zeros(max(cap, 1), np.int32)
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        total = L.zcu_moe_ep_plan(n_experts, world, rank, p(counts_all), p(send_rows), p(recv_rows), p(recv_cnt),
                                  p(perm), cap)
        assert total == cap, (total, cap)
        if cap > 0:
            assert L.zcu_moe_ep_plan(n_experts, world, rank, p(counts_all), None, None, None, p(perm), cap - 1) == -6
        for q in range(world):
            assert send_rows[q] == cnt[q * epr:(q + 1) * epr].sum()
            assert recv_rows[q] == counts_all[q, rank * epr:(rank + 1) * epr].sum()
            assert np.array_equal(recv_cnt[q], counts_all[q, rank * epr:(rank + 1) * epr])
        # dispatch: rows tagged (source rank, token, slot, expert), this rank's rows in expert order
        send = torch.tensor([[rank, t, s, e] for (e, t, s) in pairs], dtype=torch.int64).reshape(-1, 4)
        recv = torch.empty((total, 4), dtype=torch.int64)
        dist.all_to_all_single(recv, send, output_split_sizes=recv_rows.tolist(), input_split_sizes=send_rows.tolist())
        # the expert-contiguous order: received row i goes to position perm[i]
        order = torch.empty_like(recv)
        order[torch.from_numpy(perm[:total].astype(np.int64))] = recv
        o = order.numpy()
        base = 0
        for le in range(epr):
            n = int(recv_cnt[:, le].sum())
            blk = o[base:base + n]
            assert np.all(blk[:, 3] == rank * epr + le)  # one expert's rows, contiguous
            assert np.all(np.diff(blk[:, 0]) >= 0)      # by source rank
            base += n
        assert base == total
        # experts run: the result of a row names its source, token, slot and the expert that processed it
        out = torch.tensor([_tag(int(r[0]), int(r[1]), int(r[2]), int(r[3])) for r in o], dtype=torch.int64)
        back_send = out[torch.from_numpy(perm[:total].astype(np.int64))]  # back to arrival order
        back = torch.empty(len(pairs), dtype=torch.int64)
        dist.all_to_all_single(back, back_send, output_split_sizes=send_rows.tolist(),
                               input_split_sizes=recv_rows.tolist())
        want = [_tag(rank, t, s, e) for (e, t, s) in pairs]
        assert back.tolist() == want
        dist.barrier()
        dist.destroy_process_group()
    except Exception as ex:  # reported to the parent process
        errs.put(f"rank {rank}: {type(ex).__name__}: {ex}")
        raise


@pytest.mark.parametrize("world,n_experts,top_k,tokens,ties", [(2, 8, 2, 37, False), (4, 8, 2, 64, False),
                                                                (4, 16, 4, 23, True), (2, 4, 1, 5, True)])
def test_expert_parallel_dispatch_plan_on_cpu_ranks(world, n_experts, top_k, tokens, ties):
    ctx = mp.get_context("spawn")
    errs = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_experts, top_k, tokens, ties, errs))
             for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
    alive = [pr for pr in procs if pr.is_alive()]
    for pr in alive:
        pr.kill()
    msgs = []
    while not errs.empty():
        msgs.append(errs.get())
    assert not alive, "a rank did not finish"
    assert not msgs, msgs
    assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]


def test_plan_rejects_bad_arguments():
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    counts = np.ones((2, 6), np.int32)
    p = counts.ctypes.data_as(ctypes.c_void_p)
    assert L.zcu_moe_ep_plan(6, 4, 0, p, None, None, None, None, 0) == -2   # 6 experts over 4 ranks
    assert L.zcu_moe_ep_plan(6, 2, 2, p, None, None, None, None, 0) == -2   # rank out of range
    neg = -counts
    assert L.zcu_moe_ep_plan(6, 2, 0, neg.ctypes.data_as(ctypes.c_void_p), None, None, None, None, 0) == -2
    assert L.zcu_moe_ep_plan(6, 2, 0, p, None, None, None, None, 0) == -6  # no room for the permutation
