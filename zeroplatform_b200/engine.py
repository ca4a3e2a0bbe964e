"""LlmEngine mirror over the device decode engine in libzero_tensor.so (zcu_engine_*).

Follows ZeroLlm's LlmEngine (ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs): `prefill` is PrefillPrompt
(:157-315), `forward_token` is ForwardToken (:347-461), `generate_greedy` is GenerateStreamAsync with greedy
sampling (:71-150).  Models are dictionaries of the reference's tensors: Q8_0 packed blocks (uint8) for
tok_emb, lm_head and the per-layer projections stacked over layers ([L, rows, cols/32*34]), fp32 norms.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import EngineConfig, TpShard, ZcError, lib

KINDS = {"tok_emb": 0, "lm_head": 1, "final_norm": 2, "attn_norm": 3, "ffn_norm": 4, "wq": 5, "wk": 6, "wv": 7,
         "wo": 8, "wgate": 9, "wup": 10, "wdown": 11}


def _ptr_nbytes(arr):
    """(address, bytes) of a contiguous numpy array or torch tensor (host or device memory)."""
    if hasattr(arr, "data_ptr"):
        if not arr.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return arr.data_ptr(), arr.numel() * arr.element_size(), arr
    a = np.ascontiguousarray(arr)
    return a.ctypes.data, a.nbytes, a


def make_config(model: dict, total_pages=256, page_size=16, max_batch=4, max_pages_per_seq=None,
                max_prefill_tokens=1024, reference_causal_quirk=True) -> EngineConfig:
    cfg = EngineConfig()
    for k in ("vocab", "dim", "layers", "heads", "kv_heads", "ffn"):
        setattr(cfg, k, int(model[k]))
    cfg.context_length = int(model.get("context_length", 2048))
    cfg.eps = float(model.get("eps", 1e-5))
    cfg.rope_base = float(model.get("rope_base", 10000.0))
    cfg.total_pages = total_pages
    cfg.page_size = page_size
    cfg.max_batch = max_batch
    cfg.max_pages_per_seq = max_pages_per_seq or total_pages
    cfg.max_prefill_tokens = max_prefill_tokens
    cfg.reference_causal_quirk = int(bool(reference_causal_quirk))
    return cfg


class LlmEngine:
    """One engine per GPU.  With tp_size > 1 every rank constructs its engine with the same model and its own
    tp_rank (a collective: all ranks must construct together) and then makes the same calls in the same order.
    `model` holds the shapes and, unless load=False, every tensor (numpy arrays or torch tensors on the host
    or the device; each rank is given the FULL tensors and keeps its slice)."""

    def __init__(self, model: dict, total_pages=256, page_size=16, max_batch=4, max_pages_per_seq=None,
                 max_prefill_tokens=1024, reference_causal_quirk=True, stream=None, tp_size=1, tp_rank=0,
                 nccl_id: bytes | None = None, load=True):
        self.model = model
        cfg = make_config(model, total_pages, page_size, max_batch, max_pages_per_seq, max_prefill_tokens,
                          reference_causal_quirk)
        self.cfg = cfg
        self.tp_size, self.tp_rank = tp_size, tp_rank
        h = C.c_void_p()
        idbuf = None
        if tp_size > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("tp_size > 1 needs the 128-byte NCCL unique id of rank 0")
            idbuf = (C.c_uint8 * 128).from_buffer_copy(bytes(nccl_id))
        rc = lib().zcu_engine_create_tp(C.byref(cfg), tp_size, tp_rank, idbuf, stream, C.byref(h))
        if rc != 0:
            raise ZcError(f"zcu_engine_create_tp failed: {rc} {lib().zc_cuda_last_error().decode(errors='replace')}")
        self._h = h
        if load:
            for name in KINDS:
                arr = model[name]
                if name in ("tok_emb", "lm_head", "final_norm"):
                    self.set_weight(name, 0, arr)
                else:
                    for layer in range(cfg.layers):
                        self.set_weight(name, layer, arr[layer])

    def shard(self) -> dict:
        return tp_plan(self.cfg, self.tp_size, self.tp_rank)

    def set_weight(self, name, layer, arr):
        kind = KINDS[name] if isinstance(name, str) else int(name)
        ptr, nbytes, _keep = _ptr_nbytes(arr)
        rc = lib().zcu_engine_set_weight(self._h, kind, layer, ptr, nbytes)
        if rc != 0:
            raise ZcError(f"zcu_engine_set_weight({name}, {layer}) failed: {rc} {self.last_error()}")

    _set = set_weight

    def last_error(self) -> str:
        return lib().zcu_engine_last_error(self._h).decode(errors="replace")

    def close(self):
        if getattr(self, "_h", None):
            lib().zcu_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc, what):
        if rc < 0:
            raise ZcError(f"{what} failed: {rc} {self.last_error()}")
        return rc

    def prefill(self, seq_id: int, tokens, start_pos: int = 0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.cfg.vocab, dtype=np.float32)
        self._check(lib().zcu_engine_prefill(self._h, seq_id, t.ctypes.data, t.size, start_pos, logits.ctypes.data),
                    "prefill")
        return logits

    def forward_token(self, seq_id: int, token: int, pos: int) -> np.ndarray:
        return self.decode([seq_id], [token], [pos])[0]

    def decode(self, seq_ids, tokens, positions, want_logits=True):
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        b = s.size
        logits = np.empty((b, self.cfg.vocab), dtype=np.float32) if want_logits else None
        nxt = np.empty(b, dtype=np.int32)
        self._check(lib().zcu_engine_decode(self._h, s.ctypes.data, t.ctypes.data, p.ctypes.data, b,
                                            logits.ctypes.data if want_logits else None, nxt.ctypes.data), "decode")
        return logits if want_logits else nxt

    def generate_greedy(self, seq_id: int, prompt, n_new: int, repetition_penalty: float = 1.0, eos_token: int = -1):
        """Returns (generated tokens, prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max(n_new, 1), dtype=np.int32)
        timing = (C.c_float * 2)()
        n = self._check(lib().zcu_engine_generate(self._h, seq_id, p.ctypes.data, p.size, n_new, repetition_penalty,
                                                  eos_token, out.ctypes.data, timing), "generate")
        return out[:n].copy(), float(timing[0]), float(timing[1])

    def generate_sampled(self, seq_id: int, prompt, n_new: int, temperature=0.7, top_p=0.9, min_p=0.0, top_k=40,
                         repetition_penalty=1.1, seed=0, eos_token: int = -1):
        """GenerateStreamAsync with a SamplingConfig (defaults: SamplingConfig's), the sampler on the device; the i-th
        token's draw is zcu_sample_uniform(seed, i).  Returns (tokens, prefill_ms, decode_ms)."""
        from ._lib import SamplingConfig
        cfg = SamplingConfig(temperature, top_p, min_p, top_k, repetition_penalty)
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max(n_new, 1), dtype=np.int32)
        timing = (C.c_float * 2)()
        n = self._check(lib().zcu_engine_generate_sampled(self._h, seq_id, p.ctypes.data, p.size, n_new, C.byref(cfg),
                                                          seed, eos_token, out.ctypes.data, timing), "generate_sampled")
        return out[:n].copy(), float(timing[0]), float(timing[1])

    # ---- continuous batching (zcu_engine_submit / zcu_engine_serve_step) ----

    def submit(self, seq_id: int, prompt, max_new: int, temperature=0.7, top_p=0.9, min_p=0.0, top_k=40,
               repetition_penalty=1.1, seed=0, eos_token: int = -1, stop_tokens=()):
        """Queues one GenerateStreamAsync request (SamplingConfig's fields; MaxTokens = max_new); it runs in the
        following serve_step calls together with every other running request."""
        from ._lib import SamplingConfig
        cfg = SamplingConfig(temperature, top_p, min_p, top_k, repetition_penalty)
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        st = np.ascontiguousarray(sorted(set(int(t) for t in stop_tokens)), dtype=np.int32)
        self._check(lib().zcu_engine_submit(self._h, seq_id, p.ctypes.data, p.size, max_new, C.byref(cfg), seed,
                                            eos_token, st.ctypes.data if st.size else None, st.size), "submit")

    def serve_step(self):
        """One scheduler iteration; returns [(seq_id, token, finished, reason)] (reason: _lib.SERVE_*)."""
        from ._lib import ServeEvent
        if not hasattr(self, "_events"):
            self._events = (ServeEvent * (2 * self.cfg.max_batch + 4096))()
        n = self._check(lib().zcu_engine_serve_step(self._h, self._events, len(self._events)), "serve_step")
        return [(e.seq_id, e.token, e.finished, e.reason) for e in self._events[:n]]

    def cancel(self, seq_id: int):
        self._check(lib().zcu_engine_cancel(self._h, seq_id), "cancel")

    def serve_counts(self):
        """(running, queued) requests."""
        a, q = C.c_int32(), C.c_int32()
        lib().zcu_engine_serve_counts(self._h, C.byref(a), C.byref(q))
        return a.value, q.value

    def step_kind(self):
        """(1, "") when generation runs one cooperative kernel per token, (0, reason) for the per-operator graph,
        (-1, "") before the first generate call."""
        buf = C.create_string_buffer(256)
        k = lib().zcu_engine_step_kind(self._h, buf, 256)
        return k, buf.value.decode(errors="replace")

    def free_sequence(self, seq_id: int):
        lib().zcu_engine_free_sequence(self._h, seq_id)

    def seq_len(self, seq_id: int) -> int:
        return lib().zcu_engine_seq_len(self._h, seq_id)

    def free_pages(self) -> int:
        return lib().zcu_engine_free_pages(self._h)

    def page_table(self, seq_id: int):
        buf = np.empty(self.cfg.max_pages_per_seq, dtype=np.int32)
        n = lib().zcu_engine_page_table(self._h, seq_id, buf.ctypes.data, buf.size)
        return buf[:n].copy()

    def append_kv(self, seq_id: int, layer: int, start_pos: int, k, v):
        """PagedKvCache.AppendTokenAt for k, v [n][kv_heads][hd] (fp32 or fp16; numpy or torch, host or device)."""
        kp, kb, _k = _ptr_nbytes(k)
        vp_, vb, _v = _ptr_nbytes(v)
        esz = k.element_size() if hasattr(k, "element_size") else np.asarray(k).itemsize
        if kb != vb or esz not in (2, 4):
            raise ValueError("k and v must have the same size and be fp16 or fp32")
        row = self.cfg.kv_heads * (self.cfg.dim // self.cfg.heads) * esz
        self._check(lib().zcu_engine_append_kv(self._h, seq_id, layer, start_pos, kb // row, kp, vp_, int(esz == 2)),
                    "append_kv")

    def generate_batch(self, seq_ids, tokens, n_new: int):
        """Batched greedy generation; returns (tokens [batch][n_new], device ms of the n_new steps)."""
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((s.size, max(n_new, 1)), dtype=np.int32)
        timing = (C.c_float * 1)()
        self._check(lib().zcu_engine_generate_batch(self._h, s.size, s.ctypes.data, t.ctypes.data, n_new,
                                                    out.ctypes.data, timing), "generate_batch")
        return out[:, :n_new].copy(), float(timing[0])

    def get_kv(self, seq_id: int, layer: int, token: int, value: bool = False) -> np.ndarray:
        out = np.empty(self.cfg.kv_heads * (self.cfg.dim // self.cfg.heads), dtype=np.float32)
        self._check(lib().zcu_engine_get_kv(self._h, seq_id, layer, token, int(value), out.ctypes.data), "get_kv")
        return out


def tp_plan(cfg: EngineConfig, tp_size: int, tp_rank: int) -> dict:
    """zcu_tp_plan: the heads, K/V heads, FFN units and vocabulary rows rank tp_rank holds (host only)."""
    sh = TpShard()
    rc = lib().zcu_tp_plan(C.byref(cfg), tp_size, tp_rank, C.byref(sh))
    if rc != 0:
        raise ZcError(f"zcu_tp_plan(tp_size={tp_size}, rank={tp_rank}) failed: {rc}")
    return sh.as_dict()


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (rank 0 makes it; the others receive it out of band)."""
    buf = (C.c_uint8 * 128)()
    rc = lib().zcu_nccl_unique_id(buf, 128)
    if rc != 0:
        raise ZcError(f"zcu_nccl_unique_id failed: {rc} {lib().zc_cuda_last_error().decode(errors='replace')}")
    return bytes(buf)


def broadcast_unique_id(rank: int, group=None) -> bytes:
    """Rank 0's NCCL unique id on every rank of a torch.distributed group (any backend, gloo included)."""
    import torch.distributed as dist
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]
