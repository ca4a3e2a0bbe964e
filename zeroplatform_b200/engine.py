"""LlmEngine mirror over the device decode engine in libzero_tensor.so (zcu_engine_*).

Follows ZeroLlm's LlmEngine (ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs): `prefill` is PrefillPrompt
(:157-315), `forward_token` is ForwardToken (:347-461), `generate_greedy` is GenerateStreamAsync with greedy
sampling (:71-150).  Models are dictionaries of the reference's tensors: Q8_0 packed blocks (uint8) for
tok_emb, lm_head and the per-layer projections stacked over layers ([L, rows, cols/32*34]), fp32 norms.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import EngineConfig, ZcError, lib

KINDS = {"tok_emb": 0, "lm_head": 1, "final_norm": 2, "attn_norm": 3, "ffn_norm": 4, "wq": 5, "wk": 6, "wv": 7,
         "wo": 8, "wgate": 9, "wup": 10, "wdown": 11}


class LlmEngine:
    def __init__(self, model: dict, total_pages=256, page_size=16, max_batch=4, max_pages_per_seq=None,
                 max_prefill_tokens=1024, reference_causal_quirk=True, stream=None):
        self.model = model
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
        self.cfg = cfg
        h = C.c_void_p()
        rc = lib().zcu_engine_create(C.byref(cfg), stream, C.byref(h))
        if rc != 0:
            raise ZcError(f"zcu_engine_create failed: {rc}")
        self._h = h
        for name, kind in KINDS.items():
            arr = model[name]
            if name in ("tok_emb", "lm_head", "final_norm"):
                self._set(kind, 0, arr)
            else:
                for layer in range(cfg.layers):
                    self._set(kind, layer, arr[layer])

    def _set(self, kind, layer, arr):
        a = np.ascontiguousarray(arr)
        rc = lib().zcu_engine_set_weight(self._h, kind, layer, a.ctypes.data, a.nbytes)
        if rc != 0:
            raise ZcError(f"zcu_engine_set_weight({kind}, {layer}) failed: {rc} {self.last_error()}")

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

    def get_kv(self, seq_id: int, layer: int, token: int, value: bool = False) -> np.ndarray:
        out = np.empty(self.cfg.kv_heads * (self.cfg.dim // self.cfg.heads), dtype=np.float32)
        self._check(lib().zcu_engine_get_kv(self._h, seq_id, layer, token, int(value), out.ctypes.data), "get_kv")
        return out
