"""SparseMoeLayer mirror over the device MoE layer in libzero_tensor.so (zcu_moe_*).

Follows ZeroLlm's SparseMoeLayer.Forward (ZeroLlm/src/ZeroLlm.Core/Layers/SparseMoeLayer.cs:32-125) for a batch
of tokens: top-k routing with softmax over the selected logits, SwiGLU experts with Q4_0 / Q8_0 weights, and the
weighted residual add.  With ep_size > 1 every rank constructs the layer with the same configuration (a
collective), owns n_experts / ep_size experts and passes its own tokens to forward().
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import MoeConfig, ZcError, lib

WHICH = {"gate": 0, "up": 1, "down": 2}


def _ptr_nbytes(arr):
    if hasattr(arr, "data_ptr"):
        if not arr.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return arr.data_ptr(), arr.numel() * arr.element_size(), arr
    a = np.ascontiguousarray(arr)
    return a.ctypes.data, a.nbytes, a


class SparseMoeLayer:
    def __init__(self, n_experts: int, top_k: int, dim: int, ffn: int, qtype: int = 4, max_tokens: int = 256,
                 ep_size: int = 1, ep_rank: int = 0, nccl_id: bytes | None = None, stream=None):
        cfg = MoeConfig(n_experts, top_k, dim, ffn, qtype, max_tokens)
        self.cfg, self.ep_size, self.ep_rank = cfg, ep_size, ep_rank
        idbuf = None
        if ep_size > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("ep_size > 1 needs the 128-byte NCCL unique id of rank 0")
            idbuf = (C.c_uint8 * 128).from_buffer_copy(bytes(nccl_id))
        h = C.c_void_p()
        rc = lib().zcu_moe_create(C.byref(cfg), ep_size, ep_rank, idbuf, stream, C.byref(h))
        if rc != 0:
            raise ZcError(f"zcu_moe_create failed: {rc} {lib().zc_cuda_last_error().decode(errors='replace')}")
        self._h = h

    def last_error(self) -> str:
        return lib().zcu_moe_last_error(self._h).decode(errors="replace")

    def _check(self, rc, what):
        if rc != 0:
            raise ZcError(f"{what} failed: {rc} {self.last_error()}")

    def set_expert(self, expert: int, which, blocks):
        """The reference's packed Q4_0 / Q8_0 blocks of one projection (host or device memory)."""
        ptr, nbytes, _keep = _ptr_nbytes(blocks)
        w = WHICH[which] if isinstance(which, str) else int(which)
        self._check(lib().zcu_moe_set_expert(self._h, expert, w, ptr, nbytes), f"set_expert({expert}, {which})")

    def set_router(self, w):
        ptr, nbytes, _keep = _ptr_nbytes(w)
        self._check(lib().zcu_moe_set_router(self._h, ptr, nbytes), "set_router")

    def forward(self, xnorm, residual, router_logits=None):
        """xnorm, residual (updated in place) and router_logits are torch CUDA tensors; returns the routing
        (expert ids [T][top_k], weights [T][top_k]) as numpy arrays."""
        T = int(xnorm.shape[0]) if xnorm.dim() > 1 else 1
        k = self.cfg.top_k
        idx = np.empty((T, k), dtype=np.int32)
        wts = np.empty((T, k), dtype=np.float32)
        rl = router_logits.data_ptr() if router_logits is not None else None
        self._check(lib().zcu_moe_forward(self._h, xnorm.data_ptr(), rl, residual.data_ptr(), T, idx.ctypes.data,
                                          wts.ctypes.data), "forward")
        return idx, wts

    def close(self):
        if getattr(self, "_h", None):
            lib().zcu_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
