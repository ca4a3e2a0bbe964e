"""ctypes binding of libzero_tensor.so (the in-tree CUDA library).

Loading fails loudly when the library has not been built: there is no CPU or
PyTorch fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libzero_tensor.so")
_lib = None

sz = C.c_size_t
i32 = C.c_int32
i64 = C.c_int64
vp = C.c_void_p
f32 = C.c_float

# Every exported symbol with its C signature (include/zero_tensor.h, include/zero_tensor_cuda.h).
SIGNATURES = {
    # reference bridge ABI (host pointers)
    "zc_version": (C.c_uint32, []),
    "zc_is_simd_supported": (i32, []),
    "zc_gemm_f32": (i32, [sz, sz, sz, f32, vp, C.c_ssize_t, C.c_ssize_t, vp, C.c_ssize_t, C.c_ssize_t, f32, vp,
                          C.c_ssize_t, C.c_ssize_t, i32]),
    "zc_flash_attention_f32": (i32, [sz, sz, sz, sz, sz, f32, i32, sz, sz, sz, vp, vp, vp, vp, vp]),
    "zc_gemv_q4_0": (i32, [vp, vp, vp, sz, sz]),
    "zc_gemv_q8_0": (i32, [vp, vp, vp, sz, sz]),
    "zc_rmsnorm_f32": (i32, [sz, vp, vp, vp, f32]),
    "zc_silu_f32": (i32, [sz, vp, vp]),
    "zc_swiglu_f32": (i32, [sz, vp, vp, vp]),
    "zc_rope_f32": (i32, [sz, sz, sz, sz, f32, vp]),
    "zc_paged_attention_f32": (i32, [sz, sz, sz, sz, sz, f32, vp, vp, vp, vp, vp]),
    "zc_dot_i8": (i32, [sz, vp, vp, vp]),
    "zc_register_weights": (i32, [i32, vp, sz, sz]),
    "zc_unregister_weights": (i32, [vp]),
    "zc_cuda_last_error": (C.c_char_p, []),
    # device-pointer extension
    "zcu_quantize_q8_0": (i32, [vp, vp, sz, vp]),
    "zcu_quantize_q4_0": (i32, [vp, vp, sz, vp]),
    "zcu_q8_0_repack": (i32, [vp, vp, vp, sz, sz, vp]),
    "zcu_q4_0_repack": (i32, [vp, vp, vp, sz, sz, vp]),
    "zcu_gemv_q8_0": (i32, [vp, vp, vp, vp, sz, sz, i32, vp]),
    "zcu_gemv_q4_0": (i32, [vp, vp, vp, vp, sz, sz, i32, vp]),
    "zcu_gemm_q8_0": (i32, [vp, vp, vp, vp, sz, sz, sz, i32, vp]),
    "zcu_gemm_q4_0": (i32, [vp, vp, vp, vp, sz, sz, sz, i32, vp]),
    "zcu_device_status": (i32, [i32]),
    "zcu_paged_attention": (i32, [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i64, i64, i64,
                                  f32, i32, vp]),
    "zcu_paged_attention_noalloc": (i32, [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i64, i64,
                                          i64, f32, i32, vp]),
    "zcu_rmsnorm": (i32, [vp, vp, vp, i32, i32, f32, vp]),
    "zcu_swiglu": (i32, [vp, vp, vp, sz, vp]),
    "zcu_rope": (i32, [vp, i32, i32, i32, vp, i32, vp, vp, i32, vp]),
    "zcu_embed_q8_0": (i32, [vp, vp, vp, i32, i32, i32, vp, vp]),
}


class EngineConfig(C.Structure):
    """zcu_engine_config (include/zero_tensor_cuda.h)."""

    _fields_ = [(n, C.c_int32) for n in ("vocab", "dim", "layers", "heads", "kv_heads", "ffn", "context_length")] + \
        [("eps", C.c_float), ("rope_base", C.c_float)] + \
        [(n, C.c_int32) for n in ("total_pages", "page_size", "max_batch", "max_pages_per_seq", "max_prefill_tokens",
                                  "reference_causal_quirk")]


SIGNATURES.update({
    "zcu_engine_create": (i32, [C.POINTER(EngineConfig), vp, C.POINTER(vp)]),
    "zcu_engine_destroy": (i32, [vp]),
    "zcu_engine_last_error": (C.c_char_p, [vp]),
    "zcu_engine_set_weight": (i32, [vp, i32, i32, vp, sz]),
    "zcu_engine_prefill": (i32, [vp, i32, vp, i32, i32, vp]),
    "zcu_engine_decode": (i32, [vp, vp, vp, vp, i32, vp, vp]),
    "zcu_engine_generate": (i32, [vp, i32, vp, i32, i32, f32, i32, vp, vp]),
    "zcu_engine_free_sequence": (i32, [vp, i32]),
    "zcu_engine_seq_len": (i32, [vp, i32]),
    "zcu_engine_free_pages": (i32, [vp]),
    "zcu_engine_page_table": (i32, [vp, i32, vp, i32]),
    "zcu_engine_get_kv": (i32, [vp, i32, i32, i32, i32, vp]),
    "zcu_engine_append_kv": (i32, [vp, i32, i32, i32, i32, vp, vp, i32]),
    "zcu_engine_generate_batch": (i32, [vp, i32, vp, vp, i32, vp, vp]),
    "zcu_nccl_unique_id": (i32, [vp, sz]),
})


class SamplingConfig(C.Structure):
    """zcu_sampling_config (include/zero_tensor_cuda.h): SamplingConfig's numeric fields."""

    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("min_p", C.c_float), ("top_k", C.c_int32),
                ("repetition_penalty", C.c_float)]


class TpShard(C.Structure):
    """zcu_tp_shard (include/zero_tensor_cuda.h): one rank's slice of a tensor-parallel model."""

    _fields_ = [(n, C.c_int32) for n in ("head_begin", "heads", "kv_head_begin", "kv_heads", "ffn_begin", "ffn",
                                         "vocab_begin", "vocab")]

    def as_dict(self):
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


SIGNATURES.update({
    "zcu_tp_plan": (i32, [C.POINTER(EngineConfig), i32, i32, C.POINTER(TpShard)]),
    "zcu_engine_create_tp": (i32, [C.POINTER(EngineConfig), i32, i32, vp, vp, C.POINTER(vp)]),
})


class MoeConfig(C.Structure):
    """zcu_moe_config (include/zero_tensor_cuda.h)."""

    _fields_ = [(n, C.c_int32) for n in ("n_experts", "top_k", "dim", "ffn", "qtype", "max_tokens")]


SIGNATURES.update({
    "zcu_moe_create": (i32, [C.POINTER(MoeConfig), i32, i32, vp, vp, C.POINTER(vp)]),
    "zcu_moe_destroy": (i32, [vp]),
    "zcu_moe_last_error": (C.c_char_p, [vp]),
    "zcu_moe_set_expert": (i32, [vp, i32, i32, vp, sz]),
    "zcu_moe_set_router": (i32, [vp, vp, sz]),
    "zcu_moe_forward": (i32, [vp, vp, vp, vp, i32, vp, vp]),
    "zcu_moe_ep_plan": (i32, [i32, i32, i32, vp, vp, vp, vp, vp, i32]),
    "zcu_peer_wait_selftest": (i32, [i32, i32, vp]),
    "zcu_engine_step_kind": (i32, [vp, vp, i32]),
    "zcu_sample": (i32, [vp, i32, i32, vp, vp, i32, C.POINTER(SamplingConfig), vp, vp, vp, vp, vp, i32, vp]),
    "zcu_sample_uniform": (C.c_float, [C.c_uint64, C.c_uint64]),
    "zcu_engine_generate_sampled": (i32, [vp, i32, vp, i32, i32, C.POINTER(SamplingConfig), C.c_uint64, i32, vp,
                                          vp]),
})


class ServeEvent(C.Structure):
    """zcu_serve_event (include/zero_tensor_cuda.h)."""

    _fields_ = [(n, C.c_int32) for n in ("seq_id", "token", "finished", "reason")]


SERVE_RUNNING, SERVE_STOP_TOKEN, SERVE_MAX_TOKENS, SERVE_CANCELLED, SERVE_REFUSED = range(5)

SIGNATURES.update({
    "zcu_engine_submit": (i32, [vp, i32, vp, i32, i32, C.POINTER(SamplingConfig), C.c_uint64, i32, vp, i32]),
    "zcu_engine_serve_step": (i32, [vp, C.POINTER(ServeEvent), i32]),
    "zcu_engine_cancel": (i32, [vp, i32]),
    "zcu_engine_serve_counts": (i32, [vp, C.POINTER(i32), C.POINTER(i32)]),
})


class ZcError(RuntimeError):
    pass


def lib():
    """Load libzero_tensor.so (raises when it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ZcError(f"{LIB_PATH} is not built; run `python -m zeroplatform_b200.build` "
                      "(this package has no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().zc_cuda_last_error().decode(errors="replace")
        raise ZcError(f"{what} failed with status {rc}: {msg}")
