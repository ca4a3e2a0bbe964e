"""The C-ABI library loads and exports every symbol include/*.h declares (no compute on CPU)."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

from tests.conftest import ROOT


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        for m in re.finditer(r"^ZC_API\s+[\w\s\*]+?\b(zcu?_\w+)\s*\(", open(h).read(), re.M):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_reference_bridge_set():
    names = set(declared_symbols())
    # ZeroTensorNativeBridge.Initialize requires these six (ZeroTensorNativeBridge.cs:144-157)
    for required in ["zc_version", "zc_is_simd_supported", "zc_gemm_f32", "zc_flash_attention_f32",
                     "zc_gemv_q4_0", "zc_gemv_q8_0"]:
        assert required in names
    for optional in ["zc_paged_attention_f32", "zc_dot_i8", "zc_rmsnorm_f32", "zc_swiglu_f32", "zc_silu_f32",
                     "zc_rope_f32"]:
        assert optional in names


def test_library_exports_every_declared_symbol():
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes signature table"
    assert L.zc_version() == 0x000100


def test_no_silent_cpu_fallback_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    assert L.zc_is_simd_supported() == 0
    x = (ctypes.c_float * 32)(*([1.0] * 32))
    y = (ctypes.c_float * 1)()
    w = (ctypes.c_uint8 * 34)()
    rc = L.zc_gemv_q8_0(ctypes.addressof(w), ctypes.addressof(x), ctypes.addressof(y), 1, 32)
    assert rc != 0  # not handled: the C# caller runs its managed path; the library itself never computes on CPU
    assert L.zc_cuda_last_error()


def test_bad_arguments_are_refused_before_any_device_work():
    """The bridge entries validate their arguments on the host first (non-zero = the C# caller runs its managed
    path): a k that is not a whole number of 32-blocks, null buffers, tensor types other than Q8_0 / Q4_0."""
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    x = (ctypes.c_float * 48)()
    y = (ctypes.c_float * 1)()
    w = (ctypes.c_uint8 * 64)()
    assert L.zc_gemv_q8_0(ctypes.addressof(w), ctypes.addressof(x), ctypes.addressof(y), 1, 48) == -2
    assert b"k_cols" in L.zc_cuda_last_error()
    assert L.zc_gemv_q4_0(None, ctypes.addressof(x), ctypes.addressof(y), 1, 32) == -2
    assert L.zc_register_weights(0, ctypes.addressof(w), 1, 32) == -4   # F32 tensors are not registered
    assert L.zc_register_weights(8, ctypes.addressof(w), 1, 48) == -2   # not a whole number of blocks


def test_paged_attention_shapes_are_checked_before_any_device_work():
    """Both device attention entries reject an impossible shape on the host before choosing a split count or
    touching scratch: hkv == 0 (no division by zero), hq not a multiple of hkv, a non-positive page size or head
    size (-2), and a head size the kernel has no form for (-4)."""
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    buf = (ctypes.c_float * 64)()
    p = ctypes.addressof(buf)  # never dereferenced: every call below is refused first

    def call(fn, hq=8, hkv=2, hd=64, page_size=16, max_pages=4, batch=1):
        return fn(p, p, p, 1, p, p, p, batch, hq, hkv, hd, page_size, max_pages, 8, hkv * page_size * hd, hd,
                  page_size * hd, 0.125, 64, None)

    for fn in (L.zcu_paged_attention, L.zcu_paged_attention_noalloc):
        assert call(fn, hkv=0) == -2
        assert call(fn, hq=6, hkv=4) == -2
        assert call(fn, page_size=0) == -2
        assert call(fn, hd=0) == -2
        assert call(fn, hd=-64) == -2
        assert call(fn, max_pages=0) == -2
        assert call(fn, hd=48) == -4
        assert L.zc_cuda_last_error()


def test_sampler_draw_is_splitmix64():
    """zcu_sample_uniform(seed, i) = the top 24 bits of SplitMix64(seed + i) over 2^24 (the sampled generation's
    i-th draw), restated here in Python; the sampler refuses a null config or a negative Top-K on the host."""
    from zeroplatform_b200 import _lib
    L = _lib.lib()
    M = (1 << 64) - 1

    def splitmix(x):
        z = (x + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        z ^= z >> 31
        return (z >> 40) / float(1 << 24)

    for seed, i in [(0, 0), (1234567, 5), (2 ** 63 + 11, 999), (42, 2 ** 40)]:
        assert L.zcu_sample_uniform(seed, i) == splitmix((seed + i) & M)
    us = [L.zcu_sample_uniform(7, i) for i in range(4000)]
    assert 0.0 <= min(us) and max(us) < 1.0 and abs(float(np.mean(us)) - 0.5) < 0.02
    from zeroplatform_b200._lib import SamplingConfig
    buf = (ctypes.c_float * 8)()
    p = ctypes.addressof(buf)
    assert L.zcu_sample(p, 1, 8, None, None, 0, None, p, p, None, None, None, 0, None) == -2
    bad = SamplingConfig(1.0, 0.9, 0.0, -1, 1.0)
    assert L.zcu_sample(p, 1, 8, None, None, 0, ctypes.byref(bad), p, p, None, None, None, 0, None) == -2
