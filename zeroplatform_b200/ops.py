"""Host-side mirror of the reference operators on the quantized-linear + paged-KV path.

Names and argument meaning follow the reference (kzxl/ZeroPlatform):

* ``QuantizedKernels.mat_vec_mul_q8_0 / mat_vec_add_q8_0 / ..._q4_0`` --
  ZeroLlm/src/ZeroLlm.Core/Quantization/QuantizedKernels.cs:190-349 (y = W x, y += W x)
* ``TensorBlas.gemv_q8_0 / gemv_q4_0`` -- ZeroTensor/src/ZeroTensor.Core/TensorBlas.Quantized.cs:447-485
  (host arrays in, host array out; goes through the reference bridge ABI ``zc_gemv_*``)
* ``TensorOps.paged_attention`` -- ZeroTensor/src/ZeroTensor.Core/TensorOps.Neural.cs:2372-2476
* ``QuantizedWeight`` -- a weight uploaded once and kept in the device layout (the repack of the
  reference's BlockQ8_0 / BlockQ4_0 arrays, BlockQ8_0.cs:10-17, BlockQ4_0.cs:10-17).

Device tensors are torch CUDA tensors (PyTorch provides the memory and the stream); every compute
call goes through libzero_tensor.so.  Errors raise ZcError (the C# bridge instead falls back to its
managed code on a non-zero status).
"""
from __future__ import annotations

import numpy as np
import torch

import ctypes as C

from ._lib import ZcError, check, lib

QK = 32
Q8_BYTES = 34
Q4_BYTES = 18


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _np_ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def quantize(qtype: int, w: torch.Tensor, stream=None) -> torch.Tensor:
    """LlmQuantizer.QuantizeToQ8_0 / QuantizeToQ4_0 on the device: fp32 [..., cols] -> packed AoS blocks
    (uint8 [..., cols/32*34] or [..., cols/32*18]), bit-identical to the reference quantizer."""
    w = w.contiguous()
    if w.dtype != torch.float32 or w.shape[-1] % QK:
        raise ZcError("quantize expects fp32 with a last dimension that is a multiple of 32")
    bpb = Q8_BYTES if qtype == 8 else Q4_BYTES
    out = torch.empty(w.shape[:-1] + (w.shape[-1] // QK * bpb,), dtype=torch.uint8, device=w.device)
    fn = lib().zcu_quantize_q8_0 if qtype == 8 else lib().zcu_quantize_q4_0
    check(fn(w.data_ptr(), out.data_ptr(), w.numel(), _stream(stream)), "quantize")
    return out


class QuantizedWeight:
    """A Q8_0 or Q4_0 weight matrix [rows][cols] resident on the GPU in the SoA layout."""

    def __init__(self, qtype: int, qs: torch.Tensor, d: torch.Tensor, rows: int, cols: int):
        self.qtype, self.qs, self.d, self.rows, self.cols = qtype, qs, d, rows, cols

    @staticmethod
    def upload(qtype: int, blocks, rows: int, cols: int, device="cuda", stream=None) -> "QuantizedWeight":
        """Upload the reference's packed blocks (numpy uint8 or a torch uint8 tensor) and repack."""
        if cols % QK:
            raise ZcError("cols must be a multiple of 32")
        bpb = Q8_BYTES if qtype == 8 else Q4_BYTES
        nbytes = rows * (cols // QK) * bpb
        if isinstance(blocks, np.ndarray):
            aos = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)[:nbytes]).to(device, non_blocking=False)
        else:
            aos = blocks.reshape(-1)[:nbytes].to(device).contiguous()
        if aos.numel() != nbytes:
            raise ZcError(f"expected {nbytes} bytes of blocks, got {aos.numel()}")
        if qtype == 8:
            qs = torch.empty((rows, cols), dtype=torch.int8, device=device)
            fn = lib().zcu_q8_0_repack
        else:
            qs = torch.empty((rows, cols // 2), dtype=torch.uint8, device=device)
            fn = lib().zcu_q4_0_repack
        d = torch.empty((rows, cols // QK), dtype=torch.int16, device=device)
        check(fn(aos.data_ptr(), qs.data_ptr(), d.data_ptr(), rows, cols, _stream(stream)), "repack")
        return QuantizedWeight(qtype, qs, d, rows, cols)

    @property
    def nbytes(self) -> int:
        return self.qs.numel() * self.qs.element_size() + self.d.numel() * 2

    def gemv(self, x: torch.Tensor, y: torch.Tensor | None = None, accumulate: bool = False, stream=None):
        if y is None:
            y = torch.empty(self.rows, dtype=torch.float32, device=x.device)
        fn = lib().zcu_gemv_q8_0 if self.qtype == 8 else lib().zcu_gemv_q4_0
        check(fn(self.qs.data_ptr(), self.d.data_ptr(), x.data_ptr(), y.data_ptr(), self.rows, self.cols,
                 int(accumulate), _stream(stream)), "gemv")
        return y


class QuantizedKernels:
    """QuantizedKernels (QuantizedKernels.cs) over device-resident weights."""

    @staticmethod
    def mat_vec_mul_q8_0(w: QuantizedWeight, x, y, rows, cols, stream=None):
        assert w.qtype == 8 and (rows, cols) == (w.rows, w.cols)
        return w.gemv(x, y, False, stream)

    @staticmethod
    def mat_vec_add_q8_0(w: QuantizedWeight, x, y, rows, cols, stream=None):
        assert w.qtype == 8 and (rows, cols) == (w.rows, w.cols)
        return w.gemv(x, y, True, stream)

    @staticmethod
    def mat_vec_mul_q4_0(w: QuantizedWeight, x, y, rows, cols, stream=None):
        assert w.qtype == 4 and (rows, cols) == (w.rows, w.cols)
        return w.gemv(x, y, False, stream)

    @staticmethod
    def mat_vec_add_q4_0(w: QuantizedWeight, x, y, rows, cols, stream=None):
        assert w.qtype == 4 and (rows, cols) == (w.rows, w.cols)
        return w.gemv(x, y, True, stream)


class TensorBlas:
    """TensorBlas.GemvQ8_0 / GemvQ4_0 (TensorBlas.Quantized.cs:447-485) through the bridge ABI."""

    @staticmethod
    def gemv_q8_0(activation: np.ndarray, packed_weights: np.ndarray, n_rows: int, k_cols: int) -> np.ndarray:
        x = np.ascontiguousarray(activation, dtype=np.float32)
        w = np.ascontiguousarray(packed_weights, dtype=np.uint8)
        y = np.empty(n_rows, dtype=np.float32)
        check(lib().zc_gemv_q8_0(_np_ptr(w), _np_ptr(x), _np_ptr(y), n_rows, k_cols), "zc_gemv_q8_0")
        return y

    @staticmethod
    def gemv_q4_0(activation: np.ndarray, packed_weights: np.ndarray, n_rows: int, k_cols: int) -> np.ndarray:
        x = np.ascontiguousarray(activation, dtype=np.float32)
        w = np.ascontiguousarray(packed_weights, dtype=np.uint8)
        y = np.empty(n_rows, dtype=np.float32)
        check(lib().zc_gemv_q4_0(_np_ptr(w), _np_ptr(x), _np_ptr(y), n_rows, k_cols), "zc_gemv_q4_0")
        return y


class TensorOps:
    @staticmethod
    def paged_attention(q, k_cache, v_cache, block_table, context_len: int, scale: float | None = None):
        """TensorOps.PagedAttention: q [hq, hd]; caches [num_blocks, block_size, hkv, hd] fp32.

        numpy inputs run through the bridge ABI (zc_paged_attention_f32, host memory); torch CUDA
        tensors run the device entry point on the current stream.
        """
        hq, hd = q.shape
        nb, bs, hkv, _ = k_cache.shape
        if scale is None:
            scale = float(np.float32(1.0) / np.float32(np.sqrt(np.float64(hd))))
        if isinstance(q, np.ndarray):
            qn = np.ascontiguousarray(q, dtype=np.float32)
            kn = np.ascontiguousarray(k_cache, dtype=np.float32)
            vn = np.ascontiguousarray(v_cache, dtype=np.float32)
            bt = np.ascontiguousarray(block_table, dtype=np.int32)
            out = np.empty_like(qn)
            check(lib().zc_paged_attention_f32(hq, hkv, hd, bs, context_len, scale, _np_ptr(qn), _np_ptr(kn),
                                               _np_ptr(vn), _np_ptr(bt) if bt.size else 0, _np_ptr(out)),
                  "zc_paged_attention_f32")
            return out
        dev = q.device
        bt = torch.as_tensor(np.asarray(block_table, dtype=np.int32)).to(dev) if not torch.is_tensor(
            block_table) else block_table.to(dev, torch.int32)
        ctx = torch.tensor([context_len], dtype=torch.int32, device=dev)
        out = torch.empty_like(q)
        kv_dtype = 1 if k_cache.dtype == torch.float16 else 0
        check(lib().zcu_paged_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), kv_dtype,
                                        bt.data_ptr(), ctx.data_ptr(), out.data_ptr(), 1, hq, hkv, hd, bs,
                                        max(1, bt.numel()), nb, bs * hkv * hd, hkv * hd, hd, scale, context_len,
                                        _stream()), "zcu_paged_attention")
        return out


def paged_attention_batched(q, k_pool, v_pool, page_table, ctx_len, hkv: int, page_size: int, num_pages: int,
                            page_stride: int, slot_stride: int, head_stride: int, scale: float, max_ctx: int,
                            out=None, stream=None):
    """Device paged attention for a batch of sequences (GqaAttention.Forward per sequence).

    q [batch, hq, hd] fp32; k_pool/v_pool fp16 or fp32 device buffers addressed with the given element
    strides; page_table [batch, max_pages] int32; ctx_len [batch] int32, both on the device."""
    batch, hq, hd = q.shape
    if out is None:
        out = torch.empty_like(q)
    kv_dtype = 1 if k_pool.dtype == torch.float16 else 0
    check(lib().zcu_paged_attention(q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), kv_dtype,
                                    page_table.data_ptr(), ctx_len.data_ptr(), out.data_ptr(), batch, hq, hkv, hd,
                                    page_size, page_table.shape[1], num_pages, page_stride, slot_stride,
                                    head_stride, scale, max_ctx, _stream(stream)), "zcu_paged_attention")
    return out


class LlmSampler:
    """LlmSampler.Sample (ZeroLlm/src/ZeroLlm.Core/Sampling/LlmSampler.cs:21-172) on device logits."""

    @staticmethod
    def sample(logits: torch.Tensor, past=None, temperature=0.7, top_p=0.9, min_p=0.0, top_k=40,
               repetition_penalty=1.1, u=None, stream=None) -> torch.Tensor:
        """logits [rows][vocab] fp32 on the device (modified in place, as the reference modifies its span); past: a
        list of token sequences, one per row (or None); u [rows]: the draws standing for (float)random.NextDouble()
        (unused on the greedy branch).  Returns the tokens [rows] (int32, device)."""
        from ._lib import SamplingConfig
        lg = logits if logits.dim() == 2 else logits.view(1, -1)
        rows, vocab = lg.shape
        cfg = SamplingConfig(temperature, top_p, min_p, top_k, repetition_penalty)
        past_t = plen_t = None
        pcap = 0
        if past is not None:
            pcap = max(1, max(len(p) for p in past))
            buf = np.zeros((rows, pcap), np.int32)
            lens = np.zeros(rows, np.int32)
            for r, p in enumerate(past):
                buf[r, :len(p)] = p
                lens[r] = len(p)
            past_t, plen_t = torch.from_numpy(buf).to(lg.device), torch.from_numpy(lens).to(lg.device)
        u_t = None if u is None else torch.as_tensor(u, dtype=torch.float32, device=lg.device).reshape(rows)
        out = torch.empty(rows, dtype=torch.int32, device=lg.device)
        check(lib().zcu_sample(lg.data_ptr(), rows, vocab, _ptr(past_t), _ptr(plen_t), pcap, C.byref(cfg), _ptr(u_t),
                               out.data_ptr(), None, None, None, 0, _stream(stream)), "sample")
        return out
