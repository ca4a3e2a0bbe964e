"""ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the timed CPU
baseline of bench.py.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
import this package; the product (zeroplatform_b200) never does.

Every wrapper forwards to a C++ restatement of the reference C# (see oracle.h for
the file:line each one follows).  Inputs are numpy arrays; weights are the
reference's own packed AoS block layout (Q8_0: 34 B, Q4_0: 18 B per 32 values).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

QK = 32
Q8_BYTES = 34
Q4_BYTES = 18

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i8p = C.POINTER(C.c_int8)
_i32p = C.POINTER(C.c_int32)
_u16p = C.POINTER(C.c_uint16)


class OrcModel(C.Structure):
    """Mirror of orc_model in oracle.h."""

    _fields_ = [
        ("vocab", C.c_int), ("dim", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
        ("kv_heads", C.c_int), ("ffn", C.c_int), ("context_length", C.c_int),
        ("eps", C.c_float), ("rope_base", C.c_float),
        ("tok_emb", _u8p), ("lm_head", _u8p), ("final_norm", _f32p),
        ("attn_norm", _f32p), ("ffn_norm", _f32p),
        ("wq", _u8p), ("wk", _u8p), ("wv", _u8p), ("wo", _u8p),
        ("wgate", _u8p), ("wup", _u8p), ("wdown", _u8p),
    ]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc only, no GPU)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "oracle.cpp")):
        build()
    L = C.CDLL(_LIB_PATH)
    sz = C.c_size_t
    sig = {
        "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_f32_to_f16_array": (None, [_f32p, _u16p, sz]),
        "orc_quantize_q8_0": (None, [_f32p, sz, _u8p]),
        "orc_quantize_q4_0": (None, [_f32p, sz, _u8p]),
        "orc_dequantize_q8_0": (None, [_u8p, sz, _f32p]),
        "orc_dequantize_q4_0": (None, [_u8p, sz, _f32p]),
        "orc_dot_q8_0": (C.c_float, [_f32p, _u8p, sz, C.c_int]),
        "orc_dot_q4_0": (C.c_float, [_f32p, _u8p, sz, C.c_int]),
        "orc_matvec_q8_0": (None, [_u8p, _f32p, _f32p, sz, sz, C.c_int, C.c_int]),
        "orc_matvec_q4_0": (None, [_u8p, _f32p, _f32p, sz, sz, C.c_int, C.c_int]),
        "orc_matmul_q8_0": (None, [_u8p, _f32p, _f32p, sz, sz, sz, C.c_int, C.c_int]),
        "orc_matmul_q4_0": (None, [_u8p, _f32p, _f32p, sz, sz, sz, C.c_int, C.c_int]),
        "orc_gemm_i8": (None, [_i8p, _i8p, _i32p, sz, sz, sz]),
        "orc_dot_i8": (C.c_int32, [_i8p, _i8p, sz]),
        "orc_block_dots_i8": (None, [_i8p, _u8p, _i32p, sz, sz, sz]),
        "orc_rmsnorm": (None, [_f32p, _f32p, _f32p, sz, C.c_float]),
        "orc_rope_table": (None, [C.c_int, C.c_int, C.c_float, _f32p, _f32p]),
        "orc_rope_apply": (None, [_f32p, C.c_int, C.c_int, _f32p, _f32p]),
        "orc_swiglu": (None, [_f32p, _f32p, _f32p, sz]),
        "orc_dot_f32": (C.c_float, [_f32p, _f32p, C.c_int]),
        "orc_gqa_attention": (None, [_f32p, _f32p, _f32p, _i32p, C.c_int, sz, C.c_int, C.c_int, C.c_int,
                                     C.c_int, _f32p]),
        "orc_flash_attention": (None, [sz, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int,
                                       C.c_int, _f32p, _f32p, _f32p, _f32p, sz, _f32p]),
        "orc_paged_attention": (None, [_f32p, _f32p, _f32p, _i32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_int, C.c_float, _f32p]),
        "orc_moe_forward": (None, [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, _u8p, _u8p, _u8p,
                                   C.c_int, C.c_int, _f32p, _i32p, _f32p]),
        "orc_sample_greedy": (C.c_int32, [_f32p, sz, _i32p, sz, C.c_float]),
        "orc_sample": (C.c_int32, [_f32p, sz, _i32p, sz, C.c_float, C.c_float, C.c_float, C.c_int32, C.c_float,
                                   C.c_float, _i32p, _f32p, _i32p, C.c_int32]),
        "orc_engine_create": (C.c_void_p, [C.POINTER(OrcModel), C.c_int, C.c_int, C.c_int, C.c_int]),
        "orc_engine_destroy": (None, [C.c_void_p]),
        "orc_engine_prefill": (C.c_int, [C.c_void_p, C.c_int, _i32p, C.c_int, C.c_int, _f32p]),
        "orc_engine_forward_token": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, _f32p]),
        "orc_engine_seq_len": (C.c_int, [C.c_void_p, C.c_int]),
        "orc_engine_free_blocks": (C.c_int, [C.c_void_p]),
        "orc_engine_free_sequence": (None, [C.c_void_p, C.c_int]),
        "orc_engine_get_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]),
        "orc_engine_page_table": (C.c_int, [C.c_void_p, C.c_int, _i32p, C.c_int]),
        "orc_engine_append_token": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p]),
        "orc_num_threads": (C.c_int, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(t)


def _opt(a, t):
    return None if a is None else _p(a, t)


# ---- fp16 --------------------------------------------------------------------------
def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(_p(x, _f32p), _p(out, _u16p), x.size)
    return out


# ---- block formats -------------------------------------------------------------------
def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """[rows, cols] fp32 -> [rows, cols/32*34] uint8 (LlmQuantizer.QuantizeToQ8_0)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    assert w.shape[-1] % QK == 0
    out = np.empty(w.shape[:-1] + (w.shape[-1] // QK * Q8_BYTES,), dtype=np.uint8)
    lib().orc_quantize_q8_0(_p(w, _f32p), w.size, _p(out, _u8p))
    return out


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    """[rows, cols] fp32 -> [rows, cols/32*18] uint8 (LlmQuantizer.QuantizeToQ4_0)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    assert w.shape[-1] % QK == 0
    out = np.empty(w.shape[:-1] + (w.shape[-1] // QK * Q4_BYTES,), dtype=np.uint8)
    lib().orc_quantize_q4_0(_p(w, _f32p), w.size, _p(out, _u8p))
    return out


def dequantize_q8_0(blocks: np.ndarray, cols: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // Q8_BYTES * QK
    out = np.empty(n, dtype=np.float32)
    lib().orc_dequantize_q8_0(_p(blocks, _u8p), n, _p(out, _f32p))
    return out.reshape(-1, cols)


def dequantize_q4_0(blocks: np.ndarray, cols: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // Q4_BYTES * QK
    out = np.empty(n, dtype=np.float32)
    lib().orc_dequantize_q4_0(_p(blocks, _u8p), n, _p(out, _f32p))
    return out.reshape(-1, cols)


def dot_q8_0(x, blocks, path=0) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    return lib().orc_dot_q8_0(_p(x, _f32p), _p(blocks, _u8p), blocks.size // Q8_BYTES, path)


def dot_q4_0(x, blocks, path=0) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    return lib().orc_dot_q4_0(_p(x, _f32p), _p(blocks, _u8p), blocks.size // Q4_BYTES, path)


def matvec(qtype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int, y: np.ndarray | None = None,
           threads: int = 0) -> np.ndarray:
    """MatVecMulQ*_0 (y is None) or MatVecAddQ*_0 (y updated in place and returned)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    acc = y is not None
    if y is None:
        y = np.empty(rows, dtype=np.float32)
    fn = lib().orc_matvec_q8_0 if qtype == 8 else lib().orc_matvec_q4_0
    fn(_p(w, _u8p), _p(x, _f32p), _p(y, _f32p), rows, cols, int(acc), threads)
    return y


def matmul(qtype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int, y: np.ndarray | None = None,
           threads: int = 0) -> np.ndarray:
    """Token-parallel Y[m] (=|+=) W X[m] as LlmEngine.PrefillPrompt runs it."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    m = x.shape[0]
    acc = y is not None
    if y is None:
        y = np.empty((m, rows), dtype=np.float32)
    fn = lib().orc_matmul_q8_0 if qtype == 8 else lib().orc_matmul_q4_0
    fn(_p(w, _u8p), _p(x, _f32p), _p(y, _f32p), m, rows, cols, int(acc), threads)
    return y


def gemm_i8(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.int32)
    lib().orc_gemm_i8(_p(a, _i8p), _p(b, _i8p), _p(c, _i32p), m, n, k)
    return c


def dot_i8(a, b) -> int:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    return int(lib().orc_dot_i8(_p(a, _i8p), _p(b, _i8p), a.size))


# ---- layers ----------------------------------------------------------------------------
def rmsnorm(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(x, _f32p), _p(w, _f32p), _p(out, _f32p), x.size, eps)
    return out


def rope_table(max_pos, head_dim, base=10000.0):
    c = np.empty((max_pos, head_dim // 2), dtype=np.float32)
    s = np.empty_like(c)
    lib().orc_rope_table(max_pos, head_dim, base, _p(c, _f32p), _p(s, _f32p))
    return c, s


def rope_apply(v, pos, head_dim, cos_t, sin_t):
    v = np.array(v, dtype=np.float32, copy=True)
    lib().orc_rope_apply(_p(v, _f32p), pos, head_dim, _p(cos_t, _f32p), _p(sin_t, _f32p))
    return v


def swiglu(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().orc_swiglu(_p(g, _f32p), _p(u, _f32p), _p(out, _f32p), g.size)
    return out


def gqa_attention(q, kpool, vpool, page_table, page_size, seq_len, hq, hkv, hd, page_stride=None):
    """GqaAttention.Forward over per-layer pools laid out [page][slot][hkv][hd] (page_stride defaults
    to page_size*hkv*hd floats)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kpool = np.ascontiguousarray(kpool, dtype=np.float32)
    vpool = np.ascontiguousarray(vpool, dtype=np.float32)
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    if page_stride is None:
        page_stride = page_size * hkv * hd
    out = np.empty(hq * hd, dtype=np.float32)
    lib().orc_gqa_attention(_p(q, _f32p), _p(kpool, _f32p), _p(vpool, _f32p), _p(pt, _i32p), page_size,
                            page_stride, seq_len, hq, hkv, hd, _p(out, _f32p))
    return out


def flash_attention(q, k, v, mask=None, scale=None):
    """TensorOps.FlashAttentionCpu on [..., s, d] tensors: rank-4 q [B, hq, sq, d] and k / v [B, hkv, sk, d|dv]
    take the grouped-query form; lower ranks flatten the leading dimensions into the batch."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    sq, d = q.shape[-2:]
    sk, dv = k.shape[-2], v.shape[-1]
    hq = hkv = 1
    if q.ndim == 4 and k.ndim == 4:
        hq, hkv = q.shape[1], k.shape[1]
    group = hq // hkv
    batch = int(np.prod(q.shape[:-2], dtype=np.int64))
    out = np.empty(q.shape[:-1] + (dv,), dtype=np.float32)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
        mb = mask.size // (sq * sk) if sq * sk else 1
        mp = _p(mask, _f32p)
    else:
        mb, mp = 1, None
    sc = np.float32(1.0) / np.float32(np.sqrt(np.float64(d))) if scale is None else np.float32(scale)
    lib().orc_flash_attention(batch, sq, sk, d, dv, float(sc), int(group > 1), hq, hkv, group, _p(q, _f32p),
                              _p(k, _f32p), _p(v, _f32p), mp, mb, _p(out, _f32p))
    return out


def paged_attention(q, kcache, vcache, block_table, context_len, scale=None):
    """TensorOps.PagedAttention: q [hq, hd], caches [nb, bs, hkv, hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kcache = np.ascontiguousarray(kcache, dtype=np.float32)
    vcache = np.ascontiguousarray(vcache, dtype=np.float32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    hq, hd = q.shape
    bs, hkv = kcache.shape[1], kcache.shape[2]
    if scale is None:
        scale = float(np.float32(1.0) / np.float32(np.sqrt(np.float64(hd))))
    out = np.empty_like(q)
    lib().orc_paged_attention(_p(q, _f32p), _p(kcache, _f32p), _p(vcache, _f32p), _p(bt, _i32p), hq, hkv, hd,
                              bs, context_len, scale, _p(out, _f32p))
    return out


def moe_forward(xnorm, qtype, eg, eu, ed, dim, ffn, n_experts, top_k, residual, router_logits=None,
                router_w=None):
    """SparseMoeLayer.Forward for one token; residual updated in place. Returns (idx, weights)."""
    xnorm = np.ascontiguousarray(xnorm, dtype=np.float32)
    idx = np.empty(top_k, dtype=np.int32)
    wts = np.empty(top_k, dtype=np.float32)
    rl = None if router_logits is None else np.ascontiguousarray(router_logits, dtype=np.float32)
    rw = None if router_w is None else np.ascontiguousarray(router_w, dtype=np.float32)
    lib().orc_moe_forward(_p(xnorm, _f32p), _opt(rw, _f32p), _opt(rl, _f32p), n_experts, top_k, qtype,
                          _p(eg, _u8p), _p(eu, _u8p), _p(ed, _u8p), dim, ffn, _p(residual, _f32p),
                          _p(idx, _i32p), _p(wts, _f32p))
    return idx, wts


def sample_greedy(logits, past=(), penalty=1.0) -> int:
    lg = np.array(logits, dtype=np.float32, copy=True)
    past = np.ascontiguousarray(np.asarray(past, dtype=np.int32))
    return int(lib().orc_sample_greedy(_p(lg, _f32p), lg.size, _p(past, _i32p) if past.size else None,
                                       past.size, penalty))


def sample(logits, past=(), temperature=0.7, top_p=0.9, min_p=0.0, top_k=40, penalty=1.1, u=0.5, cap=65536):
    """LlmSampler.Sample with the random draw given (u for (float)random.NextDouble()).  Returns (token, kept
    candidate ids, their renormalised probabilities, logits after the in-place updates)."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    past = np.ascontiguousarray(np.asarray(past, dtype=np.int32))
    ci = np.zeros(cap, np.int32)
    cp = np.zeros(cap, np.float32)
    n = np.zeros(1, np.int32)
    tok = int(lib().orc_sample(_p(lg, _f32p), lg.size, _p(past, _i32p) if past.size else None, past.size,
                               temperature, top_p, min_p, top_k, penalty, u, _p(ci, _i32p), _p(cp, _f32p),
                               _p(n, _i32p), cap))
    k = int(n[0])
    return tok, ci[:k].copy(), cp[:k].copy(), lg


# ---- model + engine ----------------------------------------------------------------------
def q8_bytes(rows, cols):
    return rows * (cols // QK) * Q8_BYTES


def make_model(vocab, dim, layers, heads, kv_heads, ffn, seed=0, std=0.02, context_length=2048,
               eps=1e-5, rope_base=10000.0):
    """Seeded Llama-style model: every 2-D weight ~ N(0, std) quantized to Q8_0 with the oracle's
    quantizer; norm weights are 1.0 (LlmModel.CreateSynthetic draws uniform(-0.02, 0.02), this
    generator draws the normal distribution the benchmark configuration specifies)."""
    hd = dim // heads
    qdim, kvdim = heads * hd, kv_heads * hd
    rng = np.random.default_rng(seed)

    def q8(rows, cols, n=1):
        w = rng.standard_normal((n, rows, cols), dtype=np.float32) * np.float32(std)
        return quantize_q8_0(w).reshape(n, rows, cols // QK * Q8_BYTES)

    m = dict(vocab=vocab, dim=dim, layers=layers, heads=heads, kv_heads=kv_heads, ffn=ffn, hd=hd,
             context_length=context_length, eps=eps, rope_base=rope_base)
    m["tok_emb"] = q8(vocab, dim)[0]
    m["wq"] = q8(qdim, dim, layers)
    m["wk"] = q8(kvdim, dim, layers)
    m["wv"] = q8(kvdim, dim, layers)
    m["wo"] = q8(dim, qdim, layers)
    m["wgate"] = q8(ffn, dim, layers)
    m["wup"] = q8(ffn, dim, layers)
    m["wdown"] = q8(dim, ffn, layers)
    m["lm_head"] = q8(vocab, dim)[0]
    m["attn_norm"] = np.ones((layers, dim), dtype=np.float32)
    m["ffn_norm"] = np.ones((layers, dim), dtype=np.float32)
    m["final_norm"] = np.ones(dim, dtype=np.float32)
    return m


class Engine:
    """Oracle LlmEngine + PagedKvCache over a model from make_model()."""

    def __init__(self, model: dict, total_pages=256, page_size=16, kv_fp16=False, threads=0):
        self.model = model
        L = lib()
        s = OrcModel()
        for k in ("vocab", "dim", "layers", "heads", "kv_heads", "ffn", "context_length"):
            setattr(s, k, int(model[k]))
        s.eps = model["eps"]
        s.rope_base = model["rope_base"]
        self._keep = []
        for k in ("tok_emb", "lm_head", "wq", "wk", "wv", "wo", "wgate", "wup", "wdown"):
            a = np.ascontiguousarray(model[k])
            self._keep.append(a)
            setattr(s, k, _p(a, _u8p))
        for k in ("final_norm", "attn_norm", "ffn_norm"):
            a = np.ascontiguousarray(model[k], dtype=np.float32)
            self._keep.append(a)
            setattr(s, k, _p(a, _f32p))
        self._s = s
        self._h = L.orc_engine_create(C.byref(s), total_pages, page_size, int(kv_fp16), threads)
        if not self._h:
            raise RuntimeError("orc_engine_create failed")

    def close(self):
        if self._h:
            lib().orc_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, seq_id, tokens, start_pos=0):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.model["vocab"], dtype=np.float32)
        rc = lib().orc_engine_prefill(self._h, seq_id, _p(t, _i32p), t.size, start_pos, _p(logits, _f32p))
        if rc != 0:
            raise RuntimeError("Paged KV-cache exhausted")
        return logits

    def forward_token(self, seq_id, token, pos):
        logits = np.empty(self.model["vocab"], dtype=np.float32)
        rc = lib().orc_engine_forward_token(self._h, seq_id, int(token), int(pos), _p(logits, _f32p))
        if rc != 0:
            raise RuntimeError("Paged KV-cache exhausted")
        return logits

    def append_token(self, seq_id, layer, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        if lib().orc_engine_append_token(self._h, seq_id, layer, _p(k, _f32p), _p(v, _f32p)) != 0:
            raise RuntimeError("Paged KV-cache exhausted")

    def seq_len(self, seq_id):
        return lib().orc_engine_seq_len(self._h, seq_id)

    def free_blocks(self):
        return lib().orc_engine_free_blocks(self._h)

    def free_sequence(self, seq_id):
        lib().orc_engine_free_sequence(self._h, seq_id)

    def get_kv(self, seq_id, layer, token, value=False):
        kvdim = self.model["kv_heads"] * self.model["hd"]
        out = np.empty(kvdim, dtype=np.float32)
        if lib().orc_engine_get_kv(self._h, seq_id, layer, token, int(value), _p(out, _f32p)) != 0:
            raise KeyError(seq_id)
        return out

    def page_table(self, seq_id):
        buf = np.empty(4096, dtype=np.int32)
        n = lib().orc_engine_page_table(self._h, seq_id, _p(buf, _i32p), buf.size)
        return buf[:n].copy()

    def generate_greedy(self, seq_id, prompt, n_new, penalty=1.0):
        """GenerateStreamAsync with greedy sampling: prefill, then sample -> ForwardToken."""
        logits = self.prefill(seq_id, prompt, 0)
        past = list(int(t) for t in prompt)
        out = []
        pos = len(prompt)
        for _ in range(n_new):
            tok = sample_greedy(logits, past, penalty)
            out.append(tok)
            past.append(tok)
            logits = self.forward_token(seq_id, tok, pos)
            pos += 1
        return out, logits
