"""GGUF loader (zeroplatform_b200/gguf.py) against the reference's format rules.

* the reference's own round-trip test (ZeroLlm/tests/ZeroLlm.Tests/GgufFormatTests.cs:10-50): the same metadata and
  the same 32 x 2 F32 tensor, read back with the same assertions;
* typed metadata lookups fall back to the default when a key holds another type (GgufMetadata.TryGet<T>);
* a model saved with LlmModel.SaveGguf's names and dimensions loads back bit-identical, with LoadGguf's shape rules
  (vocabulary and width from token_embd.weight) and the tied LM head when output.weight is absent;
* truncated payloads, bad magic and unsupported versions are refused;
* (GPU) the engine loaded from the file reproduces the oracle engine's logits.
"""
import os
import struct

import numpy as np
import pytest

import oracle as O
from tests.conftest import rel_err
from zeroplatform_b200 import gguf as G


def test_reference_round_trip(tmp_path):
    p = str(tmp_path / "m.gguf")
    meta = [("general.architecture", G.STRING, "llama"), ("llama.context_length", G.U32, 4096),
            ("llama.embedding_length", G.U32, 2048), ("llama.attention.head_count", G.U32, 16),
            ("llama.attention.head_count_kv", G.U32, 4), ("llama.attention.layer_norm_rms_epsilon", G.F32, 1e-5)]
    G.write_gguf(p, meta, [("token_embd.weight", [32, 2], G.T_F32, bytes(range(64)))])
    with G.GgufFile(p) as g:
        assert g.version == 3 and g.tensor_count == 1
        assert g.architecture == "llama"
        assert g.get("llama.context_length", G.U32, 2048) == 4096
        assert g.get("llama.embedding_length", G.U32, 4096) == 2048
        assert g.get("llama.attention.head_count", G.U32, 32) == 16
        assert g.get("llama.attention.head_count_kv", G.U32, 16) == 4
        assert g.get("llama.attention.layer_norm_rms_epsilon", G.F32, 0.0) == np.float32(1e-5)
        (t,) = g.tensors
        assert t.name == "token_embd.weight" and t.type == G.T_F32 and t.dims == [32, 2]
        assert t.element_count == 64 and t.size_in_bytes() == 256  # 64 F32 elements
        assert g.data_offset % 32 == 0


def test_typed_lookup_and_case_insensitive_keys(tmp_path):
    p = str(tmp_path / "m.gguf")
    meta = [("LLAMA.Block_Count", G.U64, 7), ("llama.feed_forward_length", G.U32, 96),
            ("general.alignment", G.U32, 64)]
    G.write_gguf(p, meta, [], alignment=64)
    with G.GgufFile(p) as g:
        assert g.get("llama.block_count", G.U32, 4) == 4   # stored as UInt64: the UInt32 lookup keeps the default
        assert g.get("llama.block_count", G.U64, 4) == 7
        assert g.get("LLAMA.FEED_FORWARD_LENGTH", G.U32, 0) == 96
        assert g.alignment == 64 and g.data_offset % 64 == 0


def _model():
    return O.make_model(vocab=320, dim=128, layers=2, heads=4, kv_heads=2, ffn=256, seed=41)


def test_saved_model_loads_back_bit_identical(tmp_path):
    m = _model()
    p = str(tmp_path / "m.gguf")
    G.save_gguf(m, p)
    with G.GgufFile(p) as g:
        lm = G.model_from_gguf(g)
        for k in ("vocab", "dim", "layers", "heads", "kv_heads", "ffn", "context_length", "hd"):
            assert lm[k] == m[k], k
        assert lm["eps"] == np.float32(m["eps"]) and lm["rope_base"] == np.float32(m["rope_base"])
        for k in ("tok_emb", "lm_head", "final_norm"):
            assert np.array_equal(np.asarray(lm[k]).reshape(-1), np.asarray(m[k]).reshape(-1).view(lm[k].dtype)), k
        for k in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wgate", "wup", "wdown"):
            for l in range(m["layers"]):
                want = np.ascontiguousarray(m[k][l]).reshape(-1).view(lm[k][l].dtype)
                assert np.array_equal(lm[k][l], want), (k, l)
        assert g.tensor("blk.1.attn_output.weight").dims == [m["heads"] * m["hd"], m["dim"]]
        del lm


def test_tied_lm_head_and_truncated_payload(tmp_path):
    m = _model()
    p = str(tmp_path / "m.gguf")
    G.save_gguf(m, p)
    with G.GgufFile(p) as g:
        tensors = [(t.name, t.dims, t.type, bytes(g.tensor_bytes(t))) for t in g.tensors if t.name != "output.weight"]
        meta = [(k, v.type, v.value) for k, v in g.metadata.items()]
    q = str(tmp_path / "tied.gguf")
    G.write_gguf(q, meta, tensors)
    with G.GgufFile(q) as g:
        lm = G.model_from_gguf(g)
        assert lm["lm_head"] is lm["tok_emb"]
        del lm
    size = os.path.getsize(q)
    with open(q, "rb") as f:
        head = f.read(size - 40)
    r = str(tmp_path / "short.gguf")
    with open(r, "wb") as f:
        f.write(head)
    with G.GgufFile(r) as g:
        with pytest.raises(ValueError, match="beyond file boundary"):
            g.tensor_bytes(g.tensors[-1])


def test_bad_magic_and_version(tmp_path):
    p = str(tmp_path / "bad.gguf")
    with open(p, "wb") as f:
        f.write(struct.pack("<IIQQ", 0x12345678, 3, 0, 0))
    with pytest.raises(ValueError, match="magic"):
        G.GgufFile(p)
    with open(p, "wb") as f:
        f.write(struct.pack("<IIQQ", G.GGUF_MAGIC, 4, 0, 0))
    with pytest.raises(ValueError, match="version"):
        G.GgufFile(p)


@pytest.mark.gpu
def test_engine_from_gguf_matches_oracle(tmp_path):
    m = _model()
    p = str(tmp_path / "m.gguf")
    G.save_gguf(m, p)
    e = G.load_engine(p, max_batch=2, total_pages=32)
    ref = O.Engine(m, kv_fp16=True)
    prompt = np.random.default_rng(3).integers(0, m["vocab"], 11).astype(np.int32)
    assert rel_err(e.prefill(0, prompt, 0), ref.prefill(0, prompt, 0)) <= 1e-3
    assert rel_err(e.forward_token(0, 7, 11), ref.forward_token(0, 7, 11)) <= 1e-3
    e.close()
