"""Host-side checks of the C++ GGUF loader and config validation (no GPU): the library loads,
exports every declared symbol, accepts valid models and rejects malformed ones with the
reference's error categories."""
import ctypes
import re
import struct
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, spec_path
from voxgen_b200 import api, gguf, synth


def test_library_exports_every_header_symbol():
    header = (ROOT / "include" / "voxgen_cuda.h").read_text()
    declared = set(re.findall(r"^\s*(?:int|const char \*)\s*(vg_\w+)\(", header, re.M))
    assert declared == set(api.EXPORTS)
    L = ctypes.CDLL(str(api._build.LIB if api._build.LIB.exists() else api._build.build()))
    for name in declared:
        assert hasattr(L, name), name


def test_inspect_valid_models(model_dir):
    for name in ("tiny", "tiny_f16", "cfg0", "g6"):
        spec = synth.preset(name)
        info = api.inspect_gguf(spec_path(model_dir, name))
        assert info["embedding_length"] == spec.hidden
        assert info["block_count"] == spec.layers
        assert info["feed_forward_length"] == spec.ffn
        assert info["head_count"] == spec.heads and info["head_count_kv"] == spec.kv_heads
        assert info["head_dim"] == spec.head_dim and info["kv_dim"] == spec.kv_dim
        assert info["vocab_size"] == spec.vocab
        assert info["format"] == spec.fmt
        assert info["tied_output"] == 1
        assert info["rope_scaling_factor"] == 1.0
        H, F, KV = spec.hidden, spec.ffn, spec.kv_dim
        el = spec.layers * (2 * H * H + 2 * H * KV + 3 * H * F)
        per = 34 / 32 if spec.fmt == gguf.GGML_Q8_0 else 2
        assert info["layer_weight_bytes"] == int(el * per)


def test_cfg0_algorithmic_bytes(model_dir):
    # 15,876,096 Q8_0 bytes per layer at cfg0's shape
    info = api.inspect_gguf(spec_path(model_dir, "cfg0"))
    assert info["layer_weight_bytes"] == 15_876_096


def test_format_request_mismatch(model_dir):
    with pytest.raises(api.VoxGenError) as e:
        api.inspect_gguf(spec_path(model_dir, "tiny"), "f16")
    assert e.value.code == -4 and "format mismatch" in str(e.value)


def _write(tmp_path, spec, mutate=None, name="m.gguf"):
    g, plan = synth.build_gguf(spec)
    for tname, dims, ty, gen in plan:
        g.tensors.append(gguf.Tensor(tname, dims, ty, np.ascontiguousarray(gen()).view(np.uint8).reshape(-1)))
    if mutate:
        mutate(g)
    p = tmp_path / name
    gguf.write_gguf(p, g)
    return p


SMALL = synth.preset("tiny", layers=1, vocab=64)


def _err(path, code=None, text=None):
    with pytest.raises(api.VoxGenError) as e:
        api.inspect_gguf(path)
    if code is not None:
        assert e.value.code == code, str(e.value)
    if text is not None:
        assert text in str(e.value), str(e.value)


def test_bad_magic_and_version(tmp_path):
    p = _write(tmp_path, SMALL)
    b = bytearray(p.read_bytes())
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"XXXX" + b[4:])
    _err(bad, -3, "not a GGUF file")
    b2 = bytearray(b)
    b2[4:8] = struct.pack("<I", 4)
    bad.write_bytes(bytes(b2))
    _err(bad, -3, "unsupported GGUF version")


def test_truncated_file(tmp_path):
    p = _write(tmp_path, SMALL)
    b = p.read_bytes()
    t = tmp_path / "trunc.gguf"
    t.write_bytes(b[:200])
    _err(t, -3, "EOF")
    t.write_bytes(b[:-100])
    _err(t, -3, "extends beyond end")


def test_missing_file():
    _err("/nonexistent/x.gguf", -2)


def test_wrong_architecture(tmp_path):
    p = _write(tmp_path, SMALL, lambda g: g.metadata.__setitem__("general.architecture", "llama"))
    _err(p, -4, "minicpm4")


def test_missing_metadata(tmp_path):
    p = _write(tmp_path, SMALL, lambda g: g.metadata.pop("minicpm4.block_count"))
    _err(p, -4, "missing required metadata: minicpm4.block_count")


def test_missing_tensor(tmp_path):
    def drop(g):
        g.tensors = [t for t in g.tensors if t.name != "blk.0.ffn_up.weight"]
    _err(_write(tmp_path, SMALL, drop), -4, "blk.0.ffn_up.weight")


def test_wrong_dims(tmp_path):
    def bad(g):
        for t in g.tensors:
            if t.name == "blk.0.attn_k.weight":
                t.dims = (t.dims[1], t.dims[0])
    _err(_write(tmp_path, SMALL, bad), -4, "has dimensions")


def test_unsupported_tensor_type(tmp_path):
    def bad(g):
        for t in g.tensors:
            if t.name == "blk.0.attn_norm.weight":
                t.ggml_type = 2  # Q4_0: not supported by the reference BaseLM path
    _err(_write(tmp_path, SMALL, bad), None, None)


def test_heads_not_divisible(tmp_path):
    p = _write(tmp_path, SMALL, lambda g: g.metadata.__setitem__("minicpm4.attention.head_count_kv", gguf.U32(3)))
    _err(p, -4)


def test_partial_rope_rejected(tmp_path):
    p = _write(tmp_path, SMALL, lambda g: g.metadata.__setitem__("minicpm4.rope.dimension_count", gguf.U32(16)))
    _err(p, -4, "partial RoPE")


def test_unsupported_rope_scaling(tmp_path):
    p = _write(tmp_path, SMALL, lambda g: g.metadata.__setitem__("minicpm4.rope.scaling.type", "yarn"))
    _err(p, -4, "RoPE scaling")


def test_mixed_qkv_types_rejected(tmp_path):
    spec = SMALL

    def mix(g):
        for t in g.tensors:
            if t.name == "blk.0.attn_v.weight":
                rows, cols = t.dims[1], t.dims[0]
                t.ggml_type = gguf.GGML_F16
                t.data = np.zeros(rows * cols, np.float16).view(np.uint8)
    _err(_write(tmp_path, spec, mix), -4, "Q/K/V")


def test_alignment_and_version2(tmp_path):
    spec = replace(SMALL, alignment=64)
    p = _write(tmp_path, spec)
    assert gguf.read_gguf(p).data_offset % 64 == 0
    info = api.inspect_gguf(p)
    assert info["embedding_length"] == spec.hidden


def test_untied_output_and_scales(tmp_path):
    spec = replace(SMALL, tied_output=False, embedding_scale=12.0, residual_scale=0.25, logit_scale=0.125)
    info = api.inspect_gguf(_write(tmp_path, spec))
    assert info["tied_output"] == 0
    assert info["embedding_scale"] == 12.0 and info["residual_scale"] == 0.25
    assert info["logit_scale"] == 0.125


def test_long_rope_factor_selection(tmp_path):
    # context_length > original_context_length selects the long factors and a scaling factor
    # sqrt(1 + ln(max/orig)/ln(orig)) (src/baselm.rs:194-205, :902-913)
    def longctx(g):
        g.metadata["minicpm4.context_length"] = gguf.U32(65536)
        g.metadata["minicpm4.rope.scaling.original_context_length"] = gguf.U32(32768)
    info = api.inspect_gguf(_write(tmp_path, SMALL, longctx))
    want = np.float32(np.sqrt(np.float32(1.0) + np.log(np.float32(2.0)) / np.log(np.float32(32768.0))))
    assert abs(info["rope_scaling_factor"] - want) < 1e-6
    assert info["rope_long_factors"] == 1


def test_python_reader_roundtrip(model_dir):
    spec = synth.preset("tiny")
    g = gguf.read_gguf(spec_path(model_dir, "tiny"))
    assert g.metadata["general.architecture"] == "minicpm4"
    assert g.tensors["blk.1.ffn_down.weight"].dims == (spec.ffn, spec.hidden)
    w = g.matrix_f32("blk.0.attn_q.weight")
    assert w.shape == (spec.hidden, spec.hidden)
    # regenerate the same tensor from its seed: byte-identical
    _, plan = synth.build_gguf(spec)
    gen = dict((n, f) for n, _, _, f in plan)["blk.0.attn_q.weight"]
    assert np.array_equal(np.asarray(gen()).view(np.uint8).reshape(-1), g.tensor_bytes("blk.0.attn_q.weight"))
