"""Pins the oracle restatement to the reference's own BaseLM shader code.

The reference's GLSL compute shaders (shaders/*.comp in the VoxGen checkout) are compiled as C++
and run on the CPU by oracle/ref_shim (workgroups emulated with fibers, barriers honoured); the
dispatch sequence, bindings and push constants restate src/baselm.rs:892-1202. Every comparison
here is bit-exact: the oracle follows each shader's arithmetic order, so a single differing bit is
a restatement error.

These tests need the reference checkout (to build oracle/_ref) and skip without it; the golden
vectors under tests/golden/ carry the same pin to machines without the checkout
(test_oracle_matches_reference_golden).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from oracle import ref as R
from voxgen_b200 import gguf, synth

needs_ref = pytest.mark.skipif(not R.available(), reason="reference shaders not available here")
GOLDEN = Path(__file__).resolve().parent / "golden" / "ref_shader_pin.npz"


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def words(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    return np.concatenate([raw, np.zeros((-raw.size) % 4, np.uint8)]).view(np.uint32).copy()


def q8_matrix(rng, rows, cols):
    d = (np.abs(rng.standard_normal((rows, cols // 32))) * 0.02 / 127).astype(np.float16)
    qs = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    return gguf.q8_0_pack(d, qs)


def f16_matrix(rng, rows, cols):
    return (rng.standard_normal(rows * cols) * 0.02).astype(np.float16).view(np.uint8)


MATS = {8: q8_matrix, 1: f16_matrix}


@needs_ref
@pytest.mark.parametrize("dtype", [8, 1])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (37, 1024), (64, 4096)])
def test_matvec_and_swiglu_shaders(dtype, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols + dtype)
    w = MATS[dtype](rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    R.dispatch("matvec", [words(w), x, y], R.push("IIIIIf", 0, rows, cols, dtype, 0, 0.75), [rows])
    assert bits_equal(y, O.matvec(dtype, w, rows, cols, x, 0.75)), "matvec.comp"
    u = MATS[dtype](rng, rows, cols)
    both = np.concatenate([w, u])
    g = np.zeros(rows, np.float32)
    R.dispatch("matvec_swiglu", [words(both), x, g], R.push("IIIIII", 0, w.size, rows, cols, dtype, 0), [rows])
    assert bits_equal(g, O.swiglu(dtype, w, u, rows, cols, x)), "matvec_swiglu.comp"


@needs_ref
@pytest.mark.parametrize("n", [64, 1000, 2048])
def test_norm_shaders(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    br = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(n)).astype(np.float32)
    y = np.zeros(n, np.float32)
    R.dispatch("rmsnorm", [words(w.view(np.uint8)), x.copy(), y], R.push("IIf", 0, n, 1e-5), [1])
    assert bits_equal(y, O.rmsnorm(x, w, 1e-5)), "rmsnorm.comp"
    h = x.copy()
    R.dispatch("residual_rmsnorm", [words(w.view(np.uint8)), h, br, y], R.push("IIff", 0, n, 1e-5, 0.25), [1])
    oh, oy = O.residual_rmsnorm(x, br, w, 1e-5, 0.25)
    assert bits_equal(h, oh) and bits_equal(y, oy), "residual_rmsnorm.comp"


@needs_ref
@pytest.mark.parametrize("dtype", [8, 1])
def test_embedding_shader(dtype):
    rng = np.random.default_rng(5 + dtype)
    vocab, cols = 40, 512
    w = MATS[dtype](rng, vocab, cols)
    for tok in (0, 17, vocab - 1):
        out = np.zeros(cols, np.float32)
        R.dispatch("embedding", [words(w), out], R.push("IIIIf", 0, cols, tok, dtype, 12.0), [1])
        assert bits_equal(out, O.embedding(dtype, w, cols, tok, 12.0)), "embedding.comp"


@needs_ref
@pytest.mark.parametrize("heads,kv_heads", [(16, 2), (2, 1), (4, 4), (12, 2)])
@pytest.mark.parametrize("position", [0, 5, 300])
def test_rope_and_attention_shaders(heads, kv_heads, position):
    D, ctx = 128, 320
    kvd = kv_heads * D
    rng = np.random.default_rng(heads * 1000 + position)
    q = rng.standard_normal(heads * D).astype(np.float32)
    k = rng.standard_normal(kvd).astype(np.float32)
    ext = (1 + rng.random(D // 2)).astype(np.float32)
    rq, rk = q.copy(), k.copy()
    R.dispatch("rope", [words(ext.view(np.uint8)), rq, rk],
               R.push("IIIIIff", 0, position, heads, kv_heads, D, 10000.0, 1.1), [heads + kv_heads])
    oq, ok = O.rope(q, k, ext, position, heads, kv_heads, D, 10000.0, 1.1)
    assert bits_equal(rq, oq) and bits_equal(rk, ok), "rope.comp"

    kc = rng.standard_normal((ctx, kvd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((ctx, kvd)).astype(np.float16).view(np.uint16)
    scores = np.zeros(heads * ctx, np.float32)
    out = np.zeros(heads * D, np.float32)
    push = R.push("IIIIII", 0, ctx, position, D, heads // kv_heads, kv_heads)
    R.dispatch("attn_scores", [rq, words(kc.view(np.uint8)), scores], push, [position + 1, heads])
    R.dispatch("softmax", [scores], R.push("II", ctx, position), [heads])
    R.dispatch("attn_values", [scores, words(vc.view(np.uint8)), out], push, [heads])
    want, wscores = O.attention(rq, kc, vc, heads, kv_heads, D, position)
    sl = np.s_[:, :position + 1]
    assert bits_equal(scores.reshape(heads, ctx)[sl], wscores[sl]), "attn_scores.comp + softmax.comp"
    assert bits_equal(out, want), "attn_values.comp"


@needs_ref
def test_store_kv_shader():
    rng = np.random.default_rng(9)
    kvd, ctx, layer, pos = 256, 16, 1, 11
    k = (rng.standard_normal(kvd) * 3).astype(np.float32)
    v = (rng.standard_normal(kvd) * 1e-5).astype(np.float32)   # fp16 subnormals too
    kc = np.zeros(2 * ctx * kvd // 2, np.uint32)
    vc = np.zeros_like(kc)
    R.dispatch("store_kv", [k, v, kc, vc], R.push("IIII", layer, pos, ctx, kvd), [1])
    got_k = kc.view(np.uint16).reshape(2, ctx, kvd)[layer, pos]
    got_v = vc.view(np.uint16).reshape(2, ctx, kvd)[layer, pos]
    assert np.array_equal(got_k, [O.float_to_half(float(x)) for x in k])
    assert np.array_equal(got_v, [O.float_to_half(float(x)) for x in v])


def _session(name, tmp):
    spec = synth.preset(name)
    path = synth.model_path(spec, tmp)
    return spec, path


@needs_ref
@pytest.mark.parametrize("name", ["pin", "pin_f16", "g6"])
def test_decode_steps_bit_exact(tmp_path_factory, name):
    """Whole decode steps: embedding input, token input with logits, the KV cache (g6: groups of 6
    query heads per KV head)."""
    spec, path = _session(name, tmp_path_factory.mktemp("pin"))
    ref = R.RefEngine(path, 48)
    om = O.OracleModel(path)
    st = O.OracleState(om, 48)
    k, v = synth.kv_prefill(spec, 20)
    ref.write_kv(k, v)
    st.write_kv(k, v)
    for h in synth.hidden_inputs(spec, 2):
        ref.decode_embedding(h)
        st.decode_embedding(h)
        assert bits_equal(ref.output(), st.output()), f"{name}: embedding step"
    for t in synth.token_ids(spec, 2):
        ref.decode_token(int(t), want_logits=True)
        st.decode_token(int(t), want_logits=True)
        assert bits_equal(ref.output(), st.output()), f"{name}: token step"
        assert bits_equal(ref.logits, st.logits()), f"{name}: logits"
    rk, rv = ref.read_kv(24)
    ok, ov = st.read_kv(24)
    assert np.array_equal(rk, ok) and np.array_equal(rv, ov), f"{name}: KV cache"
    st.close()
    om.close()


def test_oracle_matches_reference_golden(tmp_path_factory):
    """The committed outputs of the reference shaders (tests/golden/make_ref_pin.py) against the
    oracle: the pin without the reference checkout."""
    from golden.make_ref_pin import MODELS, run_session
    g = np.load(GOLDEN)
    d = tmp_path_factory.mktemp("golden")
    for name in MODELS:
        spec = synth.preset(name)
        path = synth.model_path(spec, d)
        import hashlib
        assert hashlib.sha256(path.read_bytes()).hexdigest() == str(g[f"{name}_sha256"]), \
            f"{name}: the synthetic model generator changed; regenerate the golden vectors"
        om = O.OracleModel(path)
        st = O.OracleState(om, 48)
        outs = run_session(spec, st)
        for i, (h, lg) in enumerate(outs):
            assert bits_equal(h, g[f"{name}_hidden"][i]), f"{name}: step {i} hidden"
            if lg is not None:
                assert bits_equal(lg, g[f"{name}_logits"][i - 2]), f"{name}: step {i} logits"
        st.close()
        om.close()
