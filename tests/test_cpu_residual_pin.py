"""Pins the ResidualLM oracle (oracle/residual.py) to the reference's own shaders for the three
operations ResidualLM adds around BaseLM's layers: linear_bias.comp (FSQ's projections),
fsq_quantize.comp and fusion_linear.comp, compiled as C++ by oracle/ref_shim and dispatched as
ResidualFsqEngine records them (src/acoustic.rs:921-966). Bit-exact, like test_cpu_ref_pin.py.
Also checks the oracle's ResidualLM step end to end on a synthetic acoustic GGUF (shapes,
determinism, FSQ on and off)."""
import numpy as np
import pytest

from oracle import ref as R
from oracle import residual as RS
from voxgen_b200 import synth

needs_ref = pytest.mark.skipif(not R.available(), reason="reference shaders not available here")


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def model_words(*parts):
    """One model buffer holding the parts back to back (4-byte aligned); returns the uint32
    words and each part's byte offset."""
    offs, chunks, off = [], [], 0
    for p in parts:
        b = np.ascontiguousarray(p).view(np.uint8).reshape(-1)
        b = np.concatenate([b, np.zeros((-b.size) % 4, np.uint8)])
        offs.append(off)
        chunks.append(b)
        off += b.size
    return np.concatenate(chunks).view(np.uint32).copy(), offs


@needs_ref
@pytest.mark.parametrize("rows,cols", [(64, 256), (37, 300), (256, 64)])
def test_linear_bias_matches_reference(rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    b = (rng.standard_normal(rows) * 0.02).astype(np.float16)
    x = rng.standard_normal(cols).astype(np.float32)
    mw, (ow, ob) = model_words(w, b)
    y = np.zeros(rows, np.float32)
    # LinearBiasPush: weight_offset, bias_offset, rows, cols, weight_dtype, bias_dtype, row_base, alpha
    R.dispatch("linear_bias", [mw, x.copy(), y], R.push("IIIIIIIf", ow, ob, rows, cols, 1, 1, 0, 1.0), [rows])
    got = RS.linear_bias(1, w.view(np.uint8), rows, cols, x, b.astype(np.float32))
    assert bits_equal(got, y)


@needs_ref
def test_fsq_quantize_matches_reference():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(500).astype(np.float32) * 2.0,
                        np.array([0.0, -0.0, 1e-8, 40.0, -40.0, 0.5, -0.5], np.float32)])
    for scale in (9.0, 1.0, 0.375):
        y = x.copy()
        R.dispatch("fsq_quantize", [y], R.push("If", x.size, scale), [(x.size + 255) // 256])
        assert bits_equal(RS.fsq_quantize(x, scale), y)


@needs_ref
def test_fusion_matches_reference():
    rng = np.random.default_rng(11)
    rows, left_cols = 48, 128
    w = (rng.standard_normal((rows, 2 * left_cols)) * 0.02).astype(np.float16)
    b = (rng.standard_normal(rows) * 0.02).astype(np.float16)
    left = rng.standard_normal(left_cols).astype(np.float32)
    right = rng.standard_normal(left_cols).astype(np.float32)
    mw, (ow, ob) = model_words(w, b)
    y = np.zeros(rows, np.float32)
    snap = np.zeros(rows, np.float32)
    # FusionPush: weight_offset, bias_offset, rows, left_cols, right_cols, weight_dtype, bias_dtype, row_base
    R.dispatch("fusion_linear", [mw, left.copy(), right.copy(), y, snap],
               R.push("IIIIIIII", ow, ob, rows, left_cols, left_cols, 1, 1, 0), [rows])
    got = RS.fusion(1, w.view(np.uint8), rows, left, right, b.astype(np.float32))
    assert bits_equal(got, y) and bits_equal(got, snap)


def test_oracle_residual_step_shapes_and_determinism(tmp_path):
    aspec = synth.acoustic_preset("res_tiny")
    ap = synth.acoustic_model_path(aspec, tmp_path)
    bp = synth.model_path(aspec.base, tmp_path)
    h = synth.hidden_inputs(aspec.base, 4)
    outs = []
    for _ in range(2):
        o = RS.ResidualOracle(ap, bp, 8)
        o.step(h[0], None, fsq_applied=False)   # text prefix: the raw hidden is the LM state
        assert np.array_equal(o.current_lm, h[0])
        o.step(h[1], h[2], fsq_applied=True)    # audio: FSQ(hidden) is the LM state
        assert np.array_equal(o.current_lm, o.fsq_output)
        # FSQ output is an affine image of a lattice: out_proj(q / scale) + bias, q integer in
        # [-scale, scale] after tanh
        assert o.position == 2 and np.all(np.isfinite(o.output()))
        outs.append(o.output())
    assert bits_equal(outs[0], outs[1])
