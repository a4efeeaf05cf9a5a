"""The RX 7900 XTX mode (the reference's _xtx7900 shader variants) against the oracle.

In that mode GpuContext::select_spirv swaps rmsnorm, residual_rmsnorm, qkv_matvec,
matvec_swiglu, matvec, attn_scores and softmax for their _xtx7900 files (baselm.rs:515-546,
:1241). Those files change the summation order: a lane sums 4 consecutive columns every 1024
(matvec_xtx7900.comp:14-15), and a workgroup sum is a wave32 subgroupAdd per wave, then one more
subgroupAdd over the waves' sums. GLSL does not fix the order inside subgroupAdd; the shader
emulation (oracle/ref_shim) and the oracle both take the balanced pairwise tree over the 32
invocations, which is what a shuffle-xor butterfly computes.

- The oracle's XTX restatement is pinned bit-exactly to the emulated shaders, kernel by kernel
  and over whole decode steps, and to committed golden vectors (tests/golden/ref_shader_pin_xtx.npz,
  written by tests/golden/make_ref_pin.py --xtx).
- The two modes are then compared over whole decode steps. This is what the CUDA path's parity
  tolerance (2e-3 absolute, 1e-3 relative) has to cover, measured instead of argued.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from oracle import ref as R
from test_cpu_ref_pin import MATS, bits_equal, words
from voxgen_b200 import synth

needs_ref = pytest.mark.skipif(not R.available(), reason="reference shaders not available here")
GOLDEN = Path(__file__).resolve().parent / "golden" / "ref_shader_pin_xtx.npz"


@needs_ref
@pytest.mark.parametrize("dtype", [8, 1])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (37, 1024), (5, 4096), (3, 2080)])
def test_matvec_and_swiglu_xtx_shaders(dtype, rows, cols):
    rng = np.random.default_rng(rows * 11 + cols + dtype)
    w = MATS[dtype](rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    R.dispatch("matvec_xtx7900", [words(w), x, y], R.push("IIIIIf", 0, rows, cols, dtype, 0, 0.75), [rows])
    assert bits_equal(y, O.matvec(dtype, w, rows, cols, x, 0.75, xtx=True)), "matvec_xtx7900.comp"
    u = MATS[dtype](rng, rows, cols)
    g = np.zeros(rows, np.float32)
    R.dispatch("matvec_swiglu_xtx7900", [words(np.concatenate([w, u])), x, g],
               R.push("IIIIII", 0, w.size, rows, cols, dtype, 0), [rows])
    assert bits_equal(g, O.swiglu(dtype, w, u, rows, cols, x, xtx=True)), "matvec_swiglu_xtx7900.comp"


@needs_ref
@pytest.mark.parametrize("n", [64, 1000, 2048])
def test_norm_xtx_shaders(n):
    rng = np.random.default_rng(n + 3)
    x = rng.standard_normal(n).astype(np.float32)
    br = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(n)).astype(np.float32)
    y = np.zeros(n, np.float32)
    R.dispatch("rmsnorm_xtx7900", [words(w.view(np.uint8)), x.copy(), y], R.push("IIf", 0, n, 1e-5), [1])
    assert bits_equal(y, O.rmsnorm(x, w, 1e-5, xtx=True)), "rmsnorm_xtx7900.comp"
    h = x.copy()
    R.dispatch("residual_rmsnorm_xtx7900", [words(w.view(np.uint8)), h, br, y],
               R.push("IIff", 0, n, 1e-5, 0.25), [1])
    oh, oy = O.residual_rmsnorm(x, br, w, 1e-5, 0.25, xtx=True)
    assert bits_equal(h, oh) and bits_equal(y, oy), "residual_rmsnorm_xtx7900.comp"


@needs_ref
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("position", [0, 5, 300])
def test_attention_xtx_shaders(D, position):
    """attn_scores_xtx7900 (128 lanes, one dimension each) and softmax_xtx7900, then the
    unchanged attn_values."""
    heads, kv_heads, ctx = 16, 2, 320
    kvd = kv_heads * D
    rng = np.random.default_rng(D * 100 + position)
    q = rng.standard_normal(heads * D).astype(np.float32)
    kc = rng.standard_normal((ctx, kvd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((ctx, kvd)).astype(np.float16).view(np.uint16)
    scores = np.zeros(heads * ctx, np.float32)
    out = np.zeros(heads * D, np.float32)
    push = R.push("IIIIII", 0, ctx, position, D, heads // kv_heads, kv_heads)
    R.dispatch("attn_scores_xtx7900", [q, words(kc.view(np.uint8)), scores], push, [position + 1, heads])
    R.dispatch("softmax_xtx7900", [scores], R.push("II", ctx, position), [heads])
    R.dispatch("attn_values", [scores, words(vc.view(np.uint8)), out], push, [heads])
    want, wscores = O.attention(q, kc, vc, heads, kv_heads, D, position, xtx=True)
    sl = np.s_[:, :position + 1]
    assert bits_equal(scores.reshape(heads, ctx)[sl], wscores[sl]), "attn_scores_xtx7900 + softmax_xtx7900"
    assert bits_equal(out, want), "attn_values.comp after the XTX softmax"


@needs_ref
@pytest.mark.parametrize("name", ["pin", "pin_f16", "g6"])
def test_decode_steps_xtx_bit_exact(tmp_path_factory, name):
    """Whole XTX-mode decode steps (embedding and token inputs, logits, KV cache) on the
    emulated shaders and on the oracle."""
    from golden.make_ref_pin import CONTEXT, run_session
    spec = synth.preset(name)
    path = synth.model_path(spec, tmp_path_factory.mktemp("xtx"))
    ref = R.RefEngine(path, CONTEXT, xtx=True)
    om = O.OracleModel(path)
    st = O.OracleState(om, CONTEXT, xtx=True)
    for i, ((rh, rl), (oh, ol)) in enumerate(zip(run_session(spec, ref), run_session(spec, st))):
        assert bits_equal(rh, oh), f"{name}: step {i} hidden"
        if rl is not None:
            assert bits_equal(rl, ol), f"{name}: step {i} logits"
    rk, rv = ref.read_kv(24)
    ok, ov = st.read_kv(24)
    assert np.array_equal(rk, ok) and np.array_equal(rv, ov), f"{name}: KV cache"
    st.close()
    om.close()


def test_oracle_xtx_matches_reference_golden(tmp_path_factory):
    """The committed XTX-mode outputs of the emulated reference shaders against the oracle's
    XTX restatement: the pin without the reference checkout."""
    from golden.make_ref_pin import CONTEXT, MODELS, run_session
    g = np.load(GOLDEN)
    d = tmp_path_factory.mktemp("golden_xtx")
    for name in MODELS:
        spec = synth.preset(name)
        path = synth.model_path(spec, d)
        assert hashlib.sha256(path.read_bytes()).hexdigest() == str(g[f"{name}_sha256"]), \
            f"{name}: the synthetic model generator changed; regenerate the golden vectors"
        om = O.OracleModel(path)
        st = O.OracleState(om, CONTEXT, xtx=True)
        for i, (h, lg) in enumerate(run_session(spec, st)):
            assert bits_equal(h, g[f"{name}_hidden"][i]), f"{name}: step {i} hidden"
            if lg is not None:
                assert bits_equal(lg, g[f"{name}_logits"][i - 2]), f"{name}: step {i} logits"
        st.close()
        om.close()


@pytest.mark.parametrize("name,prefill,steps", [("pin", 300, 6), ("cfg1", 128, 4)])
def test_normal_and_xtx_orders_agree(tmp_path_factory, name, prefill, steps):
    """The two modes' summation orders over whole decode steps: the gap between them must sit
    well inside the CUDA path's parity tolerance (2e-3 absolute + 1e-3 relative), so one
    tolerance covers a reference run in either mode. Measured here at a quarter of it."""
    spec = synth.preset(name)
    path = synth.model_path(spec, tmp_path_factory.mktemp("modes"))
    om = O.OracleModel(path)
    ctx = prefill + steps + 1
    a, b = O.OracleState(om, ctx), O.OracleState(om, ctx, xtx=True)
    k, v = synth.kv_prefill(spec, prefill)
    a.write_kv(k, v)
    b.write_kv(k, v)
    worst = 0.0
    for t in synth.token_ids(spec, steps, seed_index=77):
        a.decode_token(int(t))
        b.decode_token(int(t))
        x, y = a.output(), b.output()
        excess = np.abs(x - y) - 0.25 * (2e-3 + 1e-3 * np.abs(x))
        worst = max(worst, float(np.abs(x - y).max()))
        assert excess.max() <= 0, f"{name}: normal vs XTX order differ by {np.abs(x - y).max():.3g}"
    print(f"{name}: largest normal-vs-XTX difference over {steps} steps: {worst:.3g}")
    a.close()
    b.close()
    om.close()
