"""CPU checks of the oracle: fp16 conversions, reference known-answer tests, and agreement with an
independent float64 restatement of the decode step."""
import numpy as np
import pytest

from conftest import spec_path
from oracle import oracle as O
from voxgen_b200 import api, gguf, synth


def test_half_to_float_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([O.half_to_float(int(b)) for b in bits], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.isnan(got[~finite & np.isnan(want)]).all()
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])


def test_float_to_half_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-8, 5, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.9, 65520.0, 1e6, -1e6, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -26, 2.0 ** -14, 6.1e-5, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32)])
    want = x.astype(np.float16).view(np.uint16)
    got = np.array([O.float_to_half(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, want)


def test_reference_kats():
    # effective_scale: src/baselm.rs:1320-1323 (0 means identity); exercised through the
    # oracle's embedding alpha below. kv_bytes_match_packed_f16_layout: src/baselm.rs:1332-1358.
    info = dict(block_count=28, kv_dim=256)
    assert api.kv_cache_bytes(info, 32768) == 939_524_096
    assert api.kv_cache_bytes(info, 32768) // 2 == 469_762_048
    # top_k_is_descending: src/baselm.rs:1326-1329
    got = api.top_k_logits(np.array([1.0, -2.0, 5.0, 3.0], np.float32), 3)
    assert [t.token_id for t in got] == [2, 3, 0]
    # non-finite logits are dropped (src/baselm.rs:1300)
    got = api.top_k_logits(np.array([np.nan, 1.0, np.inf, -np.inf, 0.5], np.float32), 5)
    assert [t.token_id for t in got] == [1, 4]
    # Q8_0 storage: 34 bytes per 32 elements (src/gguf.rs:41-45)
    assert gguf.storage_bytes(gguf.GGML_Q8_0, 2048 * 6144) == 2048 * 6144 // 32 * 34
    with pytest.raises(ValueError):
        gguf.storage_bytes(gguf.GGML_Q8_0, 33)


def test_q8_dequant_matches_reference_formula():
    rng = np.random.default_rng(3)
    raw = synth.q8_matrix(rng, 3, 64)
    d, qs = gguf.q8_0_unpack(raw, 3, 64)
    for r in range(3):
        for c in (0, 1, 31, 32, 63):
            # embedding.comp:33-40: d * float(q) with d = unpackHalf2x16(scale)
            want = np.float32(np.float32(d[r, c // 32]) * np.float32(qs[r, c]))
            got = O.embedding(gguf.GGML_Q8_0, raw, 64, r)[c]
            assert got == want


def _numpy_decode(g, spec, h0, k, v, pos):
    """float64 restatement of record_transformer (src/baselm.rs:892-1052)."""
    H, L, nh, nkv, d = spec.hidden, spec.layers, spec.heads, spec.kv_heads, spec.head_dim
    W = lambda n: g.matrix_f32(n).astype(np.float64)

    def rms(x, w):
        return x / np.sqrt(np.mean(x * x) + spec.eps) * w

    Kf = np.zeros((L, pos + 1, nkv * d))
    Vf = np.zeros_like(Kf)
    Kf[:, :pos] = k.view(np.float16).astype(np.float64)
    Vf[:, :pos] = v.view(np.float16).astype(np.float64)
    h = h0.astype(np.float64)
    x = rms(h, W("blk.0.attn_norm.weight"))
    i = np.arange(d // 2)
    ang = pos * (1.0 / spec.theta ** (2 * i / d))
    c, s = np.cos(ang), np.sin(ang)

    def rope(z):
        z = z.reshape(-1, d).copy()
        a, b = z[:, :d // 2].copy(), z[:, d // 2:].copy()
        z[:, :d // 2] = a * c - b * s
        z[:, d // 2:] = b * c + a * s
        return z.reshape(-1)

    for l in range(L):
        q = rope(W(f"blk.{l}.attn_q.weight") @ x)
        kk = rope(W(f"blk.{l}.attn_k.weight") @ x)
        vv = W(f"blk.{l}.attn_v.weight") @ x
        Kf[l, pos] = kk.astype(np.float16)
        Vf[l, pos] = vv.astype(np.float16)
        att = np.zeros(H)
        for hh in range(nh):
            gi = hh // (nh // nkv)
            sc = Kf[l, :, gi * d:(gi + 1) * d] @ q[hh * d:(hh + 1) * d] / np.sqrt(d)
            p = np.exp(sc - sc.max())
            att[hh * d:(hh + 1) * d] = (p / p.sum()) @ Vf[l, :, gi * d:(gi + 1) * d]
        h = h + W(f"blk.{l}.attn_output.weight") @ att
        x = rms(h, W(f"blk.{l}.ffn_norm.weight"))
        gg = W(f"blk.{l}.ffn_gate.weight") @ x
        uu = W(f"blk.{l}.ffn_up.weight") @ x
        h = h + W(f"blk.{l}.ffn_down.weight") @ (gg / (1 + np.exp(-gg)) * uu)
        x = rms(h, W(f"blk.{l + 1}.attn_norm.weight" if l + 1 < L else "output_norm.weight"))
    return x, Kf[:, pos], Vf[:, pos]


@pytest.mark.parametrize("name", ["tiny", "tiny_f16"])
def test_oracle_matches_float64_restatement(model_dir, name):
    spec = synth.preset(name)
    path = spec_path(model_dir, name)
    g = gguf.read_gguf(path)
    m = O.OracleModel(path)
    st = O.OracleState(m, 64)
    k, v = synth.kv_prefill(spec, 10)
    st.write_kv(k, v)
    h0 = synth.hidden_inputs(spec, 1)[0]
    st.decode_embedding(h0)
    want, kpos, vpos = _numpy_decode(g, spec, h0, k, v, 10)
    got = st.output()
    assert np.max(np.abs(got - want)) < 1e-5
    kk, vv = st.read_kv(11)
    # fp16 stores of the new position agree except where the float64 and fp32 values
    # straddle a rounding boundary (at most one unit in the last place)
    dk = np.abs(kk[:, 10].astype(np.int32) - kpos.astype(np.float16).view(np.uint16).astype(np.int32))
    dv = np.abs(vv[:, 10].astype(np.int32) - vpos.astype(np.float16).view(np.uint16).astype(np.int32))
    assert dk.max() <= 1 and dv.max() <= 1
    assert (dk == 0).mean() > 0.98 and (dv == 0).mean() > 0.98


def test_oracle_errors(model_dir):
    path = spec_path(model_dir, "tiny")
    m = O.OracleModel(path)
    st = O.OracleState(m, 4)
    with pytest.raises(O.OracleError) as e:
        st.decode_token(10_000)
    assert e.value.code == -5
    for t in range(4):
        st.decode_token(t)
    with pytest.raises(O.OracleError) as e:
        st.decode_token(0)
    assert e.value.code == -6
    st.reset()
    assert st.position == 0
