"""Full decode-step parity of the CUDA engine against the oracle, through the C ABI, on the
BASELINE configurations (seeded synthetic models) and small edge-case models."""
from dataclasses import replace

import numpy as np
import pytest

from conftest import assert_close, spec_path
from oracle import oracle as O
from voxgen_b200 import api, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = api.Context(0)
    yield c
    c.close()


def _ordinal(bits):
    """fp16 bit patterns mapped to integers that are monotonic in the value."""
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


class Pair:
    """The same session on the CUDA engine and on the oracle."""

    def __init__(self, ctx, path, max_context):
        self.model = api.Model(ctx, path)
        self.eng = api.BaseLmEngine(self.model, max_context)
        self.om = O.OracleModel(path)
        self.ost = O.OracleState(self.om, max_context)

    def write_kv(self, k, v):
        self.eng.write_kv(k, v)
        self.ost.write_kv(k, v)

    def step_embedding(self, h, logits=False):
        self.eng.decode_embedding_gpu_only(h, want_logits=logits)
        self.ost.decode_embedding(h, want_logits=logits)

    def step_token(self, t, logits=False):
        self.eng.decode_token_gpu_only(int(t), want_logits=logits)
        self.ost.decode_token(int(t), want_logits=logits)

    def compare(self, what):
        assert self.eng.position == self.ost.position
        assert_close(self.eng.output(), self.ost.output(), what=what)

    def compare_kv(self, n, what):
        ke, ve = self.eng.read_kv(n)
        ko, vo = self.ost.read_kv(n)
        for a, b, name in ((ke, ko, "K"), (ve, vo, "V")):
            fa = a.view(np.float16).astype(np.float32)
            fb = b.view(np.float16).astype(np.float32)
            assert_close(fa, fb, what=f"{what} {name} cache")
            # Layer 0 projects bit-identical inputs (the embedding lookup is exact), so its
            # fp16 stores of ordinary-magnitude values are at most one unit in the last place
            # apart; deeper layers carry accumulated fp32 differences and are held to the
            # value tolerance above.
            big = np.abs(fb[0]) >= 1e-2
            diff = np.abs(_ordinal(a[0]) - _ordinal(b[0]))[big]
            assert diff.max(initial=0) <= 1, f"{what} {name} layer 0: fp16 values {diff.max()} ulp apart"

    def close(self):
        self.eng.close()
        self.model.close()


@pytest.mark.parametrize("name", ["tiny", "tiny_f16"])
def test_tiny_steps(ctx, model_dir, name):
    spec = synth.preset(name)
    p = Pair(ctx, spec_path(model_dir, name), 64)
    k, v = synth.kv_prefill(spec, 10)
    p.write_kv(k, v)
    hs = synth.hidden_inputs(spec, 4)
    for i in range(4):
        p.step_embedding(hs[i])
        p.compare(f"{name} embedding step {i}")
    for t in synth.token_ids(spec, 4):
        p.step_token(t)
        p.compare(f"{name} token step")
    p.compare_kv(18, name)
    p.close()


def test_position_zero_and_reset_determinism(ctx, model_dir):
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 32)
    toks = synth.token_ids(spec, 5)
    outs = []
    for t in toks:
        p.step_token(t)
        p.compare("from position 0")
        outs.append(p.eng.output())
    p.eng.reset()
    p.ost.reset()
    assert p.eng.position == 0
    for i, t in enumerate(toks):
        p.step_token(t)
        assert np.array_equal(p.eng.output(), outs[i]), "replay after reset is not bitwise identical"
    p.close()


def test_scales_untied_logits_topk(ctx, model_dir):
    spec = synth.preset("tiny", tied_output=False, embedding_scale=12.0, residual_scale=0.25, logit_scale=0.125,
                        seed=21)
    path = synth.model_path(spec, model_dir)
    p = Pair(ctx, path, 16)
    for t in synth.token_ids(spec, 3):
        p.step_token(t, logits=True)
        p.compare("scaled model")
        assert_close(p.eng.logits(), p.ost.logits(), what="logits")
    res = p.eng.decode_token(5, top_k=8)
    p.ost.decode_token(5, want_logits=True)
    ol = p.ost.logits()
    want = np.argsort(-ol, kind="stable")[:8]
    got = [t.token_id for t in res.top_logits]
    assert len(got) == 8
    # the top set agrees except for near-ties within the parity tolerance
    for g, w in zip(got, want):
        assert g == w or abs(ol[g] - ol[w]) <= 2e-3 + 1e-3 * abs(ol[w])
    o = p.ost.output().astype(np.float64)
    assert abs(res.final_hidden_checksum - o.sum()) < 1e-2
    assert abs(res.final_hidden_l2 - np.sqrt((o * o).sum())) < 1e-3 * np.sqrt((o * o).sum())
    p.close()


def test_device_embedding_input(ctx, model_dir):
    import torch
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 16)
    h = synth.hidden_inputs(spec, 1)[0]
    hd = torch.from_numpy(h).cuda()
    torch.cuda.synchronize()
    p.eng.decode_embedding_from_gpu_only(hd.data_ptr())
    p.ost.decode_embedding(h)
    p.compare("device embedding")
    p.close()


def test_errors(ctx, model_dir):
    spec = synth.preset("tiny")
    m = api.Model(ctx, spec_path(model_dir, "tiny"))
    with pytest.raises(api.VoxGenError) as e:
        api.BaseLmEngine(m, spec.context_length + 1)
    assert e.value.code == -1
    eng = api.BaseLmEngine(m, 3)
    with pytest.raises(api.VoxGenError) as e:
        eng.decode_token_gpu_only(spec.vocab)
    assert e.value.code == -5 and "outside vocabulary" in str(e.value)
    for t in range(3):
        eng.decode_token_gpu_only(t)
    with pytest.raises(api.VoxGenError) as e:
        eng.decode_token_gpu_only(0)
    assert e.value.code == -6 and "KV cache is full" in str(e.value)
    with pytest.raises(api.VoxGenError) as e:
        eng.prefill_tokens([])
    eng.sync()
    # model destroy with a live stream is refused; destroyed handles are rejected
    assert api.lib().vg_model_destroy(m.h) == -11
    h = eng.h
    eng.close()
    assert api.lib().vg_stream_reset(h) == -11
    assert api.lib().vg_decode_token(h, 0, 0) == -11
    m.close()


def test_cfg0(ctx, model_dir):
    """config[0]: one Q8_0 layer, H=1024, 512 prior positions, one step at position 512."""
    spec = synth.preset("cfg0")
    p = Pair(ctx, spec_path(model_dir, "cfg0"), 1024)
    k, v = synth.kv_prefill(spec, 512)
    p.write_kv(k, v)
    hs = synth.hidden_inputs(spec, 3)
    for i in range(3):
        p.step_embedding(hs[i])
        p.compare(f"cfg0 step {i}")
    p.compare_kv(515, "cfg0")
    p.close()


def test_cfg1_prefill_and_decode(ctx, model_dir):
    """config[1]: 24 layers, F16 embedding table, token prefill then decode steps."""
    spec = synth.preset("cfg1")
    p = Pair(ctx, spec_path(model_dir, "cfg1"), 512)
    toks = synth.token_ids(spec, 128 + 8)
    for t in toks[:128]:
        p.step_token(t)
    p.compare("cfg1 after 128-token prefill")
    for t in toks[128:]:
        p.step_token(t)
        p.compare("cfg1 decode")
    p.compare_kv(136, "cfg1")
    p.close()


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_backbone_long_context(ctx, model_dir, name):
    """config[2]/[3]: 28 layers, H=2048; steps at 1023-1024 and at the end of a 4096 context."""
    spec = synth.preset(name)
    p = Pair(ctx, spec_path(model_dir, name), 4096)
    k, v = synth.kv_prefill(spec, 4094)
    p.write_kv(k[:, :1023], v[:, :1023])
    hs = synth.hidden_inputs(spec, 4)
    p.step_embedding(hs[0])
    p.compare(f"{name} pos 1023")
    p.step_token(7)
    p.compare(f"{name} pos 1024")
    p.write_kv(k, v)
    p.step_embedding(hs[1])
    p.compare(f"{name} pos 4094")
    p.step_embedding(hs[2])
    p.compare(f"{name} pos 4095")
    with pytest.raises(api.VoxGenError) as e:
        p.eng.decode_embedding_gpu_only(hs[3])
    assert e.value.code == -6
    p.close()


@pytest.mark.parametrize("name", ["tiny", "tiny_f16", "pin"])
def test_attention_merge_long_context(ctx, model_dir, name):
    """Contexts long enough that the attention units outnumber the CTAs left free for the merge
    slices (tiny: 188 units on 148 CTAs, so some CTAs run two units and the last eight run a
    unit and then a slice), and that a slice loads its chunks' rows in more than one batch
    (pin: 94 chunks of one KV head at head_dim 128, 64 rows per batch)."""
    spec = synth.preset(name)
    n = 6000
    p = Pair(ctx, spec_path(model_dir, name), n + 8)
    k, v = synth.kv_prefill(spec, n)
    p.write_kv(k, v)
    hs = synth.hidden_inputs(spec, 3)
    for i in range(3):
        p.step_embedding(hs[i])
        p.compare(f"{name} pos {n + i}")
    p.close()


def test_decode_batch_matches_single_streams(ctx, model_dir):
    """vg_decode_batch: every stream advances as if decoded alone (ragged positions)."""
    spec = synth.preset("tiny")
    path = spec_path(model_dir, "tiny")
    m = api.Model(ctx, path)
    engines = [api.BaseLmEngine(m, 64) for _ in range(3)]
    solo = [api.BaseLmEngine(m, 64) for _ in range(3)]
    for i, (e, s) in enumerate(zip(engines, solo)):
        k, v = synth.kv_prefill(spec, 5 + 7 * i, seed_index=1100 + i)
        e.write_kv(k, v)
        s.write_kv(k, v)
    toks = synth.token_ids(spec, 12).reshape(4, 3)
    for row in toks:
        api.decode_batch(engines, [int(t) for t in row])
        for s, t in zip(solo, row):
            s.decode_token_gpu_only(int(t))
    for e, s in zip(engines, solo):
        assert e.position == s.position
        assert np.array_equal(e.output(), s.output())
    with pytest.raises(api.VoxGenError) as err:
        api.decode_batch([engines[0], engines[0]], [1, 2])
    assert err.value.code == -1
    with pytest.raises(api.VoxGenError) as err:
        api.decode_batch(engines, [1, spec.vocab, 2])
    assert err.value.code == -5
    assert [e.position for e in engines] == [s.position for s in solo], "a failed batch advanced a stream"
    for e in engines + solo:
        e.close()
    m.close()
