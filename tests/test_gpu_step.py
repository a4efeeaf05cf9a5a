"""Full decode-step parity of the CUDA engine against the oracle, through the C ABI, on the
BASELINE configurations (seeded synthetic models) and small edge-case models."""
import numpy as np
import pytest

from conftest import assert_close, spec_path
from gpu_pair import Pair
from voxgen_b200 import api, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = api.Context(0)
    yield c
    c.close()


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
    """config[1]: 24 layers, F16 embedding table, a 128-token prefill then the config's 256
    decode steps with seeded token ids, every step's final hidden state checked."""
    spec = synth.preset("cfg1")
    p = Pair(ctx, spec_path(model_dir, "cfg1"), 512)
    toks = synth.token_ids(spec, 128 + 256)
    for t in toks[:128]:
        p.step_token(t)
    p.compare("cfg1 after 128-token prefill")
    for i, t in enumerate(toks[128:]):
        p.step_token(t)
        p.compare(f"cfg1 decode step {i}")
    p.compare_kv(384, "cfg1")
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


def outlier_hidden(spec, n, seed_index=2500):
    """N(0,1) hidden states with four "massive activation" channels at +-300 and +-3000 times
    the rms of the rest, as real MiniCPM-class residual streams carry."""
    hs = synth.hidden_inputs(spec, n, seed_index=seed_index)
    ch = np.random.default_rng([spec.seed, seed_index]).choice(spec.hidden, 4, replace=False)
    hs[:, ch] = np.array([300.0, -300.0, 3000.0, -3000.0], np.float32)
    return hs


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_backbone_outlier_channels(ctx, model_dir, name):
    """config[2]/[3] steps whose input hidden state has outlier channels 300x and 3000x the rms
    of the others. They stay in the residual stream through every layer, so every RMSNorm
    operand h*w carries them, and they set the activation's power of two in every matvec
    prologue while the other elements are 3-4 orders of magnitude smaller."""
    spec = synth.preset(name)
    p = Pair(ctx, spec_path(model_dir, name), 2048)
    k, v = synth.kv_prefill(spec, 1023)
    p.write_kv(k, v)
    for i, h in enumerate(outlier_hidden(spec, 3)):
        p.step_embedding(h)
        p.compare(f"{name} outlier step {i}")
    p.close()


@pytest.mark.parametrize("name", ["tiny", "tiny_f16", "pin", "g6"])
def test_attention_merge_long_context(ctx, model_dir, name):
    """Contexts long enough that the attention units outnumber the CTAs left free for the merge
    slices (tiny: 188 units on 148 CTAs, so some CTAs run two units and the last eight run a
    unit and then a slice), and that a slice loads its chunks' rows in more than one batch
    (pin: 94 chunks of one KV head at head_dim 128, 64 rows per batch); g6: groups of 6 query
    heads, which fill 6 of a unit's 8 head columns."""
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


def test_decode_batch_matches_single_streams(ctx, model_dir, monkeypatch):
    """vg_decode_batch without the batched kernel (VOXGEN_BATCH_KERNEL=0): each stream takes its
    own step, bitwise the same as a stream decoded alone (ragged positions)."""
    monkeypatch.setenv("VOXGEN_BATCH_KERNEL", "0")
    spec = synth.preset("tiny")
    path = spec_path(model_dir, "tiny")
    m = api.Model(ctx, path)
    assert m.batch_columns == 0
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


@pytest.mark.parametrize("name,prefill", [("pin", 300), ("cfg2", 1500)])
def test_matches_xtx_mode_oracle(ctx, model_dir, name, prefill):
    """The same tolerance against the reference's RX 7900 XTX mode (the _xtx7900 shaders'
    wave32 summation order, restated by the oracle and pinned to those shaders in
    test_cpu_ref_pin_xtx.py): one CUDA result is within tolerance of a reference run in either
    mode."""
    spec = synth.preset(name)
    p = Pair(ctx, spec_path(model_dir, name), prefill + 8, xtx=True)
    k, v = synth.kv_prefill(spec, prefill)
    p.write_kv(k, v)
    for i, t in enumerate(synth.token_ids(spec, 3, seed_index=88)):
        p.step_token(t)
        p.compare(f"{name} XTX-mode step {i}")
    p.close()
