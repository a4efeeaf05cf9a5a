"""Entry points of the C ABI beyond the plain decode step, each checked against the oracle:
the LM head as a phase of the step kernel, benchmark, prefill, the per-kernel profiler, seek,
the per-kernel step program (forced, and reached by a model in two weight formats), and failure
detection (a device-side wait that runs out, host waits that time out)."""
import re
import time

import numpy as np
import pytest

from conftest import assert_close, spec_path
from gpu_pair import Pair
from oracle import oracle as O
from voxgen_b200 import api, gguf, synth

pytestmark = pytest.mark.gpu

Q8, F16 = gguf.GGML_Q8_0, gguf.GGML_F16
VG_EINVAL, VG_ERANGE, VG_EFULL, VG_ECUDA, VG_ETIMEDOUT, VG_EDEVICE = -1, -5, -6, -7, -9, -10


@pytest.fixture(scope="module")
def ctx():
    c = api.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("name,over", [
    ("tiny_f16", {}),                                              # F16 layers, tied F16 head
    ("tiny", dict(embd_fmt=Q8)),                                   # Q8_0 layers, tied Q8_0 head
    ("tiny", dict(embd_fmt=Q8, tied_output=False, logit_scale=0.5, seed=23)),  # untied Q8_0 head
])
def test_lm_head_in_step_kernel(ctx, model_dir, name, over):
    """Logits from the step kernel's own LM-head phase (the head shares the layers' format, so it
    is not the separate launch a head of another format takes), with top-k."""
    spec = synth.preset(name, **over)
    p = Pair(ctx, synth.model_path(spec, model_dir), 32)
    assert p.eng.kernel_mode == 1
    for t in synth.token_ids(spec, 4, seed_index=3100):
        p.step_token(t, logits=True)
        p.compare(f"{name} {over} output")
        assert_close(p.eng.logits(), p.ost.logits(), what=f"{name} {over} logits")
    h = synth.hidden_inputs(spec, 1)[0]
    p.step_embedding(h, logits=True)
    assert_close(p.eng.logits(), p.ost.logits(), what=f"{name} {over} logits after an embedding step")
    p.close()


def test_benchmark(ctx, model_dir):
    """vg_benchmark (BaseLmEngine::benchmark, src/baselm.rs:841-880): reset, warm-up and timed
    token steps; the stream then holds the state of warmup + iterations identical steps."""
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 32)
    r = p.eng.benchmark(token_id=5, warmup=2, iterations=6, want_logits=True)
    assert r["iterations"] == 6 and r["token_id"] == 5
    assert 0 < r["min_ms"] <= r["mean_ms"] <= r["max_ms"]
    assert abs(r["tokens_per_second"] - 1000.0 / r["mean_ms"]) <= 1e-9 * r["tokens_per_second"]
    assert p.eng.position == 8
    for _ in range(8):
        p.ost.decode_token(5, want_logits=True)
    p.compare("after benchmark")
    assert_close(p.eng.logits(), p.ost.logits(), what="benchmark logits")
    for warm, iters, code in ((0, 0, VG_EINVAL), (30, 3, VG_EFULL)):
        with pytest.raises(api.VoxGenError) as e:
            p.eng.benchmark(token_id=5, warmup=warm, iterations=iters)
        assert e.value.code == code
    p.close()


@pytest.mark.parametrize("name,n0,n", [("tiny", 5, 20), ("tiny_f16", 0, 1), ("cfg1", 0, 128)])
def test_prefill_tokens(ctx, model_dir, name, n0, n):
    """vg_prefill_tokens (prefill_tokens, src/baselm.rs:823-839) after n0 cached positions: final
    hidden state, logits of the last position and top-k, and the KV rows it wrote."""
    spec = synth.preset(name)
    p = Pair(ctx, spec_path(model_dir, name), n0 + n + 8)
    if n0:
        k, v = synth.kv_prefill(spec, n0)
        p.write_kv(k, v)
    toks = synth.token_ids(spec, n, seed_index=3200)
    res = p.eng.prefill_tokens([int(t) for t in toks], top_k_last=8)
    for i, t in enumerate(toks):
        p.ost.decode_token(int(t), want_logits=i == n - 1)
    assert res.position == n0 + n - 1 and p.eng.position == n0 + n
    p.compare(f"{name} after a {n}-token prefill")
    ol = p.ost.logits()
    assert_close(p.eng.logits(), ol, what=f"{name} prefill logits")
    want = np.argsort(-ol, kind="stable")[:8]
    for g, w in zip([t.token_id for t in res.top_logits], want):
        assert g == w or abs(ol[g] - ol[w]) <= 2e-3 + 1e-3 * abs(ol[w])
    p.compare_kv(n0 + n, f"{name} prefill")
    p.close()


def test_profile_step(ctx, model_dir):
    """vg_stream_profile_step: one token step with every kernel timed on its own; the step is a
    real one (position, output) and the launches are the record_transformer sequence."""
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 32)
    k, v = synth.kv_prefill(spec, 6)
    p.write_kv(k, v)
    rows = p.eng.profile_step(9, want_logits=True)
    p.ost.decode_token(9, want_logits=True)
    L = spec.layers
    names = [r["name"] for r in rows]
    assert names == ["embedding"] + ["qkv", "attention", "o_proj", "gate_up", "down"] * L + ["final_norm", "logits"]
    assert [r["layer"] for r in rows[1:-2]] == [l for l in range(L) for _ in range(5)]
    assert all(r["ms"] > 0 for r in rows)
    H, F, KV = spec.hidden, spec.ffn, spec.kv_dim
    q8row = lambda cols: cols // 32 * 34
    by = {(r["name"], r["layer"]): r["bytes"] for r in rows}
    assert by[("gate_up", 0)] == q8row(H) * 2 * F + H * 4
    assert by[("down", 1)] == q8row(F) * H
    assert by[("attention", 0)] == 2 * KV * 2 * 7      # K and V rows of positions 0..6
    assert p.eng.position == 7
    p.compare("profiled step")
    assert_close(p.eng.logits(), p.ost.logits(), what="profiled step logits")
    p.close()


def test_seek(ctx, model_dir):
    """vg_stream_seek moves the position over a kept cache; the next step attends over the rows
    below it and overwrites the row at it."""
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 40)
    k, v = synth.kv_prefill(spec, 20)
    p.write_kv(k, v)
    for pos in (12, 3, 19, 0):
        p.eng.seek(pos)
        p.ost.set_position(pos)
        assert p.eng.position == pos
        p.step_token(7 + pos)
        p.compare(f"step after seeking to {pos}")
    with pytest.raises(api.VoxGenError) as e:
        p.eng.seek(41)
    assert e.value.code == VG_EINVAL
    p.eng.seek(40)
    with pytest.raises(api.VoxGenError) as e:
        p.eng.decode_token_gpu_only(1)
    assert e.value.code == VG_EFULL
    p.close()


@pytest.mark.parametrize("name", ["tiny", "tiny_f16", "cfg2"])
def test_per_kernel_program(ctx, model_dir, monkeypatch, name):
    """The step as one launch per projection / attention / norm (VOXGEN_STEP_KERNEL=0), the
    program a stream runs when the persistent kernel is unavailable: token and embedding steps,
    logits, and at cfg2 the positions around 1024."""
    monkeypatch.setenv("VOXGEN_STEP_KERNEL", "0")
    spec = synth.preset(name)
    p = Pair(ctx, spec_path(model_dir, name), 1100)
    assert p.eng.kernel_mode == 0
    n0 = 1022 if name == "cfg2" else 9
    k, v = synth.kv_prefill(spec, n0)
    p.write_kv(k, v)
    hs = synth.hidden_inputs(spec, 2)
    p.step_embedding(hs[0])
    p.compare(f"{name} per-kernel embedding step")
    for t in synth.token_ids(spec, 2, seed_index=3300):
        p.step_token(t, logits=name != "cfg2")
        p.compare(f"{name} per-kernel token step")
        if name != "cfg2":
            assert_close(p.eng.logits(), p.ost.logits(), what=f"{name} per-kernel logits")
    p.step_embedding(hs[1])
    p.compare(f"{name} per-kernel embedding step at {p.eng.position - 1}")
    p.compare_kv(n0 + 4, f"{name} per-kernel")
    p.close()


def test_mixed_format_model(ctx, model_dir):
    """A Q8_0 model whose down projections are F16: the persistent kernel needs one format for
    every projection, so the stream runs the per-kernel program, and matches the oracle."""
    spec = synth.preset("tiny_mixed")
    p = Pair(ctx, spec_path(model_dir, "tiny_mixed"), 32)
    assert p.eng.kernel_mode == 0
    k, v = synth.kv_prefill(spec, 4)
    p.write_kv(k, v)
    p.step_embedding(synth.hidden_inputs(spec, 1)[0])
    p.compare("mixed-format embedding step")
    for t in synth.token_ids(spec, 3, seed_index=3400):
        p.step_token(t, logits=True)
        p.compare("mixed-format token step")
        assert_close(p.eng.logits(), p.ost.logits(), what="mixed-format logits")
    p.close()


def _flag(err):
    m = re.search(r"device error flag 0x([0-9a-f]+)", str(err))
    assert m, str(err)
    return int(m.group(1), 16)


def test_device_wait_runs_out(ctx, model_dir):
    """A step whose grid barrier can never complete (vg_test_stalled_step) with the device wait
    limit cut to 50 us: the waiting CTA gives up, the others see the error flag and leave, the
    host gets VG_EDEVICE with the grid-wait bit, and the stream then decodes normally again."""
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 32)
    k, v = synth.kv_prefill(spec, 10)
    p.write_kv(k, v)
    p.eng.set_wait_limit(50e-6)
    t0 = time.perf_counter()
    assert api.lib().vg_test_stalled_step(p.eng.h, 3) == 0
    with pytest.raises(api.VoxGenError) as e:
        p.eng.sync()
    elapsed = time.perf_counter() - t0
    assert e.value.code == VG_EDEVICE
    assert _flag(e.value) & 0x20, "the grid-barrier wait did not report running out"
    assert elapsed < 1.0, f"the failed step took {elapsed:.3f} s; its waits did not end at the limit"
    assert p.eng.position == 11
    p.eng.sync()                     # the flag was cleared with the report
    p.eng.set_wait_limit(0)          # back to the 2 s default
    p.write_kv(k, v)                 # restore the cache row the failed step overwrote
    for t in synth.token_ids(spec, 3, seed_index=3500):
        p.step_token(t)
        p.compare("step after a failed step")
    with pytest.raises(api.VoxGenError) as e:
        p.eng.set_wait_limit(5.0)    # above the 32-bit nanosecond field
    assert e.value.code == VG_EINVAL
    p.close()


def test_host_waits_time_out(ctx, model_dir):
    """vg_stream_sync with a 1 ns limit on work still in flight returns VG_ETIMEDOUT and leaves
    the work alone; a host-side fake of a driver that reports a timed-out kernel
    (cudaErrorLaunchTimeout from every event query) makes the bounded waits fail with VG_ECUDA."""
    spec = synth.preset("tiny")
    p = Pair(ctx, spec_path(model_dir, "tiny"), 512)
    L = api.lib()
    toks = synth.token_ids(spec, 250, seed_index=3600)
    timeouts = 0
    for r in range(5):
        for t in toks[50 * r:50 * (r + 1)]:
            p.eng.decode_token_gpu_only(int(t))
        rc = L.vg_stream_sync(p.eng.h, 1)
        assert rc in (0, VG_ETIMEDOUT)
        timeouts += rc == VG_ETIMEDOUT
    assert timeouts > 0, "50 enqueued steps were never still in flight"
    p.eng.sync()
    for t in toks:
        p.ost.decode_token(int(t))
    p.compare("after host timeouts")
    try:
        assert L.vg_test_fake_event_status(702) == 0
        with pytest.raises(api.VoxGenError) as e:
            p.eng.sync()
        assert e.value.code == VG_ECUDA and "timed out" in str(e.value)
    finally:
        L.vg_test_fake_event_status(0)
    p.eng.sync()
    p.compare("after the faked driver timeout")
    p.close()
