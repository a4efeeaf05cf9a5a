"""The batched step kernel (one weight pass for up to 16 columns) against the oracle: 16
independent streams at ragged positions (BASELINE config[4]'s shape: config[2] / [3] layers,
contexts in [64, 4096]), smaller models with 3, 9 and 16 streams, and the streams' later
single-stream steps on the caches the batched steps wrote. Batched prefill is covered in
test_gpu_entrypoints.py (test_prefill_tokens)."""
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


class Streams:
    """n streams of one model on the CUDA engine and the same n sessions on the oracle."""

    def __init__(self, ctx, spec, path, lens, max_context, kv_seed=1100):
        self.spec = spec
        self.model = api.Model(ctx, path)
        self.om = O.OracleModel(path)
        self.eng = [api.BaseLmEngine(self.model, max_context) for _ in lens]
        self.ost = [O.OracleState(self.om, max_context) for _ in lens]
        k, v = synth.kv_prefill(spec, int(max(lens)), seed_index=kv_seed)
        for i, n in enumerate(lens):
            if n:
                ki, vi = np.roll(k, i, axis=1)[:, :n], np.roll(v, i, axis=1)[:, :n]  # distinct caches
                self.eng[i].write_kv(ki, vi)
                self.ost[i].write_kv(ki, vi)

    def batch_step(self, tokens):
        api.decode_batch(self.eng, [int(t) for t in tokens])
        for st, t in zip(self.ost, tokens):
            st.decode_token(int(t))

    def compare(self, what):
        for i, (e, o) in enumerate(zip(self.eng, self.ost)):
            assert e.position == o.position, (what, i)
            assert_close(e.output(), o.output(), what=f"{what} stream {i} at position {e.position - 1}")

    def close(self):
        for e in self.eng:
            e.close()
        self.model.close()


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_batch_16_ragged_streams(ctx, model_dir, name):
    """config[4]: 16 streams with ragged cache lengths in [64, 4096], two batched steps, each
    stream's hidden state against the oracle; then the KV rows the batched steps wrote and a
    single-stream step of every stream on them."""
    spec = synth.preset(name)
    lens = np.random.default_rng([4, 7]).integers(64, 4095, size=16)
    lens[0], lens[1] = 64, 4094            # the ends of the range
    s = Streams(ctx, spec, spec_path(model_dir, name), lens, 4096)
    assert s.model.batch_columns == 16
    toks = synth.token_ids(spec, 32, seed_index=4100).reshape(2, 16)
    for r, row in enumerate(toks):
        s.batch_step(row)
        s.compare(f"{name} batched step {r}")
    for i in (0, 5, 15):
        ke, ve = s.eng[i].read_kv(int(lens[i]) + 2)
        ko, vo = s.ost[i].read_kv(int(lens[i]) + 2)
        for a, b, nm in ((ke, ko, "K"), (ve, vo, "V")):
            assert_close(a[:, -2:].view(np.float16).astype(np.float32), b[:, -2:].view(np.float16).astype(np.float32),
                         what=f"{name} stream {i} {nm} rows written by the batched steps")
    for e, o, t in zip(s.eng, s.ost, synth.token_ids(spec, 16, seed_index=4200)):
        if e.position < e.max_context:
            e.decode_token_gpu_only(int(t))
            o.decode_token(int(t))
    s.compare(f"{name} single-stream step after the batched steps")
    s.close()


@pytest.mark.parametrize("name,n", [("tiny", 3), ("tiny", 9), ("tiny_f16", 16), ("pin", 5), ("pin_f16", 16), ("cfg1", 16),
                                    ("g6", 16), ("g6", 4)])
def test_batch_small_models(ctx, model_dir, name, n):
    """Fewer columns than 16 (one or two n8 tiles), streams at position 0 and at chunk boundaries,
    ragged matrix widths (F = 608: the last column group reaches into the padding), GQA 2, 4
    and 6, head_dim 32 / 64 / 128, F16 and Q8_0, merge slices 16 and 32 dimensions wide, several
    batched steps."""
    spec = synth.preset(name)
    lens = [0, 63, 64, 65, 127, 128, 129, 200, 1, 300, 17, 33, 250, 301, 99, 5][:n]
    s = Streams(ctx, spec, spec_path(model_dir, name), lens, 320)
    toks = synth.token_ids(spec, 4 * n, seed_index=4300).reshape(4, n)
    for r, row in enumerate(toks):
        s.batch_step(row)
        s.compare(f"{name} x{n} batched step {r}")
    s.close()


def test_batch_long_contexts(ctx, model_dir):
    """Streams past 4096 positions: more than 128 attention chunks per (stream, KV head), so the
    merge's (max, sum) pass reads chunks beyond the ones each thread keeps in registers."""
    spec = synth.preset("pin")
    lens = [4190, 10, 4300]
    s = Streams(ctx, spec, spec_path(model_dir, "pin"), lens, 4400)
    toks = synth.token_ids(spec, 6, seed_index=4400).reshape(2, 3)
    for r, row in enumerate(toks):
        s.batch_step(row)
        s.compare(f"pin long contexts batched step {r}")
    s.close()


def test_batch_then_reset_and_errors(ctx, model_dir):
    """Streams keep working on their own after batched steps (reset, single steps); a batch
    with a full stream is refused before any stream advances."""
    spec = synth.preset("tiny")
    s = Streams(ctx, spec, spec_path(model_dir, "tiny"), [10, 20, 30], 40)
    s.batch_step([1, 2, 3])
    s.compare("batched")
    for e, o in zip(s.eng, s.ost):
        e.reset()
        o.reset()
        e.decode_token_gpu_only(7)
        o.decode_token(7)
    s.compare("after reset")
    s.eng[2].seek(40)
    with pytest.raises(api.VoxGenError) as err:
        api.decode_batch(s.eng, [1, 2, 3])
    assert err.value.code == -6
    assert [e.position for e in s.eng] == [1, 1, 40]
    s.close()


def test_copy_outputs_reads_every_stream(ctx, model_dir):
    """vg_copy_outputs after batched steps: the n hidden states with one wait, equal bit for bit
    to each stream's own vg_copy_output, and within tolerance of the oracle."""
    spec = synth.preset("tiny")
    s = Streams(ctx, spec, spec_path(model_dir, "tiny"), [3, 0, 17, 40, 9], 64)
    for r, row in enumerate(synth.token_ids(spec, 10, seed_index=4400).reshape(2, 5)):
        s.batch_step(row)
        got = api.outputs(s.eng)
        assert got.shape == (5, spec.hidden)
        for i, (e, o) in enumerate(zip(s.eng, s.ost)):
            assert np.array_equal(got[i].view(np.uint32), e.output().view(np.uint32)), f"stream {i}"
            assert_close(got[i], o.output(), what=f"batched read of stream {i} after step {r}")
    s.close()
