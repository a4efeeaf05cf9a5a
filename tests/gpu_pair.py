"""A decode session on the CUDA engine (through the C ABI) and the same session on the oracle,
stepped together and compared at the parity tolerance. Shared by the ``-m gpu`` step tests."""
import numpy as np

from conftest import assert_close
from oracle import oracle as O
from voxgen_b200 import api


def _ordinal(bits):
    """fp16 bit patterns mapped to integers that are monotonic in the value."""
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


class Pair:
    """The same session on the CUDA engine and on the oracle."""

    def __init__(self, ctx, path, max_context, xtx=False):
        """xtx: the oracle follows the reference's RX 7900 XTX mode (its _xtx7900 shaders'
        summation order) instead of the normal shaders."""
        self.model = api.Model(ctx, path)
        self.eng = api.BaseLmEngine(self.model, max_context)
        self.om = O.OracleModel(path)
        self.ost = O.OracleState(self.om, max_context, xtx=xtx)

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
