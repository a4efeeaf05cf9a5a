"""A small case of the batched step kernel for an ncu capture (not a test): the cfg2 model
(28 layers, H 2048, Q8_0), S streams prefilled to seeded cache lengths in [lo, hi), and 4
batched steps. Capture one launch with `-k regex:decode_batch -s 2 -c 1`.

    python tests/batch_profile_case.py [S=16] [lo=96] [hi=200]
"""
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from voxgen_b200 import api, synth  # noqa: E402


def main():
    S = int(sys.argv[1]) if len(sys.argv) > 1 else 16
    lo = int(sys.argv[2]) if len(sys.argv) > 2 else 96
    hi = int(sys.argv[3]) if len(sys.argv) > 3 else 200
    spec = synth.preset("cfg2")
    path = synth.model_path(spec)
    ctx = api.Context(0)
    model = api.Model(ctx, path)
    assert model.batch_columns >= S, "the batched kernel is not planned for this model"
    lens = np.random.default_rng([4, 1]).integers(lo, hi, size=S)
    engs = [api.BaseLmEngine(model, hi + 64) for _ in range(S)]
    k, v = synth.kv_prefill(spec, int(lens.max()))
    for e, n in zip(engs, lens):
        e.write_kv(k[:, :n], v[:, :n])
    toks = synth.token_ids(spec, 4 * S).reshape(4, S)
    for row in toks:
        api.decode_batch(engs, [int(t) for t in row])
    for e in engs:
        e.sync()
        e.close()
    model.close()
    ctx.close()
    print("ok", S, [int(n) for n in lens])


if __name__ == "__main__":
    main()
