"""Generates ref_shader_pin.npz: hidden states and logits computed by the reference's own BaseLM
shaders (compiled as C++ by oracle/ref_shim, run on the CPU) on the seeded synthetic models
"pin" (Q8_0), "pin_f16" (F16, untied output, non-unit scales) and "g6" (Q8_0, groups of 6 query
heads per KV head).

Run where the reference checkout is available:  python tests/golden/make_ref_pin.py [--xtx]
With --xtx the same session runs the RX 7900 XTX mode's shader variants (the _xtx7900 files,
subgroup sums emulated as a pairwise tree over 32 invocations) into ref_shader_pin_xtx.npz.
The session is run_session below: 20 prefilled KV positions, two steps from external embeddings,
then two token steps with logits. The file also records each model file's SHA-256, so a change
of the synthetic-model generator is caught instead of silently comparing different weights.
"""
import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from voxgen_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "ref_shader_pin.npz"
OUT_XTX = Path(__file__).resolve().parent / "ref_shader_pin_xtx.npz"
CONTEXT = 48
MODELS = ("pin", "pin_f16", "g6")


def run_session(spec, eng):
    """[(hidden, logits or None)] per step on an engine with the BaseLmEngine-style calls."""
    k, v = synth.kv_prefill(spec, 20)
    eng.write_kv(k, v)
    outs = []
    for h in synth.hidden_inputs(spec, 2):
        eng.decode_embedding(h)
        outs.append((eng.output(), None))
    for t in synth.token_ids(spec, 2):
        eng.decode_token(int(t), want_logits=True)
        lg = eng.logits() if callable(eng.logits) else eng.logits.copy()
        outs.append((eng.output(), lg))
    return outs


def main(xtx: bool = False):
    from oracle import ref as R
    arrays = {}
    with tempfile.TemporaryDirectory() as d:
        for name in MODELS:
            spec = synth.preset(name)
            path = synth.model_path(spec, Path(d))
            outs = run_session(spec, R.RefEngine(path, CONTEXT, xtx=xtx))
            arrays[f"{name}_hidden"] = np.stack([h for h, _ in outs])
            arrays[f"{name}_logits"] = np.stack([lg for _, lg in outs if lg is not None])
            arrays[f"{name}_sha256"] = np.array(hashlib.sha256(path.read_bytes()).hexdigest())
    out = OUT_XTX if xtx else OUT
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}")


if __name__ == "__main__":
    main("--xtx" in sys.argv[1:])
