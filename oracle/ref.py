"""VoxGen's own BaseLM compute shaders run on the CPU (oracle/_ref/libvoxgen_ref.so, built from the
reference checkout by oracle/ref_shim/build_ref.py), driven the way the reference records them.

TEST INFRASTRUCTURE ONLY: this pins the oracle restatement (oracle/voxgen_oracle.c) against the
reference's own shader code. Only tests/ import it, and only where the library is present (it is
built in the development container, where the reference checkout exists).

`RefEngine` restates BaseLmEngine's buffers (src/baselm.rs:484-549: which buffer each pipeline
binds, in binding order), its push-constant structs (src/baselm.rs:287-380, #[repr(C)], 32-bit
fields) and record_transformer's dispatch sequence and grids (src/baselm.rs:892-1202), with one
dispatch per shader call; the shader code itself is the reference's.
"""
from __future__ import annotations

import ctypes as C
import struct
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libvoxgen_ref.so"

F16, Q8_0 = 1, 8   # dtype_code, src/baselm.rs:1249-1255
# the shaders the XTX mode swaps for their _xtx7900 variants (same bindings and push constants)
_XTX = {"rmsnorm", "residual_rmsnorm", "qkv_matvec", "matvec_swiglu", "matvec", "attn_scores", "softmax"}

_lib: Optional[C.CDLL] = None


def available() -> bool:
    """True when the reference-shader library exists or can be built here."""
    if LIB.exists():
        return True
    try:
        from oracle.ref_shim import build_ref
        return (build_ref.reference_dir() / "shaders").is_dir()
    except Exception:
        return False


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        from oracle.ref_shim import build_ref
        if (build_ref.reference_dir() / "shaders").is_dir():
            build_ref.build()
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} is missing and the reference checkout is not available")
        _lib = C.CDLL(str(LIB))
    return _lib


def dispatch(shader: str, buffers: Sequence[np.ndarray], push: bytes, groups: Sequence[int]) -> None:
    """vkCmdDispatch of one reference shader over host arrays bound in binding order."""
    for b in buffers:
        assert b.flags["C_CONTIGUOUS"] and b.flags["WRITEABLE"], "buffers must be contiguous and writable"
    ptrs = (C.c_void_p * len(buffers))(*[b.ctypes.data for b in buffers])
    gx, gy, gz = (list(groups) + [1, 1])[:3]
    f = getattr(lib(), f"vgref_dispatch_{shader}")
    f.argtypes = [C.c_void_p, C.c_uint32, C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
    f.restype = C.c_int
    rc = f(ptrs, len(buffers), push, len(push), gx, gy, gz)
    if rc:
        raise RuntimeError(f"dispatch {shader}: status {rc}")


def set_threads(n: int) -> None:
    f = lib().vgref_set_threads
    f.argtypes = [C.c_int]
    f(n)


def push(fmt: str, *vals) -> bytes:
    """A #[repr(C)] push-constant struct of 32-bit fields ('I' u32, 'f' f32)."""
    return struct.pack("<" + fmt, *vals)


def effective_scale(v: float) -> float:   # src/baselm.rs:1262-1264
    return 1.0 if v == 0.0 else v


class RefEngine:
    """One BaseLM decode session on the reference shaders (fp32 buffers, fp16 KV words)."""

    def __init__(self, path, max_context: int, xtx: bool = False):
        """xtx: record the RX 7900 XTX mode's shaders (the _xtx7900 variants that
        GpuContext::select_spirv picks, baselm.rs:515-546 and :1241) instead of the normal ones."""
        from oracle import oracle as O
        self.xtx = xtx
        from voxgen_b200 import gguf
        self.summary = gguf.read_gguf(path)
        om = O.OracleModel(path)   # geometry and metadata scalars (BaseLmConfig::from_gguf)
        self.g = dict(om.geom)
        self.eps, self.theta, self.scaling = om.eps, om.theta, om.scaling
        self.emb_scale, self.res_scale, self.logit_scale = om.emb_scale, om.res_scale, om.logit_scale
        om.close()
        raw = np.fromfile(path, dtype=np.uint8, offset=self.summary.data_offset)
        raw = np.concatenate([raw, np.zeros((-raw.size) % 4, np.uint8)])
        self.model = raw.view(np.uint32).copy()            # the whole data region, one buffer
        g = self.g
        H, KV, F = g["H"], g["kv_dim"], g["ffn"]
        self.ctx = max_context
        f32 = lambda n: np.zeros(n, np.float32)
        self.hidden, self.norm, self.q = f32(H), f32(H), f32(H)
        self.k, self.v, self.attention = f32(KV), f32(KV), f32(H)
        self.gate, self.branch, self.logits = f32(F), f32(H), f32(g["vocab"])
        self.scores = f32(g["heads"] * max_context)
        self.kv_k = np.zeros(g["layers"] * max_context * KV // 2, np.uint32)
        self.kv_v = np.zeros_like(self.kv_k)
        self.position = 0

    def shader(self, name: str) -> str:
        return f"{name}_xtx7900" if self.xtx and name in _XTX else name

    def t(self, name: str):
        return self.summary.tensors[name]

    def off(self, name: str) -> int:
        return self.t(name).offset

    def dtype(self, name: str) -> int:
        return {1: F16, 8: Q8_0}[self.t(name).ggml_type]

    # ---- KV cache in the reference layout [layer][ctx][kv_dim] fp16 ----
    def write_kv(self, k: np.ndarray, v: np.ndarray) -> None:
        L, n, KV = k.shape
        kk = self.kv_k.view(np.uint16).reshape(L, self.ctx, KV)
        vv = self.kv_v.view(np.uint16).reshape(L, self.ctx, KV)
        kk[:, :n] = k.view(np.uint16)
        vv[:, :n] = v.view(np.uint16)
        self.position = n

    def read_kv(self, n: int):
        L, KV = self.g["layers"], self.g["kv_dim"]
        kk = self.kv_k.view(np.uint16).reshape(L, self.ctx, KV)[:, :n].copy()
        vv = self.kv_v.view(np.uint16).reshape(L, self.ctx, KV)[:, :n].copy()
        return kk, vv

    # ---- dispatch helpers (src/baselm.rs:1054-1202) ----
    def rms(self, w: str) -> None:
        dispatch(self.shader("rmsnorm"), [self.model, self.hidden, self.norm], push("IIf", self.off(w), self.g["H"], self.eps), [1])

    def residual_rms(self, w: str) -> None:
        dispatch(self.shader("residual_rmsnorm"), [self.model, self.hidden, self.branch, self.norm],
                 push("IIff", self.off(w), self.g["H"], self.eps, effective_scale(self.res_scale)), [1])

    def matvec(self, w: str, x: np.ndarray, y: np.ndarray, rows: int, cols: int, alpha: float) -> None:
        assert self.t(w).dims == (cols, rows)
        dispatch(self.shader("matvec"), [self.model, x, y], push("IIIIIf", self.off(w), rows, cols, self.dtype(w), 0, alpha), [rows])

    def record_transformer(self, position: int, logits: bool) -> None:
        g = self.g
        H, KV, F = g["H"], g["kv_dim"], g["ffn"]
        heads, kvh, D = g["heads"], g["kv_heads"], g["head_dim"]
        rope_w = "rope_factors_long.weight" if g["ctx_len"] > g["orig_ctx"] else "rope_factors_short.weight"
        self.rms("blk.0.attn_norm.weight")
        for l in range(g["layers"]):
            n = lambda s: f"blk.{l}.{s}"
            qw, kw, vw = n("attn_q.weight"), n("attn_k.weight"), n("attn_v.weight")
            dispatch(self.shader("qkv_matvec"), [self.model, self.norm, self.q, self.k, self.v],
                     push("IIIIIIIIII", self.off(qw), self.off(kw), self.off(vw), H, KV, H,
                          self.dtype(qw), self.dtype(kw), self.dtype(vw), 0), [H + 2 * KV])
            dispatch("rope", [self.model, self.q, self.k],
                     push("IIIIIff", self.off(rope_w), position, heads, kvh, D, self.theta, self.scaling),
                     [heads + kvh])
            dispatch("store_kv", [self.k, self.v, self.kv_k, self.kv_v], push("IIII", l, position, self.ctx, KV), [1])
            attn = push("IIIIII", l, self.ctx, position, D, heads // kvh, kvh)
            dispatch(self.shader("attn_scores"), [self.q, self.kv_k, self.scores], attn, [position + 1, heads])
            dispatch(self.shader("softmax"), [self.scores], push("II", self.ctx, position), [heads])
            dispatch("attn_values", [self.scores, self.kv_v, self.attention], attn, [heads])
            self.matvec(n("attn_output.weight"), self.attention, self.branch, H, H, 1.0)
            self.residual_rms(n("ffn_norm.weight"))
            gw, uw = n("ffn_gate.weight"), n("ffn_up.weight")
            dispatch(self.shader("matvec_swiglu"), [self.model, self.norm, self.gate],
                     push("IIIIII", self.off(gw), self.off(uw), F, H, self.dtype(gw), 0), [F])
            self.matvec(n("ffn_down.weight"), self.gate, self.branch, H, F, 1.0)
            nxt = f"blk.{l + 1}.attn_norm.weight" if l + 1 < g["layers"] else "output_norm.weight"
            self.residual_rms(nxt)
        if logits:
            out = "token_embd.weight" if g["tied"] else "output.weight"
            self.matvec(out, self.norm, self.logits, g["vocab"], H, effective_scale(self.logit_scale))

    # ---- entry points (src/baselm.rs:622-681) ----
    def decode_token(self, token: int, want_logits: bool = False) -> None:
        w = "token_embd.weight"
        dispatch("embedding", [self.model, self.hidden],
                 push("IIIIf", self.off(w), self.g["H"], token, self.dtype(w), effective_scale(self.emb_scale)), [1])
        self.record_transformer(self.position, want_logits)
        self.position += 1

    def decode_embedding(self, h: np.ndarray, want_logits: bool = False) -> None:
        self.hidden[:] = h
        self.record_transformer(self.position, want_logits)
        self.position += 1

    def output(self) -> np.ndarray:
        return self.norm.copy()
