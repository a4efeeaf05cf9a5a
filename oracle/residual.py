"""CPU restatement of one ResidualLM position: FSQ, the fusion projection and the ResidualLM
layers (VoxGen src/acoustic.rs:851-1035).

TEST INFRASTRUCTURE ONLY: the checker of the CUDA ResidualLM path. It composes the C oracle's
shader restatements (oracle/voxgen_oracle.c: the lane-strided matvec, RMSNorm, attention,
SwiGLU, which are pinned against the reference shaders) with the three ResidualLM adds:

* ``linear_bias``  -- linear_bias.comp:58-78, (lane-strided W x + bias) * alpha;
* ``fsq_quantize`` -- fsq_quantize.comp:8-11, round(tanh(x) * scale) / scale with C's tanhf
  and roundf (GLSL leaves halves to the implementation; roundf takes them away from zero);
* ``fusion``       -- fusion_linear.comp:49-72, W [left | right] + bias.

The record order is ResidualFsqEngine's: record_fsq (:921-944), record_current_lm_copy
(:903-919), record_fusion (:946-966), record_residual_lm (:968-1035, no RoPE).
"""
from __future__ import annotations

import ctypes as C
import ctypes.util
from pathlib import Path
from typing import Optional

import numpy as np

from . import oracle as O
from voxgen_b200.gguf import GGML_F16, GGML_F32, read_gguf

_libm = C.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.tanhf.argtypes = [C.c_float]
_libm.tanhf.restype = C.c_float
_libm.roundf.argtypes = [C.c_float]
_libm.roundf.restype = C.c_float


def _vector(g, name: str) -> np.ndarray:
    t = g.tensors[name]
    raw = g.tensor_bytes(name)
    if t.ggml_type == GGML_F32:
        return raw.view(np.float32).copy()
    return raw.view(np.float16).astype(np.float32)


def linear_bias(dtype: int, raw: np.ndarray, rows: int, cols: int, x: np.ndarray, bias: np.ndarray,
                alpha: float = 1.0) -> np.ndarray:
    """linear_bias.comp:58-78: (partial[0] + bias) * alpha per row."""
    y = O.matvec(dtype, raw, rows, cols, x, 1.0)
    return ((y + bias.astype(np.float32)) * np.float32(alpha)).astype(np.float32)


def fsq_quantize(x: np.ndarray, scale: float) -> np.ndarray:
    """fsq_quantize.comp:8-11 in fp32."""
    s = np.float32(scale)
    out = np.empty(x.size, np.float32)
    for i, v in enumerate(np.asarray(x, np.float32)):
        t = np.float32(_libm.tanhf(float(v)))
        out[i] = np.float32(_libm.roundf(float(np.float32(t * s)))) / s
    return out


def fusion(dtype: int, raw: np.ndarray, rows: int, left: np.ndarray, right: np.ndarray,
           bias: np.ndarray) -> np.ndarray:
    """fusion_linear.comp:49-72: the lane-strided sum over [left | right], then + bias."""
    x = np.concatenate([np.asarray(left, np.float32), np.asarray(right, np.float32)])
    return linear_bias(dtype, raw, rows, x.size, x, bias)


class ResidualOracle:
    """A ResidualLM session on the CPU: its KV cache and the buffers ResidualFsqEngine keeps
    (fsq_output, fusion_snapshot, current_lm, norm)."""

    def __init__(self, acoustic_path, base_path, max_context: int):
        self.g = read_gguf(acoustic_path)
        base = O.OracleModel(base_path)
        md = self.g.metadata
        self.layers = int(md["voxcpm.residual_lm.n_layer"])
        self.H = int(md["voxcpm.residual_lm.n_embd"])
        self.latent = int(md["voxcpm.fsq.latent_dim"])
        self.scale = float(md["voxcpm.fsq.scale"])
        self.heads, self.kv_heads, self.head_dim = base.heads, base.kv_heads, base.head_dim
        self.kv_dim, self.F = base.kv_dim, base.ffn
        self.eps = base.eps
        self.rs = base.res_scale if base.res_scale != 0.0 else 1.0  # effective_scale
        base.close()
        self.ctx = max_context
        self.kv_k = np.zeros((self.layers, max_context, self.kv_dim), np.uint16)
        self.kv_v = np.zeros_like(self.kv_k)
        self.position = 0
        self.fsq_output = np.zeros(self.H, np.float32)
        self.fused = np.zeros(self.H, np.float32)
        self.current_lm = np.zeros(self.H, np.float32)
        self.norm = np.zeros(self.H, np.float32)
        self.fsq_margin = float("inf")
        self._w = {}

    def _mat(self, name: str):
        if name not in self._w:
            t = self.g.tensors[name]
            self._w[name] = (t.ggml_type, self.g.tensor_bytes(name))
        return self._w[name]

    def _vec(self, name: str) -> np.ndarray:
        if name not in self._w:
            self._w[name] = _vector(self.g, name)
        return self._w[name]

    def reset(self) -> None:
        self.position = 0

    def step(self, base_hidden: np.ndarray, embed: Optional[np.ndarray] = None,
             fsq_applied: bool = True) -> None:
        H, L = self.H, self.latent
        base_hidden = np.asarray(base_hidden, np.float32)
        if fsq_applied:  # record_fsq
            dt, w = self._mat("fsq.in_proj.weight")
            lat = linear_bias(dt, w, L, H, base_hidden, self._vec("fsq.in_proj.bias"))
            # distance of tanh(latent) * scale from the nearest rounding boundary (a half):
            # another summation order can only change the rounded value below this margin
            t = np.tanh(lat.astype(np.float64)) * self.scale
            self.fsq_margin = float(np.min(np.abs(np.abs(t - np.trunc(t)) - 0.5)))
            lat = fsq_quantize(lat, self.scale)
            dt, w = self._mat("fsq.out_proj.weight")
            self.fsq_output = linear_bias(dt, w, H, L, lat, self._vec("fsq.out_proj.bias"))
            left = self.fsq_output
        else:  # a text-prefix position: the raw BaseLM hidden
            left = base_hidden
        self.current_lm = left.copy()
        right = np.zeros(H, np.float32) if embed is None else np.asarray(embed, np.float32)
        dt, w = self._mat("projections.res_fusion_proj.weight")
        hidden = fusion(dt, w, H, left, right, self._vec("projections.res_fusion_proj.bias"))
        self.fused = hidden.copy()
        self._residual_lm(hidden)
        self.position += 1

    def _residual_lm(self, hidden: np.ndarray) -> None:
        """record_residual_lm (src/acoustic.rs:968-1035): BaseLM's layer sequence without RoPE."""
        pos, H = self.position, self.H
        if pos >= self.ctx:
            raise ValueError("ResidualLM KV cache is full")
        p = lambda l, s: f"residual_lm.blk.{l}.{s}"
        norm = O.rmsnorm(hidden, self._vec(p(0, "attn_norm.weight")), self.eps)
        qr = self.heads * self.head_dim
        for l in range(self.layers):
            q = O.matvec(*self._mat(p(l, "attn_q.weight")), qr, H, norm)
            k = O.matvec(*self._mat(p(l, "attn_k.weight")), self.kv_dim, H, norm)
            v = O.matvec(*self._mat(p(l, "attn_v.weight")), self.kv_dim, H, norm)
            self.kv_k[l, pos] = k.astype(np.float16).view(np.uint16)  # store_kv.comp, RNE
            self.kv_v[l, pos] = v.astype(np.float16).view(np.uint16)
            attn, _ = O.attention(q, self.kv_k[l], self.kv_v[l], self.heads, self.kv_heads,
                                  self.head_dim, pos)
            branch = O.matvec(*self._mat(p(l, "attn_output.weight")), H, qr, attn)
            hidden, norm = O.residual_rmsnorm(hidden, branch, self._vec(p(l, "ffn_norm.weight")),
                                              self.eps, self.rs)
            dg, wg = self._mat(p(l, "ffn_gate.weight"))
            _, wu = self._mat(p(l, "ffn_up.weight"))
            gate = O.swiglu(dg, wg, wu, self.F, H, norm)
            branch = O.matvec(*self._mat(p(l, "ffn_down.weight")), H, self.F, gate)
            nxt = p(l + 1, "attn_norm.weight") if l + 1 < self.layers else "residual_lm.output_norm.weight"
            hidden, norm = O.residual_rmsnorm(hidden, branch, self._vec(nxt), self.eps, self.rs)
        self.norm = norm

    def output(self) -> np.ndarray:
        return self.norm.copy()
