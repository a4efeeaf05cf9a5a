"""ctypes binding of the C oracle (oracle/voxgen_oracle.c).

TEST INFRASTRUCTURE ONLY. The oracle is the CPU restatement of the reference shaders that
the CUDA path is checked against, and the timed CPU baseline. Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU legs import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Optional, Tuple

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "voxgen_oracle.c"
LIB = HERE / "_build" / "libvoxgen_oracle.so"

GEOM = ["ctx_len", "H", "layers", "ffn", "vocab", "heads", "kv_heads", "head_dim", "kv_dim",
        "format", "tied", "orig_ctx"]


def build(force: bool = False) -> Path:
    """Compiles the oracle with gcc (portable -O3, OpenMP, no FMA contraction)."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(f".tmp{os.getpid()}.so")
    cmd = ["gcc", "-O3", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        P, U32, F32, I = C.c_void_p, C.c_uint32, C.c_float, C.c_int
        fp = C.POINTER(C.c_float)
        L.vgo_model_load.argtypes = [C.c_char_p, C.POINTER(P), C.c_char_p, C.c_size_t]
        L.vgo_model_free.argtypes = [P]
        L.vgo_model_geometry.argtypes = [P, C.POINTER(U32)]
        L.vgo_model_scalars.argtypes = [P, fp]
        L.vgo_state_create.argtypes = [P, U32, C.POINTER(P)]
        L.vgo_state_free.argtypes = [P]
        L.vgo_reset.argtypes = [P]
        L.vgo_position.argtypes = [P]
        L.vgo_position.restype = U32
        L.vgo_set_position.argtypes = [P, U32]
        L.vgo_write_kv.argtypes = [P, P, P, U32]
        L.vgo_read_kv.argtypes = [P, P, P, U32]
        L.vgo_decode_token.argtypes = [P, U32, I]
        L.vgo_decode_embedding.argtypes = [P, fp, I]
        L.vgo_output.argtypes = [P]
        L.vgo_output.restype = fp
        L.vgo_logits.argtypes = [P]
        L.vgo_logits.restype = fp
        L.vgo_buffer.argtypes = [P, C.c_char_p]
        L.vgo_buffer.restype = fp
        L.vgo_last_error.argtypes = [P]
        L.vgo_last_error.restype = C.c_char_p
        L.vgo_set_threads.argtypes = [I]
        L.vgo_get_threads.restype = I
        L.vgo_half_to_float.argtypes = [C.c_uint16]
        L.vgo_half_to_float.restype = F32
        L.vgo_float_to_half.argtypes = [F32]
        L.vgo_float_to_half.restype = C.c_uint16
        L.vgo_matvec.argtypes = [I, P, U32, U32, fp, fp, F32]
        L.vgo_embedding.argtypes = [I, P, U32, U32, F32, fp]
        L.vgo_rmsnorm.argtypes = [fp, fp, U32, F32, fp]
        L.vgo_residual_rmsnorm.argtypes = [fp, fp, fp, U32, F32, F32, fp]
        L.vgo_swiglu.argtypes = [I, P, P, U32, U32, fp, fp]
        L.vgo_rope.argtypes = [fp, fp, fp, U32, U32, U32, U32, F32, F32]
        L.vgo_attention.argtypes = [fp, P, P, U32, U32, U32, U32, U32, fp, fp]
        # the RX 7900 XTX mode's variants (the _xtx7900 shaders' summation order)
        L.vgo_set_xtx.argtypes = [P, I]
        L.vgo_matvec_xtx.argtypes = L.vgo_matvec.argtypes
        L.vgo_rmsnorm_xtx.argtypes = L.vgo_rmsnorm.argtypes
        L.vgo_residual_rmsnorm_xtx.argtypes = L.vgo_residual_rmsnorm.argtypes
        L.vgo_swiglu_xtx.argtypes = L.vgo_swiglu.argtypes
        L.vgo_attention_xtx.argtypes = L.vgo_attention.argtypes
        _lib = L
    return _lib


def fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.POINTER(C.c_float))


def vptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


def set_threads(n: int) -> None:
    lib().vgo_set_threads(n)


def threads() -> int:
    return lib().vgo_get_threads()


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"oracle error {code}: {msg}")
        self.code = code


class OracleModel:
    def __init__(self, path):
        L = lib()
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        rc = L.vgo_model_load(str(path).encode(), C.byref(h), err, 512)
        if rc:
            raise OracleError(rc, err.value.decode())
        self.h = h
        g = (C.c_uint32 * 12)()
        L.vgo_model_geometry(h, g)
        self.geom = dict(zip(GEOM, list(g)))
        s = (C.c_float * 6)()
        L.vgo_model_scalars(h, s)
        self.eps, self.theta, self.scaling, self.emb_scale, self.res_scale, self.logit_scale = list(s)

    def __getattr__(self, k):
        g = self.__dict__.get("geom", {})
        if k in g:
            return g[k]
        raise AttributeError(k)

    def close(self):
        if self.h:
            lib().vgo_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OracleState:
    """A decode session on the oracle: BaseLmEngine's buffers and KV cache on the CPU."""

    def __init__(self, model: OracleModel, max_context: int, xtx: bool = False):
        """xtx: follow the RX 7900 XTX mode's shaders (their wave32 summation order)."""
        self.model = model
        h = C.c_void_p()
        rc = lib().vgo_state_create(model.h, max_context, C.byref(h))
        if rc:
            raise OracleError(rc, "state create failed")
        self.h = h
        self.max_context = max_context
        lib().vgo_set_xtx(h, int(xtx))

    def close(self):
        if self.h:
            lib().vgo_state_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc:
            raise OracleError(rc, lib().vgo_last_error(self.h).decode())

    @property
    def position(self) -> int:
        return lib().vgo_position(self.h)

    def reset(self):
        lib().vgo_reset(self.h)

    def set_position(self, p: int):
        self._check(lib().vgo_set_position(self.h, p))

    def write_kv(self, k: np.ndarray, v: np.ndarray):
        n = k.shape[1]
        k = np.ascontiguousarray(k, dtype=np.uint16)
        v = np.ascontiguousarray(v, dtype=np.uint16)
        self._check(lib().vgo_write_kv(self.h, vptr(k), vptr(v), n))

    def read_kv(self, n: int) -> Tuple[np.ndarray, np.ndarray]:
        m = self.model
        k = np.empty((m.layers, n, m.kv_dim), np.uint16)
        v = np.empty_like(k)
        self._check(lib().vgo_read_kv(self.h, vptr(k), vptr(v), n))
        return k, v

    def decode_token(self, token: int, want_logits: bool = False):
        self._check(lib().vgo_decode_token(self.h, int(token), int(want_logits)))

    def decode_embedding(self, h: np.ndarray, want_logits: bool = False):
        h = np.ascontiguousarray(h, dtype=np.float32)
        self._check(lib().vgo_decode_embedding(self.h, fptr(h), int(want_logits)))

    def output(self) -> np.ndarray:
        p = lib().vgo_output(self.h)
        return np.ctypeslib.as_array(p, shape=(self.model.H,)).copy()

    def logits(self) -> np.ndarray:
        p = lib().vgo_logits(self.h)
        return np.ctypeslib.as_array(p, shape=(self.model.vocab,)).copy()

    def buffer(self, name: str) -> np.ndarray:
        m = self.model
        n = {"hidden": m.H, "norm": m.H, "q": m.H, "k": m.kv_dim, "v": m.kv_dim,
             "attention": m.H, "gate": m.ffn, "branch": m.H, "logits": m.vocab,
             "scores": m.heads * self.max_context}[name]
        p = lib().vgo_buffer(self.h, name.encode())
        return np.ctypeslib.as_array(p, shape=(n,)).copy()


# ---- shader-level helpers ----------------------------------------------------

def half_to_float(h: int) -> float:
    return lib().vgo_half_to_float(h)


def float_to_half(f: float) -> int:
    return lib().vgo_float_to_half(f)


def matvec(dtype: int, raw: np.ndarray, rows: int, cols: int, x: np.ndarray, alpha: float = 1.0,
           xtx: bool = False):
    y = np.empty(rows, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    (lib().vgo_matvec_xtx if xtx else lib().vgo_matvec)(dtype, vptr(np.ascontiguousarray(raw)), rows, cols,
                                                        fptr(x), fptr(y), alpha)
    return y


def embedding(dtype: int, raw: np.ndarray, cols: int, token: int, alpha: float = 1.0):
    y = np.empty(cols, np.float32)
    lib().vgo_embedding(dtype, vptr(np.ascontiguousarray(raw)), cols, token, alpha, fptr(y))
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, xtx: bool = False):
    y = np.empty_like(x)
    (lib().vgo_rmsnorm_xtx if xtx else lib().vgo_rmsnorm)(fptr(x), fptr(w), x.size, eps, fptr(y))
    return y


def residual_rmsnorm(hidden: np.ndarray, branch: np.ndarray, w: np.ndarray, eps: float,
                     scale: float, xtx: bool = False):
    h = hidden.copy()
    y = np.empty_like(h)
    (lib().vgo_residual_rmsnorm_xtx if xtx else lib().vgo_residual_rmsnorm)(fptr(h), fptr(branch), fptr(w), h.size,
                                                                          eps, scale, fptr(y))
    return h, y


def swiglu(dtype: int, rg: np.ndarray, ru: np.ndarray, rows: int, cols: int, x: np.ndarray, xtx: bool = False):
    y = np.empty(rows, np.float32)
    (lib().vgo_swiglu_xtx if xtx else lib().vgo_swiglu)(dtype, vptr(rg), vptr(ru), rows, cols, fptr(x), fptr(y))
    return y


def rope(q: np.ndarray, k: np.ndarray, ext: np.ndarray, position: int, heads: int, kv_heads: int,
         head_dim: int, theta: float, scaling: float):
    """rope.comp:22-51 on copies of q and k."""
    q, k = np.array(q, np.float32), np.array(k, np.float32)
    lib().vgo_rope(fptr(q), fptr(k), fptr(np.ascontiguousarray(ext, np.float32)), position, heads,
                   kv_heads, head_dim, theta, scaling)
    return q, k


def attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, heads: int,
              kv_heads: int, head_dim: int, position: int, xtx: bool = False):
    """One layer; caches are [ctx][kv_dim] fp16 bits (reference layout)."""
    ctx = k_cache.shape[0]
    scores = np.zeros(heads * ctx, np.float32)
    out = np.empty(heads * head_dim, np.float32)
    (lib().vgo_attention_xtx if xtx else lib().vgo_attention)(fptr(q), vptr(k_cache), vptr(v_cache), heads, kv_heads,
                                                              head_dim, ctx,
                        position, fptr(scores), fptr(out))
    return out, scores.reshape(heads, ctx)
