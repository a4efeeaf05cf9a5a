"""Python binding of the C ABI (include/voxgen_cuda.h), shaped like the reference engine.

``BaseLmEngine`` mirrors the Rust ``BaseLmEngine`` of src/baselm.rs:429-1232 — same method
names, argument meaning and error behaviour (errors raise :class:`VoxGenError` carrying the
library's status code and message, where the reference returns ``anyhow`` errors). All GPU
work runs in ``libvoxgen_b200.so``; this module only marshals arguments. There is no CPU
fallback: if the library cannot be loaded, construction fails.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path
from typing import List, Optional, Sequence

import numpy as np

from . import _build

VG_OK = 0
STATUS = {
    -1: "VG_EINVAL", -2: "VG_EIO", -3: "VG_EFORMAT", -4: "VG_EUNSUPPORTED", -5: "VG_ERANGE",
    -6: "VG_EFULL", -7: "VG_ECUDA", -8: "VG_ENOMEM", -9: "VG_ETIMEDOUT", -10: "VG_EDEVICE",
    -11: "VG_ESTATE",
}
FORMAT_AUTO, FORMAT_F16, FORMAT_Q8_0 = 0, 1, 8
FORMATS = {"auto": FORMAT_AUTO, "f16": FORMAT_F16, "q8_0": FORMAT_Q8_0}

# Names of every function the header declares (checked by the CPU test suite).
EXPORTS = [
    "vg_ctx_create", "vg_ctx_destroy", "vg_last_error", "vg_ctx_sm_count", "vg_gguf_inspect",
    "vg_kv_cache_bytes", "vg_top_k_logits",
    "vg_model_load_gguf", "vg_model_info_get", "vg_model_destroy", "vg_stream_create",
    "vg_stream_destroy", "vg_stream_reset", "vg_stream_position", "vg_stream_cuda_stream", "vg_stream_kernel_mode",
    "vg_stream_write_kv", "vg_stream_read_kv", "vg_decode_token", "vg_decode_embedding",
    "vg_decode_embedding_device", "vg_prefill_tokens", "vg_stream_output", "vg_stream_logits",
    "vg_copy_output", "vg_copy_outputs", "vg_copy_logits", "vg_stream_sync", "vg_step_result_get", "vg_benchmark",
    "vg_stream_profile_step", "vg_decode_batch", "vg_k_packed_bytes", "vg_k_repack", "vg_k_matvec", "vg_k_embedding",
    "vg_k_residual_rmsnorm", "vg_k_attention", "vg_k_attention_noalloc",
    "vg_residual_load_gguf", "vg_residual_step", "vg_residual_step_host", "vg_residual_state",
    "vg_residual_copy_state", "vg_stream_seek", "vg_stream_set_wait_limit", "vg_test_stalled_step",
    "vg_test_fake_event_status", "vg_model_batch_columns",
]

# which buffer vg_residual_state / vg_residual_copy_state return
RESIDUAL_STATE = {"fsq_output": 0, "fused_input": 1, "lm_state": 2}


class VoxGenError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code
        self.status = STATUS.get(code, str(code))


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "context_length", "embedding_length", "block_count", "feed_forward_length", "vocab_size",
        "head_count", "head_count_kv", "head_dim", "kv_dim", "rope_original_context_length")] + \
        [(n, C.c_float) for n in ("rms_epsilon", "rope_theta", "rope_scaling_factor", "embedding_scale",
                                  "residual_scale", "logit_scale")] + \
        [(n, C.c_int32) for n in ("format", "tied_output", "rope_long_factors", "reserved0")] + \
        [(n, C.c_uint64) for n in ("gguf_data_bytes", "layer_weight_bytes", "norm_weight_bytes",
                                   "device_weight_bytes")]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_ if k != "reserved0"}


@dataclass
class TopLogitPy:
    token_id: int
    logit: float


class TopLogit(C.Structure):
    _fields_ = [("token_id", C.c_uint32), ("logit", C.c_float)]


class KernelTime(C.Structure):
    _fields_ = [("name", C.c_char * 24), ("layer", C.c_uint32), ("ms", C.c_float), ("bytes", C.c_uint64)]


class StepResult(C.Structure):
    _fields_ = [("position", C.c_uint32), ("n_top", C.c_uint32),
                ("final_hidden_checksum", C.c_double), ("final_hidden_l2", C.c_double)]


class BenchmarkResult(C.Structure):
    _fields_ = [("iterations", C.c_uint32), ("token_id", C.c_uint32), ("mean_ms", C.c_double),
                ("min_ms", C.c_double), ("max_ms", C.c_double), ("tokens_per_second", C.c_double)]


_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """Loads (building first if needed) the native library and declares signatures."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.build() if _build.needs_build() else _build.LIB
    L = C.CDLL(str(path))
    P, U32, I, F, SZ, U64 = C.c_void_p, C.c_uint32, C.c_int, C.c_float, C.c_size_t, C.c_uint64
    PP = C.POINTER(C.c_void_p)
    sig = {
        "vg_ctx_create": ([I, PP], I), "vg_ctx_destroy": ([P], I), "vg_last_error": ([P], C.c_char_p),
        "vg_ctx_sm_count": ([P, C.POINTER(I)], I),
        "vg_gguf_inspect": ([C.c_char_p, I, C.POINTER(ModelInfo), C.c_char_p, SZ], I),
        "vg_kv_cache_bytes": ([C.POINTER(ModelInfo), U32, C.POINTER(U64)], I),
        "vg_top_k_logits": ([P, U32, U32, C.POINTER(TopLogit), C.POINTER(U32)], I),
        "vg_model_load_gguf": ([P, C.c_char_p, I, PP], I),
        "vg_model_info_get": ([P, C.POINTER(ModelInfo)], I), "vg_model_destroy": ([P], I),
        "vg_stream_create": ([P, U32, PP], I), "vg_stream_destroy": ([P], I),
        "vg_stream_reset": ([P], I), "vg_stream_position": ([P, C.POINTER(U32)], I),
        "vg_stream_cuda_stream": ([P, PP], I),
        "vg_stream_kernel_mode": ([P, C.POINTER(I)], I),
        "vg_stream_write_kv": ([P, P, P, U32], I), "vg_stream_read_kv": ([P, P, P, U32], I),
        "vg_decode_token": ([P, U32, I], I), "vg_decode_embedding": ([P, P, I], I),
        "vg_decode_embedding_device": ([P, P, I], I), "vg_prefill_tokens": ([P, P, U32, I], I),
        "vg_stream_output": ([P, PP], I), "vg_stream_logits": ([P, PP], I),
        "vg_copy_output": ([P, P, SZ], I), "vg_copy_logits": ([P, P, SZ], I),
        "vg_copy_outputs": ([P, I, P, SZ], I),
        "vg_stream_sync": ([P, U64], I),
        "vg_step_result_get": ([P, U32, C.POINTER(StepResult), C.POINTER(TopLogit)], I),
        "vg_benchmark": ([P, U32, U32, U32, I, C.POINTER(BenchmarkResult)], I),
        "vg_stream_profile_step": ([P, U32, I, C.POINTER(KernelTime), U32, C.POINTER(U32)], I),
        "vg_decode_batch": ([P, I, P], I),
        "vg_k_packed_bytes": ([I, U32, U32, C.POINTER(U64)], I),
        "vg_k_repack": ([I, P, U32, U32, P, P], I),
        "vg_k_matvec": ([I, P, U32, U32, P, P, F, P], I),
        "vg_k_embedding": ([I, P, U32, U32, U32, F, P, P], I),
        "vg_k_residual_rmsnorm": ([P, P, P, U32, F, F, P, P], I),
        "vg_k_attention": ([P, P, P, U32, U32, U32, U32, U32, P, P], I),
        "vg_k_attention_noalloc": ([P, P, P, U32, U32, U32, U32, U32, P, P], I),
        "vg_residual_load_gguf": ([P, C.c_char_p, P, PP], I),
        "vg_residual_step": ([P, P, P, I], I),
        "vg_residual_step_host": ([P, P, P, I], I),
        "vg_residual_state": ([P, I, PP], I),
        "vg_residual_copy_state": ([P, I, P, SZ], I),
        "vg_stream_seek": ([P, U32], I),
        "vg_stream_set_wait_limit": ([P, U64], I),
        "vg_test_stalled_step": ([P, U32], I),
        "vg_test_fake_event_status": ([I], I),
        "vg_model_batch_columns": ([P, C.POINTER(U32)], I),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def _ptr(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


def inspect_gguf(path, fmt: str = "auto") -> dict:
    """Host-only validation of a BaseLM GGUF (no GPU): returns the model info."""
    info = ModelInfo()
    err = C.create_string_buffer(1024)
    rc = lib().vg_gguf_inspect(str(path).encode(), FORMATS[fmt], C.byref(info), err, 1024)
    if rc:
        raise VoxGenError(rc, err.value.decode())
    return info.as_dict()


def kv_cache_bytes(info: dict, max_context: int) -> int:
    """BaseLmConfig::kv_cache_bytes (src/baselm.rs:182-192) through the C ABI."""
    mi = ModelInfo(**{k: v for k, v in info.items() if k in dict(ModelInfo._fields_)})
    out = C.c_uint64()
    rc = lib().vg_kv_cache_bytes(C.byref(mi), max_context, C.byref(out))
    if rc:
        raise VoxGenError(rc, "vg_kv_cache_bytes failed")
    return out.value


def top_k_logits(logits: np.ndarray, k: int) -> List[TopLogitPy]:
    """top_k_logits (src/baselm.rs:1295-1309) through the C ABI."""
    x = np.ascontiguousarray(logits, np.float32)
    out = (TopLogit * max(k, 1))()
    n = C.c_uint32()
    rc = lib().vg_top_k_logits(_ptr(x), x.size, k, out, C.byref(n))
    if rc:
        raise VoxGenError(rc, "vg_top_k_logits failed")
    return [TopLogitPy(out[i].token_id, out[i].logit) for i in range(n.value)]


class Context:
    """One CUDA device (replaces VulkanContext, src/vulkan.rs:96-113)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        rc = lib().vg_ctx_create(device, C.byref(h))
        if rc:
            raise VoxGenError(rc, f"vg_ctx_create({device}) failed")
        self.h = h
        self.device = device

    def check(self, rc: int) -> None:
        if rc:
            raise VoxGenError(rc, lib().vg_last_error(self.h).decode())

    @property
    def sm_count(self) -> int:
        n = C.c_int()
        self.check(lib().vg_ctx_sm_count(self.h, C.byref(n)))
        return n.value

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().vg_ctx_destroy(self.h)
            self.h = None


class Model:
    """Weights of one BaseLM GGUF repacked into HBM (shared by any number of streams)."""

    def __init__(self, ctx: Context, path, fmt: str = "auto"):
        self.ctx = ctx
        h = C.c_void_p()
        ctx.check(lib().vg_model_load_gguf(ctx.h, str(path).encode(), FORMATS[fmt], C.byref(h)))
        self.h = h
        info = ModelInfo()
        ctx.check(lib().vg_model_info_get(h, C.byref(info)))
        self.info = info.as_dict()
        self.path = Path(path)

    @property
    def batch_columns(self) -> int:
        """Columns of the batched step kernel for this model (16), or 0 when it is unavailable."""
        n = C.c_uint32()
        self.ctx.check(lib().vg_model_batch_columns(self.h, C.byref(n)))
        return n.value

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().vg_model_destroy(self.h)
            self.h = None


class ResidualModel(Model):
    """The ResidualLM + FSQ + fusion weights of an acoustic GGUF, following a BaseLM ``base``
    (ResidualFsqEngine::new, src/acoustic.rs:435-560)."""

    def __init__(self, ctx: Context, acoustic_path, base: Model):
        self.ctx = ctx
        h = C.c_void_p()
        ctx.check(lib().vg_residual_load_gguf(ctx.h, str(acoustic_path).encode(), base.h, C.byref(h)))
        self.h = h
        info = ModelInfo()
        ctx.check(lib().vg_model_info_get(h, C.byref(info)))
        self.info = info.as_dict()
        self.path = Path(acoustic_path)
        self.base = base


@dataclass
class BaseLmStepResult:
    """src/baselm.rs:404-411."""
    position: int
    elapsed_ms: float
    final_hidden_checksum: float
    final_hidden_l2: float
    top_logits: List[TopLogitPy]


class BaseLmEngine:
    """A decode session: KV cache, activations and the captured step graphs.

    Method names follow src/baselm.rs: ``decode_token`` (:622), ``decode_embedding`` (:657),
    ``decode_token_gpu_only`` (:689), ``decode_embedding_gpu_only`` (:766),
    ``decode_embedding_from_gpu_only`` (:793), ``prefill_tokens`` (:823), ``benchmark`` (:841),
    ``reset`` (:616), ``position`` (:604), ``output_buffer`` (:610).
    """

    def __init__(self, model: Model, max_context: int):
        self.model = model
        self.ctx = model.ctx
        h = C.c_void_p()
        self.ctx.check(lib().vg_stream_create(model.h, max_context, C.byref(h)))
        self.h = h
        self.max_context = max_context
        self.H = model.info["embedding_length"]
        self.vocab = model.info["vocab_size"]

    # -- lifecycle -------------------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "h", None):
            lib().vg_stream_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc: int) -> None:
        self.ctx.check(rc)

    @property
    def position(self) -> int:
        p = C.c_uint32()
        self._check(lib().vg_stream_position(self.h, C.byref(p)))
        return p.value

    def reset(self) -> None:
        self._check(lib().vg_stream_reset(self.h))

    def seek(self, position: int) -> None:
        """Moves the decode position without touching the KV cache (vg_stream_seek)."""
        self._check(lib().vg_stream_seek(self.h, int(position)))

    def set_wait_limit(self, seconds: float) -> None:
        """Limit of every bounded device-side wait of this stream (0: the 2 s default)."""
        self._check(lib().vg_stream_set_wait_limit(self.h, int(round(seconds * 1e9))))

    @property
    def kernel_mode(self) -> int:
        """1: one persistent kernel per step; 0: one kernel per projection/attention/norm."""
        m = C.c_int()
        self._check(lib().vg_stream_kernel_mode(self.h, C.byref(m)))
        return m.value

    @property
    def cuda_stream(self) -> int:
        p = C.c_void_p()
        self._check(lib().vg_stream_cuda_stream(self.h, C.byref(p)))
        return p.value or 0

    def write_kv(self, k: np.ndarray, v: np.ndarray) -> None:
        """fp16 bits ``[layer][n][kv_dim]``; sets the position to n."""
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        self._check(lib().vg_stream_write_kv(self.h, _ptr(k), _ptr(v), k.shape[1]))

    def read_kv(self, n: int):
        i = self.model.info
        k = np.empty((i["block_count"], n, i["kv_dim"]), np.uint16)
        v = np.empty_like(k)
        self._check(lib().vg_stream_read_kv(self.h, _ptr(k), _ptr(v), n))
        return k, v

    # -- decode ----------------------------------------------------------------------------
    def decode_token_gpu_only(self, token_id: int, want_logits: bool = False) -> int:
        pos = self.position
        self._check(lib().vg_decode_token(self.h, int(token_id), int(want_logits)))
        return pos

    def decode_embedding_gpu_only(self, embedding: np.ndarray, want_logits: bool = False) -> int:
        e = np.ascontiguousarray(embedding, np.float32)
        if e.size != self.H:
            raise VoxGenError(-1, f"external embedding has {e.size} floats; expected {self.H}")
        pos = self.position
        self._check(lib().vg_decode_embedding(self.h, _ptr(e), int(want_logits)))
        return pos

    def decode_embedding_from_gpu_only(self, device_ptr: int, want_logits: bool = False) -> int:
        pos = self.position
        self._check(lib().vg_decode_embedding_device(self.h, C.c_void_p(device_ptr), int(want_logits)))
        return pos

    def decode_token(self, token_id: int, top_k: int = 0) -> BaseLmStepResult:
        pos = self.decode_token_gpu_only(token_id, want_logits=True)
        return self.collect_result(pos, top_k)

    def decode_embedding(self, embedding: np.ndarray, top_k: int = 0) -> BaseLmStepResult:
        pos = self.decode_embedding_gpu_only(embedding, want_logits=True)
        return self.collect_result(pos, top_k)

    def prefill_tokens(self, tokens: Sequence[int], top_k_last: int = 0) -> BaseLmStepResult:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if t.size == 0:
            raise VoxGenError(-1, "prefill token list is empty")
        pos = self.position + t.size - 1
        self._check(lib().vg_prefill_tokens(self.h, _ptr(t), t.size, 1))
        return self.collect_result(pos, top_k_last)

    def collect_result(self, position: int, top_k: int) -> BaseLmStepResult:
        res = StepResult()
        top = (TopLogit * max(top_k, 1))()
        self._check(lib().vg_step_result_get(self.h, top_k, C.byref(res), top))
        tops = [TopLogitPy(top[i].token_id, top[i].logit) for i in range(res.n_top)]
        return BaseLmStepResult(position, float("nan"), res.final_hidden_checksum, res.final_hidden_l2, tops)

    def sync(self, timeout_s: float = 60.0) -> None:
        self._check(lib().vg_stream_sync(self.h, int(timeout_s * 1e9)))

    def output(self) -> np.ndarray:
        out = np.empty(self.H, np.float32)
        self._check(lib().vg_copy_output(self.h, _ptr(out), self.H))
        return out

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        self._check(lib().vg_copy_logits(self.h, _ptr(out), self.vocab))
        return out

    def output_buffer(self) -> int:
        """Device address of the final normalised hidden state fp32[H]."""
        p = C.c_void_p()
        self._check(lib().vg_stream_output(self.h, C.byref(p)))
        return p.value

    def logits_buffer(self) -> int:
        p = C.c_void_p()
        self._check(lib().vg_stream_logits(self.h, C.byref(p)))
        return p.value

    def profile_step(self, token_id: int, want_logits: bool = False) -> List[dict]:
        """One token step with per-kernel CUDA-event timing (no graph, no overlap)."""
        cap = 8 * self.model.info["block_count"] + 16
        buf = (KernelTime * cap)()
        n = C.c_uint32()
        self._check(lib().vg_stream_profile_step(self.h, int(token_id), int(want_logits), buf, cap, C.byref(n)))
        return [dict(name=buf[i].name.decode(), layer=buf[i].layer, ms=buf[i].ms, bytes=buf[i].bytes)
                for i in range(n.value)]

    def benchmark(self, token_id: int, warmup: int, iterations: int, want_logits: bool = True) -> dict:
        r = BenchmarkResult()
        self._check(lib().vg_benchmark(self.h, token_id, warmup, iterations, int(want_logits), C.byref(r)))
        return {k: getattr(r, k) for k, _ in r._fields_}


def decode_batch(engines: Sequence[BaseLmEngine], tokens: Sequence[int]) -> None:
    """One batched step over several sessions of the same model."""
    arr = (C.c_void_p * len(engines))(*[e.h for e in engines])
    t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
    rc = lib().vg_decode_batch(arr, len(engines), _ptr(t))
    if rc:
        engines[0]._check(rc)


def outputs(engines: Sequence[BaseLmEngine]) -> np.ndarray:
    """The final hidden states of several sessions, [n, H], with one wait for all the copies
    (vg_copy_outputs): the read-back of a batched step."""
    H = engines[0].H
    out = np.empty((len(engines), H), np.float32)
    arr = (C.c_void_p * len(engines))(*[e.h for e in engines])
    rc = lib().vg_copy_outputs(arr, len(engines), _ptr(out), H)
    if rc:
        engines[0]._check(rc)
    return out


class ResidualEngine(BaseLmEngine):
    """A ResidualLM session: KV cache and the FSQ / fusion / layer launches of one position.

    ``step`` is step_record_submit_gpu_only (src/acoustic.rs:851-869): ``fsq_applied`` selects
    FSQ(BaseLM hidden) as the LM state, else the raw BaseLM hidden (a text-prefix position);
    ``embed`` is the current acoustic embedding (None = zeros). ``output`` is the final
    normalised hidden state; ``state`` reads the FSQ output, the fusion output and the LM state.
    """

    def step(self, base_hidden, embed=None, fsq_applied: bool = True) -> None:
        if isinstance(base_hidden, int):  # device pointers
            self._check(lib().vg_residual_step(self.h, C.c_void_p(base_hidden),
                                               C.c_void_p(embed) if embed is not None else None,
                                               1 if fsq_applied else 0))
            return
        b = np.ascontiguousarray(base_hidden, np.float32)
        e = np.ascontiguousarray(embed, np.float32) if embed is not None else None
        if b.size != self.H or (e is not None and e.size != self.H):
            raise ValueError(f"ResidualLM inputs must have {self.H} values")
        self._check(lib().vg_residual_step_host(self.h, _ptr(b), _ptr(e) if e is not None else None,
                                                1 if fsq_applied else 0))

    def state(self, which: str) -> np.ndarray:
        out = np.empty(self.H, np.float32)
        self._check(lib().vg_residual_copy_state(self.h, RESIDUAL_STATE[which], _ptr(out), self.H))
        return out

    def state_buffer(self, which: str) -> int:
        p = C.c_void_p()
        self._check(lib().vg_residual_state(self.h, RESIDUAL_STATE[which], C.byref(p)))
        return p.value
