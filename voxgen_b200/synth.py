"""Seeded synthetic BaseLM models and inputs for the BASELINE configurations.

The VoxCPM2 BaseLM GGUF files are not available, so every model is generated here with the
value distributions the configurations state:

* Q8_0 matrices: int8 quants uniform in [-127, 127], one fp16 scale per 32-element block
  drawn as ``fp16(|N(0, 0.02)| / 127)``;
* F16 matrices and the token-embedding table: ``N(0, 0.02)``;
* norm weights: ``1 + N(0, 0.01)`` in fp32 (attn_norm, ffn_norm, output_norm);
* RoPE: theta 1e4, ``rope.scaling.type = longrope`` with all-ones short/long factors and
  ``context_length == original_context_length``, so ``ext = 1`` and the scaling factor is 1
  (``rope_scaling_factor``, src/baselm.rs:194-205);
* fp16 KV-cache contents and input hidden states: ``N(0, 1)``.

Every tensor draws from its own generator, ``np.random.default_rng([seed, index])``, so a
model is reproducible byte for byte and tensors can be generated lazily while writing.
"""
from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass, replace
from pathlib import Path
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np

from .gguf import (GGML_F16, GGML_F32, GGML_Q8_0, F32, U32, GgufFile, q8_0_pack,
                   storage_bytes, write_gguf)


@dataclass(frozen=True)
class ModelSpec:
    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    fmt: int                   # GGML_Q8_0 or GGML_F16 for the projection matrices
    embd_fmt: int = GGML_F16   # token_embd.weight type
    seed: int = 0
    context_length: int = 32768
    eps: float = 1e-5
    theta: float = 10000.0
    embedding_scale: float = 0.0
    residual_scale: float = 0.0
    logit_scale: float = 0.0
    tied_output: bool = True
    rope_scaling: str = "longrope"
    alignment: int = 32
    # per-matrix formats that differ from `fmt`: pairs (tensor suffix, format), for example
    # (("ffn_down", GGML_F16),) for a model whose projections do not share one format
    fmt_overrides: Tuple[Tuple[str, int], ...] = ()

    def fmt_of(self, suffix: str) -> int:
        return dict(self.fmt_overrides).get(suffix, self.fmt)

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


# BASELINE.json configs (seeds 0-4). cfg0 has no embedding input in the spec; it still
# carries a small token table because the loader requires token_embd.weight.
PRESETS: Dict[str, ModelSpec] = {
    "cfg0": ModelSpec("cfg0", 1, 1024, 16, 2, 64, 4096, 4096, GGML_Q8_0, seed=0),
    "cfg1": ModelSpec("cfg1", 24, 1024, 16, 2, 64, 4096, 73448, GGML_Q8_0, seed=1),
    "cfg2": ModelSpec("cfg2", 28, 2048, 16, 2, 128, 6144, 73448, GGML_Q8_0, seed=2),
    "cfg3": ModelSpec("cfg3", 28, 2048, 16, 2, 128, 6144, 73448, GGML_F16, seed=3),
    "cfg4": ModelSpec("cfg4", 28, 2048, 16, 2, 128, 6144, 73448, GGML_Q8_0, seed=4),
    # small shapes for parity tests (odd row counts, several layers, GQA ratio 4)
    "tiny": ModelSpec("tiny", 2, 256, 8, 2, 32, 608, 512, GGML_Q8_0, seed=11),
    "tiny_f16": ModelSpec("tiny_f16", 2, 256, 8, 2, 32, 608, 512, GGML_F16, seed=12),
    # head_dim 128, the only head size the reference's attn_scores shader reduces correctly
    # (its workgroup is 128 invocations wide): the models the reference shaders are run on
    "pin": ModelSpec("pin", 2, 256, 2, 1, 128, 512, 96, GGML_Q8_0, seed=31),
    "pin_f16": ModelSpec("pin_f16", 2, 256, 2, 1, 128, 512, 96, GGML_F16, seed=32, tied_output=False,
                         embedding_scale=12.0, residual_scale=0.25, logit_scale=0.125),
    # groups of 6 query heads per KV head (the batched merge then loads 2 heads at a time)
    "g6": ModelSpec("g6", 2, 1536, 12, 2, 128, 608, 512, GGML_Q8_0, seed=14),
    # projections in two formats (a Q8_0 model whose down projections are F16, which
    # validate_baselm accepts, src/gguf.rs:135-148): a model the persistent step kernel does not
    # take, so it runs the per-kernel program
    "tiny_mixed": ModelSpec("tiny_mixed", 2, 256, 8, 2, 32, 608, 512, GGML_Q8_0, embd_fmt=GGML_Q8_0,
                            seed=13, fmt_overrides=(("ffn_down", GGML_F16),)),
}

# Runtime inputs per config (BASELINE.json configs and the survey's measurement plan).
CFG_RUNS = {
    "cfg0": dict(prefill_positions=512, steps=1),
    "cfg1": dict(prefill_tokens=128, steps=256),
    "cfg2": dict(prefill_positions=1023, steps=3073, max_context=4096),
    "cfg3": dict(prefill_positions=1023, steps=3073, max_context=4096),
    "cfg4": dict(streams=16, kv_lo=64, kv_hi=4096, steps=256, max_context=4096 + 256),
}


def _rng(seed: int, index: int) -> np.random.Generator:
    return np.random.default_rng([seed, index])


def q8_matrix(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """Q8_0 bytes of a rows x cols matrix with the configs' distributions."""
    qs = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    d = (np.abs(rng.standard_normal((rows, cols // 32), dtype=np.float32)) * 0.02 / 127.0)
    return q8_0_pack(d.astype(np.float16), qs)


def f16_matrix(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    return (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float16)


def norm_vector(rng: np.random.Generator, n: int) -> np.ndarray:
    return (1.0 + 0.01 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)


def _matrix(spec: ModelSpec, fmt: int, rows: int, cols: int, index: int) -> Callable[[], np.ndarray]:
    def gen() -> np.ndarray:
        r = _rng(spec.seed, index)
        return q8_matrix(r, rows, cols) if fmt == GGML_Q8_0 else f16_matrix(r, rows, cols)
    return gen


def build_gguf(spec: ModelSpec) -> Tuple[GgufFile, List[Tuple[str, Tuple[int, ...], int, Callable]]]:
    H, F, KV = spec.hidden, spec.ffn, spec.kv_dim
    meta = {
        "general.architecture": "minicpm4",
        "general.name": f"voxgen-b200-synthetic-{spec.name}",
        "minicpm4.context_length": U32(spec.context_length),
        "minicpm4.embedding_length": U32(H),
        "minicpm4.block_count": U32(spec.layers),
        "minicpm4.feed_forward_length": U32(F),
        "minicpm4.attention.head_count": U32(spec.heads),
        "minicpm4.attention.head_count_kv": U32(spec.kv_heads),
        "minicpm4.attention.key_length": U32(spec.head_dim),
        "minicpm4.rope.dimension_count": U32(spec.head_dim),
        "minicpm4.attention.layer_norm_rms_epsilon": F32(spec.eps),
        "minicpm4.rope.freq_base": F32(spec.theta),
        "minicpm4.rope.scaling.type": spec.rope_scaling,
        "minicpm4.rope.scaling.original_context_length": U32(spec.context_length),
    }
    if spec.embedding_scale:
        meta["minicpm4.embedding_scale"] = F32(spec.embedding_scale)
    if spec.residual_scale:
        meta["minicpm4.residual_scale"] = F32(spec.residual_scale)
    if spec.logit_scale:
        meta["minicpm4.logit_scale"] = F32(spec.logit_scale)
    g = GgufFile(metadata=meta, alignment=spec.alignment)
    plan: List[Tuple[str, Tuple[int, ...], int, Callable]] = []
    idx = 0

    def add(name, dims, ty, gen):
        nonlocal idx
        plan.append((name, tuple(dims), ty, gen))
        idx += 1

    def vec(n, index, ones=False):
        return lambda: (np.ones(n, np.float32) if ones else norm_vector(_rng(spec.seed, index), n))

    add("token_embd.weight", (H, spec.vocab), spec.embd_fmt,
        _matrix(spec, spec.embd_fmt, spec.vocab, H, 0))
    if not spec.tied_output:
        add("output.weight", (H, spec.vocab), spec.embd_fmt,
            _matrix(spec, spec.embd_fmt, spec.vocab, H, 1))
    add("output_norm.weight", (H,), GGML_F32, vec(H, 2))
    if spec.rope_scaling == "longrope":
        add("rope_factors_short.weight", (spec.head_dim // 2,), GGML_F32,
            vec(spec.head_dim // 2, 3, ones=True))
        add("rope_factors_long.weight", (spec.head_dim // 2,), GGML_F32,
            vec(spec.head_dim // 2, 4, ones=True))
    for layer in range(spec.layers):
        base = 16 + 16 * layer
        p = f"blk.{layer}."
        add(p + "attn_norm.weight", (H,), GGML_F32, vec(H, base + 0))
        fq, fo, fg, fd = (spec.fmt_of(n) for n in ("attn_qkv", "attn_output", "ffn_gate_up", "ffn_down"))
        add(p + "attn_q.weight", (H, H), fq, _matrix(spec, fq, H, H, base + 1))
        add(p + "attn_k.weight", (H, KV), fq, _matrix(spec, fq, KV, H, base + 2))
        add(p + "attn_v.weight", (H, KV), fq, _matrix(spec, fq, KV, H, base + 3))
        add(p + "attn_output.weight", (H, H), fo, _matrix(spec, fo, H, H, base + 4))
        add(p + "ffn_norm.weight", (H,), GGML_F32, vec(H, base + 5))
        add(p + "ffn_gate.weight", (H, F), fg, _matrix(spec, fg, F, H, base + 6))
        add(p + "ffn_up.weight", (H, F), fg, _matrix(spec, fg, F, H, base + 7))
        add(p + "ffn_down.weight", (F, H), fd, _matrix(spec, fd, H, F, base + 8))
    return g, plan


class _Deferred:
    """Stands in for an ndarray inside GgufFile until the writer asks for it."""

    def __init__(self, nbytes: int, gen: Callable[[], np.ndarray]):
        self.size = nbytes
        self.gen = gen

    def tofile(self, f) -> None:
        a = self.gen()
        np.ascontiguousarray(a).view(np.uint8).reshape(-1).tofile(f)


def write_model(spec: ModelSpec, path: Path) -> Path:
    from .gguf import Tensor
    g, plan = build_gguf(spec)
    for name, dims, ty, gen in plan:
        g.tensors.append(Tensor(name, dims, ty, _Deferred(storage_bytes(ty, int(np.prod(dims))), gen)))
    tmp = Path(str(path) + f".tmp{os.getpid()}")
    write_gguf(tmp, g)
    tmp.replace(path)
    return path


def spec_digest(spec: ModelSpec) -> str:
    return hashlib.sha1(repr(spec).encode()).hexdigest()[:12]


def model_path(spec: ModelSpec, cache_dir: Optional[Path] = None) -> Path:
    """Generates (once) and returns the GGUF path of ``spec`` under ``cache_dir``
    (default: ``$VOXGEN_MODEL_CACHE`` or ``/tmp/voxgen_b200_models``)."""
    d = Path(cache_dir or os.environ.get("VOXGEN_MODEL_CACHE", "/tmp/voxgen_b200_models"))
    d.mkdir(parents=True, exist_ok=True)
    p = d / f"{spec.name}-{spec_digest(spec)}.gguf"
    if not p.exists():
        write_model(spec, p)
    return p


def preset(name: str, **overrides) -> ModelSpec:
    spec = PRESETS[name]
    return replace(spec, **overrides) if overrides else spec


def kv_prefill(spec: ModelSpec, n_positions: int, seed_index: int = 1000) -> Tuple[np.ndarray, np.ndarray]:
    """fp16 K and V ~N(0,1) in the reference cache layout [layer][pos][kv_dim]
    (store_kv.comp:21 with context = n_positions), returned as uint16 bit patterns."""
    r = _rng(spec.seed, seed_index)
    shape = (spec.layers, n_positions, spec.kv_dim)
    k = r.standard_normal(shape, dtype=np.float32).astype(np.float16).view(np.uint16)
    v = r.standard_normal(shape, dtype=np.float32).astype(np.float16).view(np.uint16)
    return k, v


def hidden_inputs(spec: ModelSpec, n: int, seed_index: int = 2000) -> np.ndarray:
    """fp32 ~N(0,1) input hidden states, shape [n, H]."""
    return _rng(spec.seed, seed_index).standard_normal((n, spec.hidden), dtype=np.float32)


def token_ids(spec: ModelSpec, n: int, seed_index: int = 3000) -> np.ndarray:
    """Uniform random token ids in [0, vocab)."""
    return _rng(spec.seed, seed_index).integers(0, spec.vocab, size=n, dtype=np.uint32)


# ---- acoustic GGUF: ResidualLM + FSQ + fusion ----------------------------------------------

@dataclass(frozen=True)
class AcousticSpec:
    """A synthetic acoustic GGUF (general.architecture = voxcpm-acoustic) whose ResidualLM
    follows the BaseLM ``base``: F16 matrices and biases ~N(0, 0.02), fp32 norms 1 + N(0, 0.01)
    (the tensor table AcousticConfig::validate_tensors checks, src/acoustic.rs:128-187)."""
    name: str
    base: ModelSpec
    layers: int = 2
    latent: int = 64
    fsq_scale: float = 9.0
    seed: int = 40
    alignment: int = 32


ACOUSTIC_PRESETS: Dict[str, AcousticSpec] = {
    # head_dim 32 (GQA 4) like "tiny"; F16 layers as the acoustic GGUF requires
    "res_tiny": AcousticSpec("res_tiny", PRESETS["tiny_f16"], layers=2, latent=64, seed=41),
    # the VoxCPM2 shape: 8 layers, 2048 wide, FSQ latent 512, over cfg2's BaseLM geometry
    "res_cfg2": AcousticSpec("res_cfg2", PRESETS["cfg2"], layers=8, latent=512, seed=42),
}


def _f16_vector(spec: AcousticSpec, n: int, index: int) -> Callable[[], np.ndarray]:
    return lambda: (_rng(spec.seed, index).standard_normal(n, dtype=np.float32) * 0.02).astype(np.float16)


def _f16_mat(spec: AcousticSpec, rows: int, cols: int, index: int) -> Callable[[], np.ndarray]:
    return lambda: f16_matrix(_rng(spec.seed, index), rows, cols)


def build_acoustic_gguf(spec: AcousticSpec) -> Tuple[GgufFile, List[Tuple[str, Tuple[int, ...], int, Callable]]]:
    b = spec.base
    H, F, KV, QR, L = b.hidden, b.ffn, b.kv_dim, b.heads * b.head_dim, spec.latent
    meta = {
        "general.architecture": "voxcpm-acoustic",
        "general.name": f"voxgen-b200-synthetic-{spec.name}",
        "voxcpm.model_version": F32(2.0),
        "voxcpm.residual_lm.n_layer": U32(spec.layers),
        "voxcpm.residual_lm.n_embd": U32(H),
        "voxcpm.residual_lm.no_rope": True,
        "voxcpm.fsq.latent_dim": U32(L),
        "voxcpm.fsq.scale": F32(spec.fsq_scale),
    }
    g = GgufFile(metadata=meta, alignment=spec.alignment)
    plan: List[Tuple[str, Tuple[int, ...], int, Callable]] = []

    def add(name, dims, ty, gen):
        plan.append((name, tuple(dims), ty, gen))

    add("fsq.in_proj.weight", (H, L), GGML_F16, _f16_mat(spec, L, H, 1))
    add("fsq.in_proj.bias", (L,), GGML_F16, _f16_vector(spec, L, 2))
    add("fsq.out_proj.weight", (L, H), GGML_F16, _f16_mat(spec, H, L, 3))
    add("fsq.out_proj.bias", (H,), GGML_F16, _f16_vector(spec, H, 4))
    add("projections.res_fusion_proj.weight", (2 * H, H), GGML_F16, _f16_mat(spec, H, 2 * H, 5))
    add("projections.res_fusion_proj.bias", (H,), GGML_F16, _f16_vector(spec, H, 6))
    add("residual_lm.output_norm.weight", (H,), GGML_F32, lambda: norm_vector(_rng(spec.seed, 7), H))
    for layer in range(spec.layers):
        base = 16 + 16 * layer
        p = f"residual_lm.blk.{layer}."
        add(p + "attn_norm.weight", (H,), GGML_F32, (lambda i: lambda: norm_vector(_rng(spec.seed, i), H))(base))
        add(p + "attn_q.weight", (H, QR), GGML_F16, _f16_mat(spec, QR, H, base + 1))
        add(p + "attn_k.weight", (H, KV), GGML_F16, _f16_mat(spec, KV, H, base + 2))
        add(p + "attn_v.weight", (H, KV), GGML_F16, _f16_mat(spec, KV, H, base + 3))
        add(p + "attn_output.weight", (QR, H), GGML_F16, _f16_mat(spec, H, QR, base + 4))
        add(p + "ffn_norm.weight", (H,), GGML_F32, (lambda i: lambda: norm_vector(_rng(spec.seed, i), H))(base + 5))
        add(p + "ffn_gate.weight", (H, F), GGML_F16, _f16_mat(spec, F, H, base + 6))
        add(p + "ffn_up.weight", (H, F), GGML_F16, _f16_mat(spec, F, H, base + 7))
        add(p + "ffn_down.weight", (F, H), GGML_F16, _f16_mat(spec, H, F, base + 8))
    return g, plan


def acoustic_model_path(spec: AcousticSpec, cache_dir: Optional[Path] = None) -> Path:
    """Generates (once) and returns the acoustic GGUF path of ``spec``."""
    from .gguf import Tensor
    d = Path(cache_dir or os.environ.get("VOXGEN_MODEL_CACHE", "/tmp/voxgen_b200_models"))
    d.mkdir(parents=True, exist_ok=True)
    p = d / f"{spec.name}-{spec_digest(spec)}.gguf"
    if not p.exists():
        g, plan = build_acoustic_gguf(spec)
        for name, dims, ty, gen in plan:
            g.tensors.append(Tensor(name, dims, ty, _Deferred(storage_bytes(ty, int(np.prod(dims))), gen)))
        tmp = Path(str(p) + f".tmp{os.getpid()}")
        write_gguf(tmp, g)
        tmp.replace(p)
    return p


def acoustic_preset(name: str, **overrides) -> AcousticSpec:
    spec = ACOUSTIC_PRESETS[name]
    return replace(spec, **overrides) if overrides else spec
