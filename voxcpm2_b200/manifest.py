"""The reference's model manifest (``model.json``) on the host side.

The reference reads ``model.json`` with a strict schema (src/model_manifest.cpp:37-308,
the types in src/model_manifest.h): every object must hold exactly its fields, and the
settings, tokenizer and component list are validated before any graph loads. This
module applies the same rules and error wording, so that a user of the reference can
point this library at the same file, and maps the settings the patch loop uses onto a
``ModelConfig`` plus the base decoder's LongRoPE factors (``Device.set_rope_factors``).

The architecture sizes (hidden width, heads, FFN width, estimator sizes, vocabulary)
are not in the manifest (the reference reads them from the exported graphs), so the
caller passes them in as a ``ModelConfig``.
"""
from __future__ import annotations

import dataclasses
import json
import math
from pathlib import Path
from typing import Dict, List, Tuple

import numpy as np

from .config import ModelConfig

MODEL_FORMAT_VERSION = 2  # src/model_manifest.h:16

# src/components.h:37-49: component names, and which export one graph per backend
# ("<name>.cpu" / "<name>.vulkan" in params)
COMPONENT_SPECS: Tuple[Tuple[str, bool], ...] = (
    ("text_embed", False),
    ("base_decoder_kv", True),
    ("residual_decoder_kv", True),
    ("fsq", False),
    ("fusion_proj", False),
    ("dit_proj", False),
    ("stop_head", False),
    ("feat_encoder", True),
    ("dit_estimator", True),
    ("audio_vae_encoder", False),
    ("audio_vae_decoder", False),
)


class ManifestError(RuntimeError):
    """A manifest that the reference's loader would reject ("<path>: <reason>")."""


@dataclasses.dataclass(frozen=True)
class RopeSettings:
    type: str
    rope_head_dim: int
    rope_theta: float
    original_max_position_embeddings: int
    short_factor: Tuple[float, ...]
    long_factor: Tuple[float, ...]


@dataclasses.dataclass(frozen=True)
class TokenIds:
    audio_start: int
    audio_end: int
    ref_audio_start: int
    ref_audio_end: int


@dataclasses.dataclass(frozen=True)
class ModelSettings:
    patch_size: int
    feat_dim: int
    latent_dim: int
    chunk_size: int
    decode_chunk_size: int
    encode_sample_rate: int
    out_sample_rate: int
    base_attn_cnt: int
    residual_attn_cnt: int
    tokens: TokenIds
    rope: RopeSettings
    decoder_context_length: int
    kv_head_cnt: int


@dataclasses.dataclass(frozen=True)
class Manifest:
    model_type: str
    format_version: int
    params: Dict[str, Tuple[str, str]]  # component key -> (param file, bin file)
    missing_components: List[str]
    tokenizer_type: str
    tokenizer_json: str
    split_multichar_cjk: bool
    setting: ModelSettings


def _fail(where: str, why: str) -> None:
    raise ManifestError(f"{where}: {why}")


def _exact(obj, where: str, fields: Tuple[str, ...]) -> None:
    """The object holds exactly these fields (require_exact_fields)."""
    if not isinstance(obj, dict):
        _fail(where, "must be an object")
    for f in fields:
        if f not in obj:
            _fail(where, f"missing field {f}")
    for k in obj:
        if k not in fields:
            _fail(where, f"unknown field {k}")


def _typed(obj: dict, field: str, where: str, kind):
    """A field read as the reference's typed read does: any JSON number for int (truncated)
    and float, a JSON boolean for bool, a JSON string for str; anything else is an error."""
    v = obj[field]
    number = isinstance(v, (int, float)) and not isinstance(v, bool)
    ok = {int: number, float: number, bool: isinstance(v, bool), str: isinstance(v, str)}[kind]
    if not ok:
        _fail(f"{where}.{field}", f"must be a {'number' if kind in (int, float) else kind.__name__}")
    return kind(v)


def _factors(obj: dict, field: str, where: str) -> Tuple[float, ...]:
    v = obj[field]
    if not isinstance(v, list) or not all(isinstance(x, (int, float)) and not isinstance(x, bool) for x in v):
        _fail(f"{where}.{field}", "must be an array of numbers")
    return tuple(float(x) for x in v)


def _settings(s: dict) -> ModelSettings:
    _exact(s, "setting", ("patch_size", "feat_dim", "latent_dim", "chunk_size", "decode_chunk_size",
                          "encode_sample_rate", "out_sample_rate", "base_attn_cnt", "residual_attn_cnt", "tokens",
                          "rope", "decoder_context_length", "kv_head_cnt"))
    t = s["tokens"]
    _exact(t, "setting.tokens", ("audio_start", "audio_end", "ref_audio_start", "ref_audio_end"))
    tokens = TokenIds(*(_typed(t, f, "setting.tokens", int)
                        for f in ("audio_start", "audio_end", "ref_audio_start", "ref_audio_end")))
    r = s["rope"]
    _exact(r, "setting.rope", ("type", "rope_head_dim", "rope_theta", "original_max_position_embeddings",
                               "short_factor", "long_factor"))
    rope = RopeSettings(_typed(r, "type", "setting.rope", str), _typed(r, "rope_head_dim", "setting.rope", int),
                        _typed(r, "rope_theta", "setting.rope", float),
                        _typed(r, "original_max_position_embeddings", "setting.rope", int),
                        _factors(r, "short_factor", "setting.rope"), _factors(r, "long_factor", "setting.rope"))
    ints = {f: _typed(s, f, "setting", int) for f in ("patch_size", "feat_dim", "latent_dim", "chunk_size",
                                                      "decode_chunk_size", "encode_sample_rate", "out_sample_rate",
                                                      "base_attn_cnt", "residual_attn_cnt", "decoder_context_length",
                                                      "kv_head_cnt")}
    return ModelSettings(tokens=tokens, rope=rope, **ints)


def _validate_settings(st: ModelSettings) -> None:
    """validate_settings, src/model_manifest.cpp:167-217."""
    for f in ("patch_size", "feat_dim", "latent_dim", "chunk_size", "decode_chunk_size", "encode_sample_rate",
              "out_sample_rate", "base_attn_cnt", "residual_attn_cnt", "decoder_context_length", "kv_head_cnt"):
        if getattr(st, f) <= 0:
            _fail(f"setting.{f}", "must be positive")
    ids = [st.tokens.audio_start, st.tokens.audio_end, st.tokens.ref_audio_start, st.tokens.ref_audio_end]
    if any(i < 0 for i in ids):
        _fail("setting.tokens", "token ids must not be negative")
    if len(set(ids)) != len(ids):
        _fail("setting.tokens", "token ids must be distinct")
    r = st.rope
    if r.type != "LongRoPE":
        _fail("setting.rope.type", "must be LongRoPE")
    if r.rope_head_dim <= 0 or r.rope_head_dim % 2 != 0:
        _fail("setting.rope.rope_head_dim", "must be a positive even number")
    if not math.isfinite(r.rope_theta) or r.rope_theta <= 0.0:
        _fail("setting.rope.rope_theta", "must be finite and positive")
    if r.original_max_position_embeddings <= 0:
        _fail("setting.rope.original_max_position_embeddings", "must be positive")
    n = r.rope_head_dim // 2
    if len(r.short_factor) != n or len(r.long_factor) != n:
        _fail("setting.rope", "factor lengths must equal rope_head_dim / 2")
    if not all(math.isfinite(f) and f > 0.0 for f in r.short_factor + r.long_factor):
        _fail("setting.rope", "factors must be finite and positive")


def _validate_components(m: Manifest) -> None:
    """validate_components, src/model_manifest.cpp:219-269: every component either has
    its params (both backends for a dual-backend one) or is declared missing."""
    missing = set()
    for name in m.missing_components:
        if name in missing:
            _fail("missing_components", f"duplicate component {name}")
        missing.add(name)
    names = {name for name, _ in COMPONENT_SPECS}
    keys = set()
    for name, dual in COMPONENT_SPECS:
        keys.update((f"{name}.cpu", f"{name}.vulkan") if dual else (name,))
    for name in missing:
        if name not in names:
            _fail("missing_components", f"unknown component {name}")
    for key, (param, binf) in m.params.items():
        if key not in keys:
            _fail("params", f"unknown component key {key}")
        if not param or not binf:
            _fail(f"params.{key}", "param and bin must not be empty")
    for name, dual in COMPONENT_SPECS:
        if dual:
            cpu, vk = f"{name}.cpu" in m.params, f"{name}.vulkan" in m.params
            if cpu != vk:
                _fail("params", f"dual-backend component is incomplete: {name}")
            has = cpu and vk
        else:
            has = name in m.params
        if (name in missing) == has:
            _fail("missing_components", f"component has params but is declared missing: {name}" if has
                  else f"component has no params but is not declared missing: {name}")


def parse_manifest(doc) -> Manifest:
    """A decoded model.json document, validated as load_model_manifest does."""
    _exact(doc, "model.json", ("model_type", "format_version", "params", "missing_components", "tokenizer",
                               "setting"))
    if not isinstance(doc["params"], dict):
        _fail("model.json.params", "must be an object")
    params = {}
    for key, files in doc["params"].items():
        _exact(files, "params.<component>", ("param", "bin"))
        params[key] = (_typed(files, "param", "params.<component>", str),
                       _typed(files, "bin", "params.<component>", str))
    mc = doc["missing_components"]
    if not isinstance(mc, list) or not all(isinstance(x, str) for x in mc):
        _fail("model.json.missing_components", "must be an array of strings")
    tok = doc["tokenizer"]
    _exact(tok, "tokenizer", ("type", "tokenizer_json", "split_multichar_cjk"))
    m = Manifest(model_type=_typed(doc, "model_type", "model.json", str),
                 format_version=_typed(doc, "format_version", "model.json", int), params=params,
                 missing_components=list(mc), tokenizer_type=_typed(tok, "type", "tokenizer", str),
                 tokenizer_json=_typed(tok, "tokenizer_json", "tokenizer", str),
                 split_multichar_cjk=_typed(tok, "split_multichar_cjk", "tokenizer", bool),
                 setting=_settings(doc["setting"]))
    # validate_manifest, src/model_manifest.cpp:271-289
    if m.model_type != "voxcpm2_tts":
        _fail("model_type", "must be voxcpm2_tts")
    if m.format_version != MODEL_FORMAT_VERSION:
        _fail("format_version", f"must be {MODEL_FORMAT_VERSION}")
    if m.tokenizer_type != "voxcpm2_tokenizer_json":
        _fail("tokenizer.type", "must be voxcpm2_tokenizer_json")
    if not m.tokenizer_json:
        _fail("tokenizer.tokenizer_json", "must not be empty")
    if not m.split_multichar_cjk:
        _fail("tokenizer.split_multichar_cjk", "must be true for this runtime")
    _validate_settings(m.setting)
    _validate_components(m)
    return m


def load_manifest(path) -> Manifest:
    """load_model_manifest (src/model_manifest.cpp:291-308): read and validate a file;
    every failure is a ManifestError naming the file."""
    path = Path(path)
    try:
        text = path.read_text(encoding="utf-8")
    except OSError:
        raise ManifestError(f"cannot open {path}") from None
    try:
        return parse_manifest(json.loads(text))
    except ManifestError as e:
        raise ManifestError(f"invalid {path}: {e}") from None
    except json.JSONDecodeError as e:
        raise ManifestError(f"invalid {path}: {e}") from None


def model_config(m: Manifest, arch: ModelConfig) -> ModelConfig:
    """The patch loop's settings from the manifest (Synthesizer::Impl::load_manifest,
    src/synthesizer.cpp:812-836) over the architecture sizes in 'arch'."""
    st = m.setting
    if st.rope.rope_head_dim != arch.head_dim:
        raise ManifestError(f"setting.rope.rope_head_dim: {st.rope.rope_head_dim} does not match the decoder's "
                            f"head dim {arch.head_dim}")
    return dataclasses.replace(arch, base_layers=st.base_attn_cnt, res_layers=st.residual_attn_cnt,
                               kv_heads=st.kv_head_cnt, patch_size=st.patch_size, feat_dim=st.feat_dim,
                               audio_start_token=st.tokens.audio_start, rope_theta=st.rope.rope_theta,
                               rope_original_max=st.rope.original_max_position_embeddings)


def rope_factors(m: Manifest) -> Tuple[np.ndarray, np.ndarray]:
    """(short_factor, long_factor) for Device.set_rope_factors."""
    return (np.asarray(m.setting.rope.short_factor, np.float32), np.asarray(m.setting.rope.long_factor, np.float32))
