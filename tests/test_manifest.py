"""model.json with the reference's strict schema (src/model_manifest.cpp), on the CPU:
the rules of tests/test_model_manifest.cpp applied to a manifest of our own, and the
mapping of its settings onto the patch loop's configuration."""
from __future__ import annotations

import copy
import json

import numpy as np
import pytest

from voxcpm2_b200 import manifest as mf
from voxcpm2_b200.config import BENCH


def manifest_doc():
    """A complete export: every component present, dual-backend ones for both backends."""
    params = {}
    for name, dual in mf.COMPONENT_SPECS:
        for key in ((f"{name}.cpu", f"{name}.vulkan") if dual else (name,)):
            params[key] = {"param": f"{key}.ncnn.param", "bin": f"{name}.ncnn.bin"}
    return {
        "model_type": "voxcpm2_tts",
        "format_version": 2,
        "params": params,
        "missing_components": [],
        "tokenizer": {"type": "voxcpm2_tokenizer_json", "tokenizer_json": "tokenizer.json",
                      "split_multichar_cjk": True},
        "setting": {
            "patch_size": 4, "feat_dim": 64, "latent_dim": 64, "chunk_size": 640, "decode_chunk_size": 1920,
            "encode_sample_rate": 16000, "out_sample_rate": 48000, "base_attn_cnt": 24, "residual_attn_cnt": 8,
            "tokens": {"audio_start": 7001, "audio_end": 7002, "ref_audio_start": 7003, "ref_audio_end": 7004},
            "rope": {"type": "LongRoPE", "rope_head_dim": 64, "rope_theta": 10000.0,
                     "original_max_position_embeddings": 4096,
                     "short_factor": [1.0 + 0.01 * j for j in range(32)],
                     "long_factor": [2.0 + 0.1 * j for j in range(32)]},
            "decoder_context_length": 4, "kv_head_cnt": 2,
        },
    }


def write(tmp_path, doc):
    p = tmp_path / "model.json"
    p.write_text(json.dumps(doc))
    return p


def test_valid_manifest_loads(tmp_path):
    m = mf.load_manifest(write(tmp_path, manifest_doc()))
    assert m.format_version == 2 and m.setting.patch_size == 4
    assert len(m.params) == 15  # 7 single-backend + 4 dual-backend components
    assert m.setting.tokens.audio_start == 7001


def test_incomplete_export_is_representable(tmp_path):
    doc = manifest_doc()
    doc["params"] = {}
    doc["missing_components"] = [name for name, _ in mf.COMPONENT_SPECS]
    assert len(mf.load_manifest(write(tmp_path, doc)).missing_components) == 11


def _edits():
    def drop(path):
        def f(d):
            obj = d
            for k in path[:-1]:
                obj = obj[k]
            del obj[path[-1]]
        return f

    def put(path, value):
        def f(d):
            obj = d
            for k in path[:-1]:
                obj = obj[k]
            obj[path[-1]] = value
        return f

    return {
        "unknown top-level field": put(("extra",), 1),
        "missing setting field": drop(("setting", "feat_dim")),
        "format version": put(("format_version", ), 1),
        "one backend of a dual component": drop(("params", "dit_estimator.cpu")),
        "unknown component key": put(("params", "vocoder"), {"param": "a", "bin": "b"}),
        "present component declared missing": put(("missing_components",), ["fsq"]),
        "absent component not declared missing": drop(("params", "stop_head")),
        "duplicate missing component": lambda d: (d["params"].pop("fsq"),
                                                  d.__setitem__("missing_components", ["fsq", "fsq"])),
        "short factor table": put(("setting", "rope", "short_factor"), [1.0] * 31),
        "non-positive factor": put(("setting", "rope", "long_factor"), [0.0] * 32),
        "extra tokenizer field": put(("tokenizer", "vocab"), "x"),
        "tokenizer split off": put(("tokenizer", "split_multichar_cjk"), False),
        "rope type": put(("setting", "rope", "type"), "RoPE"),
        "odd rope head dim": put(("setting", "rope", "rope_head_dim"), 63),
        "repeated token ids": put(("setting", "tokens", "audio_end"), 7001),
        "negative token id": put(("setting", "tokens", "ref_audio_end"), -1),
        "zero layers": put(("setting", "base_attn_cnt"), 0),
        "empty bin name": put(("params", "fsq"), {"param": "fsq.param", "bin": ""}),
        "string where a number belongs": put(("setting", "patch_size"), "4"),
    }


@pytest.mark.parametrize("what", sorted(_edits()))
def test_invalid_manifests_are_rejected(tmp_path, what):
    doc = copy.deepcopy(manifest_doc())
    _edits()[what](doc)
    with pytest.raises(mf.ManifestError, match="invalid .*model.json"):
        mf.load_manifest(write(tmp_path, doc))


def test_unreadable_and_malformed_files(tmp_path):
    with pytest.raises(mf.ManifestError, match="cannot open"):
        mf.load_manifest(tmp_path / "absent.json")
    p = tmp_path / "model.json"
    p.write_text("{not json")
    with pytest.raises(mf.ManifestError, match="invalid"):
        mf.load_manifest(p)


def test_settings_map_onto_the_patch_loop(tmp_path):
    m = mf.load_manifest(write(tmp_path, manifest_doc()))
    cfg = mf.model_config(m, BENCH)
    assert (cfg.base_layers, cfg.res_layers, cfg.kv_heads, cfg.patch_size, cfg.feat_dim) == (24, 8, 2, 4, 64)
    assert cfg.audio_start_token == 7001 and cfg.rope_original_max == 4096 and cfg.rope_theta == 10000.0
    assert (cfg.hidden, cfg.ffn, cfg.q_heads) == (BENCH.hidden, BENCH.ffn, BENCH.q_heads)
    short, long = mf.rope_factors(m)
    assert short.dtype == np.float32 and short.shape == (32,) and long[1] == np.float32(2.1)
    doc = manifest_doc()
    doc["setting"]["rope"]["rope_head_dim"] = 128
    doc["setting"]["rope"]["short_factor"] = [1.0] * 64
    doc["setting"]["rope"]["long_factor"] = [1.0] * 64
    with pytest.raises(mf.ManifestError, match="head dim"):
        mf.model_config(mf.load_manifest(write(tmp_path, doc)), BENCH)
