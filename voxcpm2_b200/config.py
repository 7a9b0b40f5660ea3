"""Model description of the VoxCPM2 patch loop and its synthetic stand-ins.

The reference reads these dimensions from ``model.json`` (src/model_manifest.cpp:145-172,
written by tools/export_assets.py:65-90). No checkpoint is available here, so the
sizes below are the scaled-down synthetic shapes of the benchmark workloads
(hidden 1024, 16 query / 2 KV heads of 64, SwiGLU 4096, 24 base / 8 residual
layers, a 12-layer DiT of width 1024) with random fp16 weights.

Layers whose math lives in the upstream ``voxcpm`` package (not vendored with the
reference) are given these stand-in definitions, shared by the CUDA library and
the CPU oracle:

* ``fsq``          in_proj(H -> fsq_dim) + tanh + round(x * s) / s + out_proj(fsq_dim -> H)
                   (finite scalar quantisation, round half to even).
* ``feat_encoder`` frames [P][D] flattened -> Linear(P*D -> H) -> SiLU -> Linear(H -> H).
* ``stop_head``    head(SiLU(proj(h))), proj H -> H with bias, head H -> 2 without bias
                   (export_components.py:581-589 with stop_actn = SiLU).
* DiT time MLPs    linear_2(SiLU(linear_1(emb))), both Hd -> Hd with bias.
* ``dit_proj``     lm_proj and res_proj each H -> Hd, concatenated to the two mu tokens
                   (export_components.py:571-578; mu is reshaped into 2 tokens of Hd at :674-681).

RoPE uses the reference's host table (synthesizer.cpp:928-974) and the rotate_half
convention of ``apply_rotary_pos_emb``. The base decoder's LongRoPE factors are 1
unless set from model.json (``Device.set_rope_factors`` / ``vxc_set_rope_factors``);
the estimator's rotary table keeps factors of 1 (its graph is not available here).
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Tuple

# component ids of src/components.h:16-29
TEXT_EMBED = 0
BASE_DECODER = 1
RESIDUAL_DECODER = 2
FSQ = 3
FUSION_PROJ = 4
DIT_PROJ = 5
STOP_HEAD = 6
FEAT_ENCODER = 7
DIT_ESTIMATOR = 8
COMPONENTS = {
    TEXT_EMBED: "text_embed",
    BASE_DECODER: "base_decoder_kv",
    RESIDUAL_DECODER: "residual_decoder_kv",
    FSQ: "fsq",
    FUSION_PROJ: "fusion_proj",
    DIT_PROJ: "dit_proj",
    STOP_HEAD: "stop_head",
    FEAT_ENCODER: "feat_encoder",
    DIT_ESTIMATOR: "dit_estimator",
}


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    hidden: int = 1024
    ffn: int = 4096
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 64
    base_layers: int = 24
    res_layers: int = 8
    dit_hidden: int = 1024
    dit_ffn: int = 4096
    dit_layers: int = 12
    dit_q_heads: int = 16
    dit_kv_heads: int = 16
    feat_dim: int = 64
    patch_size: int = 4
    vocab: int = 73448
    fsq_dim: int = 256
    fsq_scale: float = 9.0
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_original_max: int = 32768
    base_residual_scale: float = 1.0
    res_residual_scale: float = 1.0
    dit_residual_scale: float = 1.0
    embed_scale: float = 1.0
    audio_start_token: int = 101
    max_generation_patches: int = 2000

    @property
    def latent(self) -> int:
        return self.feat_dim * self.patch_size

    @property
    def dit_head_dim(self) -> int:
        return self.dit_hidden // self.dit_q_heads


# The benchmark shapes: hidden 1024, 16/2 heads of 64, SwiGLU 4096, 24 base,
# 8 residual and 12 DiT layers, 73448-token vocabulary.
BENCH = ModelConfig()

# A small model with the same structure for fast parity runs.
TINY = ModelConfig(
    hidden=256, ffn=512, q_heads=4, kv_heads=2, head_dim=64, base_layers=2, res_layers=2,
    dit_hidden=256, dit_ffn=512, dit_layers=2, dit_q_heads=4, dit_kv_heads=4, vocab=512,
    fsq_dim=64,
)

# Mid-size model: exercises the multi-CTA code paths at modest CPU cost.
SMALL = ModelConfig(
    hidden=512, ffn=1536, q_heads=8, kv_heads=2, head_dim=64, base_layers=4, res_layers=2,
    dit_hidden=512, dit_ffn=1536, dit_layers=3, dit_q_heads=8, dit_kv_heads=8, vocab=2048,
    fsq_dim=128,
)


def decoder_tensors(h: int, f: int, hq: int, hkv: int, d: int, layers: int) -> List[Tuple[str, Tuple[int, ...], str]]:
    """Per-layer tensor order of a decoder blob: kind 'w' = N(0, 0.02), 'g' = ones."""
    out: List[Tuple[str, Tuple[int, ...], str]] = []
    for i in range(layers):
        out += [
            (f"layers.{i}.input_layernorm", (h,), "g"),
            (f"layers.{i}.q_proj", (hq * d, h), "w"),
            (f"layers.{i}.k_proj", (hkv * d, h), "w"),
            (f"layers.{i}.v_proj", (hkv * d, h), "w"),
            (f"layers.{i}.o_proj", (h, hq * d), "w"),
            (f"layers.{i}.post_attention_layernorm", (h,), "g"),
            (f"layers.{i}.gate_proj", (f, h), "w"),
            (f"layers.{i}.up_proj", (f, h), "w"),
            (f"layers.{i}.down_proj", (h, f), "w"),
        ]
    out.append(("norm", (h,), "g"))
    return out


def component_tensors(cfg: ModelConfig, component: int) -> List[Tuple[str, Tuple[int, ...], str]]:
    """Tensor order of each component's fp16 blob (the layout vxc_load_weights expects)."""
    H, Hd, D, P, Q = cfg.hidden, cfg.dit_hidden, cfg.feat_dim, cfg.patch_size, cfg.fsq_dim
    if component == TEXT_EMBED:
        return [("embed_tokens", (cfg.vocab, H), "w")]
    if component == BASE_DECODER:
        return decoder_tensors(H, cfg.ffn, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.base_layers)
    if component == RESIDUAL_DECODER:
        return decoder_tensors(H, cfg.ffn, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.res_layers)
    if component == FSQ:
        return [("in_proj.weight", (Q, H), "w"), ("in_proj.bias", (Q,), "w"),
                ("out_proj.weight", (H, Q), "w"), ("out_proj.bias", (H,), "w")]
    if component == FUSION_PROJ:
        return [("weight", (H, 2 * H), "w"), ("bias", (H,), "w")]
    if component == DIT_PROJ:
        return [("lm_proj.weight", (Hd, H), "w"), ("lm_proj.bias", (Hd,), "w"),
                ("res_proj.weight", (Hd, H), "w"), ("res_proj.bias", (Hd,), "w")]
    if component == STOP_HEAD:
        return [("stop_proj.weight", (H, H), "w"), ("stop_proj.bias", (H,), "w"),
                ("stop_head.weight", (2, H), "w")]
    if component == FEAT_ENCODER:
        return [("in_proj.weight", (H, P * D), "w"), ("in_proj.bias", (H,), "w"),
                ("enc_to_lm_proj.weight", (H, H), "w"), ("enc_to_lm_proj.bias", (H,), "w")]
    if component == DIT_ESTIMATOR:
        out = [("in_proj.weight", (Hd, D), "w"), ("in_proj.bias", (Hd,), "w"),
               ("cond_proj.weight", (Hd, D), "w"), ("cond_proj.bias", (Hd,), "w")]
        for mlp in ("time_mlp", "delta_time_mlp"):
            out += [(f"{mlp}.linear_1.weight", (Hd, Hd), "w"), (f"{mlp}.linear_1.bias", (Hd,), "w"),
                    (f"{mlp}.linear_2.weight", (Hd, Hd), "w"), (f"{mlp}.linear_2.bias", (Hd,), "w")]
        out += [("decoder." + n, s, k) for n, s, k in decoder_tensors(
            Hd, cfg.dit_ffn, cfg.dit_q_heads, cfg.dit_kv_heads, cfg.dit_head_dim, cfg.dit_layers)]
        out += [("out_proj.weight", (D, Hd), "w"), ("out_proj.bias", (D,), "w")]
        return out
    raise ValueError(f"unknown component {component}")


def component_count(cfg: ModelConfig, component: int) -> int:
    n = 0
    for _, shape, _ in component_tensors(cfg, component):
        k = 1
        for s in shape:
            k *= s
        n += k
    return n


def component_offsets(cfg: ModelConfig, component: int) -> Dict[str, Tuple[int, Tuple[int, ...]]]:
    off = 0
    out: Dict[str, Tuple[int, Tuple[int, ...]]] = {}
    for name, shape, _ in component_tensors(cfg, component):
        k = 1
        for s in shape:
            k *= s
        out[name] = (off, shape)
        off += k
    return out
