"""Seeded synthetic PLaMo-3 model directories (config.json, config-mlx.json, model.safetensors).

The real checkpoint is not available offline, so benches and parity tests run on random-init
weights of the reference architecture: every 2-D tensor ~ normal(0, 0.02) cast to bf16, every
norm weight 1.0, generated in sorted tensor-name order from `torch.Generator().manual_seed(seed)`.
Tensor names and shapes follow Sources/Plamo/Runtime.swift:233-250; the config keys follow the
validation in Runtime.swift:181-189. The 64 local / 64 global RoPE inverse frequencies that the
reference reads from config-mlx.json (Runtime.swift:268-274) are synthesised as
theta ** (-2i / 128) with the config's local (1e4) and global (1e6) thetas.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, asdict
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class ModelConfig:
    hidden_size: int = 1536
    num_hidden_layers: int = 16
    num_attention_heads: int = 16
    num_key_value_heads: int = 1
    head_dim: int = 128
    intermediate_size: int = 6144
    vocab_size: int = 107520
    window_size: int = 2048
    sliding_window_pattern: int = 8

    @property
    def qkv_rows(self) -> int:
        return (self.num_attention_heads + 2 * self.num_key_value_heads) * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    def is_global(self, layer: int) -> bool:
        return layer % self.sliding_window_pattern == self.sliding_window_pattern - 1

    def shapes(self) -> dict:
        d, f = self.hidden_size, self.intermediate_size
        out = {
            "lm_head.weight": [self.vocab_size, d],
            "model.embed_tokens.weight": [self.vocab_size, d],
            "model.norm.weight": [d],
        }
        for i in range(self.num_hidden_layers):
            p = f"model.layers.layers.{i}."
            out[p + "pre_mixer_norm.weight"] = [d]
            out[p + "post_mixer_norm.weight"] = [d]
            out[p + "pre_mlp_norm.weight"] = [d]
            out[p + "post_mlp_norm.weight"] = [d]
            out[p + "mixer.qkv_proj.weight"] = [self.qkv_rows, d]
            out[p + "mixer.o_proj.weight"] = [d, self.q_dim]
            out[p + "mixer.q_norm.weight"] = [self.head_dim]
            out[p + "mixer.k_norm.weight"] = [self.head_dim]
            out[p + "mlp.gate_up_proj.weight"] = [2 * f, d]
            out[p + "mlp.down_proj.weight"] = [d, f]
        return out

    def linear_params(self) -> int:
        return sum(int(np.prod(s)) for n, s in self.shapes().items()
                   if len(s) == 2 and n != "model.embed_tokens.weight")


REFERENCE = ModelConfig()
# The example dims quoted in BASELINE.json (grouped-query attention, 4 KV heads).
EXAMPLE = ModelConfig(hidden_size=2048, num_key_value_heads=4, intermediate_size=5632, vocab_size=80000)
# Small shapes with the same structure, for fast CPU/GPU parity tests (window 32 so rings wrap).
TINY = ModelConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=1,
                   intermediate_size=512, vocab_size=2048, window_size=32, sliding_window_pattern=2)
MICRO = ModelConfig(hidden_size=128, num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1,
                    intermediate_size=256, vocab_size=512, window_size=16, sliding_window_pattern=2)

ROPE_LOCAL_THETA = 10_000.0
ROPE_THETA = 1_000_000.0


def config_json(cfg: ModelConfig) -> dict:
    out = asdict(cfg)
    out.update(tie_word_embeddings=False, scale_embedding=False, model_type="plamo3", dtype="bfloat16",
               rope_theta=ROPE_THETA, rope_local_theta=ROPE_LOCAL_THETA, rope_scaling_factor=256.0,
               rms_norm_eps=1e-6)
    return out


def rope_frequencies(cfg: ModelConfig) -> dict:
    i = np.arange(cfg.head_dim // 2, dtype=np.float64)
    return {"local": (ROPE_LOCAL_THETA ** (-2.0 * i / cfg.head_dim)).tolist(),
            "full": (ROPE_THETA ** (-2.0 * i / cfg.head_dim)).tolist()}


def _bf16_bits(t) -> np.ndarray:
    import torch
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def write_model(model_dir, cfg: ModelConfig = REFERENCE, seed: int = 0, std: float = 0.02) -> Path:
    """Write a complete synthetic model directory; returns its path."""
    import torch
    model_dir = Path(model_dir)
    model_dir.mkdir(parents=True, exist_ok=True)
    (model_dir / "config.json").write_text(json.dumps(config_json(cfg), indent=1) + "\n")
    (model_dir / "config-mlx.json").write_text(json.dumps({"plamo_rope_inv_freq": rope_frequencies(cfg)}) + "\n")
    shapes = cfg.shapes()
    names = sorted(shapes)
    header, offset = {}, 0
    for n in names:
        nbytes = int(np.prod(shapes[n])) * 2
        header[n] = {"dtype": "BF16", "shape": shapes[n], "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    header["__metadata__"] = {"format": "pt"}
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * ((-len(blob)) % 8)
    gen = torch.Generator().manual_seed(seed)
    path = model_dir / "model.safetensors"
    part = path.with_suffix(".part")
    with open(part, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for n in names:
            shape = shapes[n]
            if len(shape) == 1:
                arr = np.full(shape, 0x3F80, dtype=np.uint16)  # 1.0 in bf16
            else:
                t = torch.randn(shape, generator=gen, dtype=torch.float32).mul_(std)
                arr = _bf16_bits(t)
            f.write(arr.tobytes())
    part.replace(path)
    return model_dir


def seeded_tokens(n: int, vocab: int, seed: int = 1) -> list:
    """Uniform token ids in [0, vocab) from `seed` (the benches' synthetic prompts)."""
    import torch
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=gen).tolist()


def read_config(model_dir) -> ModelConfig:
    c = json.loads((Path(model_dir) / "config.json").read_text())
    return ModelConfig(**{k: c[k] for k in asdict(REFERENCE)})
