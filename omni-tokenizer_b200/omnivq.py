"""OMNIVQ01 model files: writer and seeded random models.

The format is the one omni-tokenizer's loader reads (src/model.cpp:96-205): an
8-byte magic, version 1, the model kind, twelve uint32 configuration fields,
the tensor count, one index record per tensor (name length, dtype 1 = fp32 /
2 = bf16, rank, a reserved zero, data offset and size, the dimensions, the
name), then the tensor data at 64-byte aligned offsets.  Audio models hold
fp32 tensors, image models bf16 ones.  Used to build test fixtures and the
randomly initialised production-shape models the full-encoder benchmarks run.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Dict

import numpy as np

AUDIO, IMAGE = 1, 2
_FIELDS = ("layers", "width", "heads", "ffn", "input_channels", "patch_size", "pool_size",
           "block_size", "pos_height", "pos_width", "code_dim", "vocab_size")


@dataclass
class Config:
    kind: int
    layers: int
    width: int
    heads: int
    ffn: int
    input_channels: int
    patch_size: int
    pool_size: int
    block_size: int
    pos_height: int
    pos_width: int
    code_dim: int
    vocab_size: int


def audio_config(layers=2, width=64, heads=4, ffn=128, mel=16, positions=64, block=16, vocab=256):
    return Config(AUDIO, layers, width, heads, ffn, mel, 0, 4, block, positions, 1, width, vocab)


def image_config(layers=2, width=64, heads=4, ffn=128, patch=8, grid=4, code_dim=16, vocab=256):
    return Config(IMAGE, layers, width, heads, ffn, 3, patch, 0, 0, grid, grid, code_dim, vocab)


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest even) and return the 16-bit patterns."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def tensor_shapes(cfg: Config) -> Dict[str, tuple]:
    W, F = cfg.width, cfg.ffn
    out: Dict[str, tuple] = {}
    if cfg.kind == AUDIO:
        out.update({"conv1.weight": (W, cfg.input_channels, 3), "conv1.bias": (W,),
                    "conv2.weight": (W, W, 3), "conv2.bias": (W,),
                    "embed_positions.weight": (cfg.pos_height, W),
                    "codebook.weight": (cfg.vocab_size, W)})
        for l in range(cfg.layers):
            p = f"layers.{l}."
            for n in ("self_attn_layer_norm", "final_layer_norm"):
                out[p + n + ".weight"] = (W,)
                out[p + n + ".bias"] = (W,)
            for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
                out[p + "self_attn." + n + ".weight"] = (W, W)
            for n in ("q_proj", "v_proj", "out_proj"):
                out[p + "self_attn." + n + ".bias"] = (W,)
            out[p + "fc1.weight"] = (F, W)
            out[p + "fc1.bias"] = (F,)
            out[p + "fc2.weight"] = (W, F)
            out[p + "fc2.bias"] = (W,)
    else:
        P = cfg.patch_size
        out.update({"patch_embed.proj.weight": (W, 3, P, P), "patch_embed.proj.bias": (W,),
                    "pos_embed": (1, cfg.pos_height * cfg.pos_width, W),
                    "quant_conv.weight": (cfg.code_dim, W, 1, 1), "quant_conv.bias": (cfg.code_dim,),
                    "quantize.embedding.weight": (cfg.vocab_size, cfg.code_dim)})
        for l in range(cfg.layers):
            p = f"blocks.{l}."
            for n in ("norm1", "norm2"):
                out[p + n + ".weight"] = (W,)
                out[p + n + ".bias"] = (W,)
            out[p + "attn.qkv.weight"] = (3 * W, W)
            out[p + "attn.qkv.bias"] = (3 * W,)
            out[p + "attn.proj.weight"] = (W, W)
            out[p + "attn.proj.bias"] = (W,)
            out[p + "mlp.fc1.weight"] = (F, W)
            out[p + "mlp.fc1.bias"] = (F,)
            out[p + "mlp.fc2.weight"] = (W, F)
            out[p + "mlp.fc2.bias"] = (W,)
    return out


def _random_tensor(rng, name, shape) -> np.ndarray:
    if name.endswith("norm.weight") or ".norm1.weight" in name or ".norm2.weight" in name \
            or name.endswith("_layer_norm.weight"):
        a = 1.0 + 0.05 * rng.standard_normal(shape)
    elif name.endswith(".bias"):
        a = 0.02 * rng.standard_normal(shape)
    elif name in ("codebook.weight", "quantize.embedding.weight"):
        a = rng.standard_normal(shape)
    elif name in ("embed_positions.weight", "pos_embed"):
        a = 0.1 * rng.standard_normal(shape)
    else:
        fan_in = int(np.prod(shape[1:]))
        a = rng.standard_normal(shape) / np.sqrt(max(fan_in, 1))
    return a.astype(np.float32)


def random_tensors(cfg: Config, seed: int = 0) -> Dict[str, np.ndarray]:
    """Seeded weights: N(0, 1/fan_in) matrices, N(1, 0.05) norm scales, N(0, 0.02)
    biases, N(0, 1) codebook rows, positions with standard deviation 0.1."""
    rng = np.random.default_rng(seed)
    return {name: _random_tensor(rng, name, shape) for name, shape in tensor_shapes(cfg).items()}


def write_model(path, cfg: Config, tensors) -> None:
    """tensors: a dict name -> array, or a callable name -> array (called once per
    tensor, in index order, so that large models never sit in memory whole)."""
    get = tensors if callable(tensors) else tensors.__getitem__
    names = list(tensor_shapes(cfg))
    shapes = tensor_shapes(cfg)
    dtype = 1 if cfg.kind == AUDIO else 2
    esize = 4 if dtype == 1 else 2
    head = b"OMNIVQ01" + struct.pack("<II", 1, cfg.kind)
    head += struct.pack("<12I", *[getattr(cfg, f) for f in _FIELDS])
    head += struct.pack("<I", len(names))
    index_len = sum(4 * 4 + 8 * 2 + 8 * len(shapes[n]) + len(n.encode()) for n in names)
    offset = (len(head) + index_len + 63) // 64 * 64
    records, offsets = [], []
    for n in names:
        size = int(np.prod(shapes[n]))
        nb = n.encode()
        records.append(struct.pack("<IIIIQQ", len(nb), dtype, len(shapes[n]), 0, offset, size * esize)
                       + struct.pack(f"<{len(shapes[n])}Q", *shapes[n]) + nb)
        offsets.append(offset)
        offset = (offset + size * esize + 63) // 64 * 64
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"".join(records))
        for n, off in zip(names, offsets):
            a = np.ascontiguousarray(get(n), np.float32)
            assert a.shape == shapes[n], n
            f.seek(off)
            f.write(a.tobytes() if dtype == 1 else _bf16_bits(a).tobytes())


def write_random_model(path, cfg: Config, seed: int = 0) -> None:
    """Same weights as random_tensors(cfg, seed), generated and written one tensor
    at a time."""
    rng = np.random.default_rng(seed)
    shapes = tensor_shapes(cfg)
    write_model(path, cfg, lambda name: _random_tensor(rng, name, shapes[name]))
