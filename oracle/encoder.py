"""Encoder graphs of omni-tokenizer restated over numpy -- TEST INFRASTRUCTURE ONLY.

Only tests/ import this module; the product library never does.

audio() follows the reference's src/runtime.cpp:31-73 and image()
src/runtime.cpp:74-123, over restatements of the CPU backend's operators
(src/cpu.cpp: linear :47-69, norm :71-90, gelu :91-97, add :98-104, bias
:105-110, conv_gather :111-121, pool :171-181, interpolate :182-200,
normalize :201-213; image patches src/internal.h:59-71), rounding to bf16
wherever the backend applies r(x, bf16).  Attention, squares and quantize are
the C restatement in oracle.py (itself pinned to the reference's cpu.cpp).

Every operator takes the rounding profile as a flag.  The reference runs audio
in fp32 and images in bf16; audio(..., bf16=True) is the bf16 audio graph of
this library's opt-in OMNI_B200_AUDIO_BF16 mode (weights and activations in
bf16 with the reference's bf16 rounding points, VQ in fp32 on the bf16
features against the fp32 codebook), which the reference cannot express: its
loader takes fp32 audio models only (src/model.cpp:138).

Summation orders are numpy's (pairwise / BLAS), not the reference's
sequential loops: results agree with the reference to fp32 rounding, and in
the bf16 profile up to occasional one-ulp flips of a rounded intermediate.
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
from scipy.special import erf

from . import oracle as O

AUDIO, IMAGE = 1, 2
_FIELDS = ("layers", "width", "heads", "ffn", "input_channels", "patch_size", "pool_size",
           "block_size", "pos_height", "pos_width", "code_dim", "vocab_size")


def load_model(path):
    """Read an OMNIVQ01 file (format of src/model.cpp:96-205) into (config,
    {name: float32 array in the stored shape})."""
    raw = Path(path).read_bytes()
    assert raw[:8] == b"OMNIVQ01", "not an OMNIVQ01 file"
    version, kind = struct.unpack_from("<II", raw, 8)
    assert version == 1
    cfg = dict(zip(_FIELDS, struct.unpack_from("<12I", raw, 16)))
    cfg["kind"] = kind
    (count,) = struct.unpack_from("<I", raw, 64)
    pos, tensors = 68, {}
    for _ in range(count):
        name_len, dtype, rank, _reserved, offset, nbytes = struct.unpack_from("<IIIIQQ", raw, pos)
        pos += 32
        shape = struct.unpack_from(f"<{rank}Q", raw, pos)
        pos += 8 * rank
        name = raw[pos:pos + name_len].decode()
        pos += name_len
        if dtype == 1:
            a = np.frombuffer(raw, np.float32, nbytes // 4, offset)
        else:
            a = (np.frombuffer(raw, np.uint16, nbytes // 2, offset).astype(np.uint32) << 16).view(np.float32)
        tensors[name] = np.array(a, np.float32).reshape(shape)
    return cfg, tensors


def r(x, bf16):
    x = np.asarray(x, np.float32)
    return O.round_bf16(x) if bf16 else x


def linear(x, w, b, bf16):
    y = np.matmul(x, w.T, dtype=np.float32)
    return r(y + b if b is not None else y, bf16)


def image_conv(x, w, b):
    return r(r(np.matmul(x, w.T, dtype=np.float32), True) + b, True)


def norm(x, w, b, eps, bf16):
    d = np.float32(x.shape[1])
    mean = x.sum(1, dtype=np.float32, keepdims=True) / d
    z = x - mean
    var = (z * z).sum(1, dtype=np.float32, keepdims=True)
    inv = np.float32(1) / np.sqrt(var / d + np.float32(eps))
    return r(z * inv * w + b, bf16)


def gelu(x, bf16):
    x = np.asarray(x, np.float32)
    return r(np.float32(0.5) * x * (np.float32(1) + erf(x * np.float32(0.7071067811865475244))), bf16)


def conv_gather(x, stride):
    rows, cols = x.shape
    out = (rows + stride - 1) // stride
    y = np.zeros((out, cols * 3), np.float32)
    for k in range(3):
        src = np.arange(out) * stride + k - 2
        ok = (src >= 0) & (src < rows)
        y[ok, k::3] = x[src[ok]]
    return y


def pool(x, factor, bf16):
    rows, cols = x.shape
    out = (rows + factor - 1) // factor
    pad = np.zeros((out * factor, cols), np.float32)
    pad[:rows] = x
    return r(pad.reshape(out, factor, cols).sum(1, dtype=np.float32) / np.float32(factor), bf16)


def interpolate(pos, source, height, width, bf16):
    cols = pos.shape[-1]
    grid = pos.reshape(source * source, cols).astype(np.float64)
    y = np.zeros((height * width, cols), np.float32)
    for i in range(height):
        for j in range(width):
            sy = max(np.float32(0), np.float32(np.float32(i + .5) * np.float32(np.float32(source) / np.float32(height))) - np.float32(.5))
            sx = max(np.float32(0), np.float32(np.float32(j + .5) * np.float32(np.float32(source) / np.float32(width))) - np.float32(.5))
            y0, x0 = int(sy), int(sx)
            y1, x1 = min(y0 + 1, source - 1), min(x0 + 1, source - 1)
            fy, fx = np.float32(sy - np.float32(y0)), np.float32(sx - np.float32(x0))
            # fma(a, b, c): exact product plus c, rounded once (through float64).
            a = np.float32((1 - fx) * grid[y0 * source + x0] + np.float32(fx * np.float32(grid[y0 * source + x1])))
            b = np.float32((1 - fx) * grid[y1 * source + x0] + np.float32(fx * np.float32(grid[y1 * source + x1])))
            y[i * width + j] = np.float32((1 - fy) * a.astype(np.float64) + np.float32(fy * b))
    return r(y, bf16)


def normalize(x, bf16):
    n = (x * x).sum(1, dtype=np.float32, keepdims=True)
    n = np.maximum(r(np.sqrt(n), bf16), r(np.float32(1e-12), bf16))
    return r(x / n, bf16)


def image_patches(pixels, patch):
    _, h, w = pixels.shape
    gh, gw = h // patch, w // patch
    p = pixels.reshape(3, gh, patch, gw, patch).transpose(1, 3, 0, 2, 4)
    return r(p.reshape(gh * gw, 3 * patch * patch), True)


def audio(model, mel, valid, bf16=False):
    """codes (uint16) and pre-VQ features of one segment, mel [mel, frames]."""
    cfg, t = model
    w = (lambda n: r(t[n], True)) if bf16 else (lambda n: t[n])
    W = cfg["width"]
    x = r(np.ascontiguousarray(np.asarray(mel, np.float32).T), bf16)

    def lin(v, name):
        b = t.get(name + ".bias")
        return linear(v, w(name + ".weight").reshape(-1, v.shape[1]), None if b is None else w(name + ".bias"), bf16)

    x = gelu(lin(conv_gather(x, 1), "conv1"), bf16)
    x = gelu(lin(conv_gather(x, 2), "conv2"), bf16)
    x = r(x + w("embed_positions.weight")[: x.shape[0]], bf16)
    keys = (valid + 1) // 2
    for i in range(cfg["layers"]):
        p = f"layers.{i}."
        z = norm(x, w(p + "self_attn_layer_norm.weight"), w(p + "self_attn_layer_norm.bias"), 1e-5, bf16)
        q, k, v = (lin(z, p + "self_attn." + n) for n in ("q_proj", "k_proj", "v_proj"))
        z = O.attention(q, k, v, cfg["heads"], cfg["block_size"], keys, False, bf16)
        z = lin(z, p + "self_attn.out_proj")
        x = r(x + z, bf16)
        z = norm(x, w(p + "final_layer_norm.weight"), w(p + "final_layer_norm.bias"), 1e-5, bf16)
        z = lin(gelu(lin(z, p + "fc1"), bf16), p + "fc2")
        x = r(x + z, bf16)
    features = pool(x, cfg["pool_size"], bf16)[: (valid + 7) // 8]
    cb = t["codebook.weight"]
    return O.quantize(features, cb, O.squares(cb)), features


def image(model, pixels):
    """codes (uint16) and L2-normalised features of one CHW image."""
    cfg, t = model
    P, W = cfg["patch_size"], cfg["width"]
    _, h, wd = pixels.shape
    gh, gw = h // P, wd // P
    x = image_conv(image_patches(np.asarray(pixels, np.float32), P), t["patch_embed.proj.weight"].reshape(W, -1),
                   t["patch_embed.proj.bias"])
    x = r(x + interpolate(t["pos_embed"], cfg["pos_height"], gh, gw, True), True)
    for i in range(cfg["layers"]):
        p = f"blocks.{i}."
        z = norm(x, t[p + "norm1.weight"], t[p + "norm1.bias"], 1e-6, True)
        z = linear(z, t[p + "attn.qkv.weight"], t[p + "attn.qkv.bias"], True)
        z = O.attention(z, None, None, cfg["heads"], 0, gh * gw, True, True)
        z = linear(z, t[p + "attn.proj.weight"], t[p + "attn.proj.bias"], True)
        x = r(x + z, True)
        z = norm(x, t[p + "norm2.weight"], t[p + "norm2.bias"], 1e-6, True)
        z = gelu(linear(z, t[p + "mlp.fc1.weight"], t[p + "mlp.fc1.bias"], True), True)
        x = r(x + linear(z, t[p + "mlp.fc2.weight"], t[p + "mlp.fc2.bias"], True), True)
    x = image_conv(x, t["quant_conv.weight"].reshape(cfg["code_dim"], W), t["quant_conv.bias"])
    features = normalize(x, True)
    cb = normalize(t["quantize.embedding.weight"], True)
    return O.quantize(features, cb, O.squares(cb, bf16=True), bf16=True), features
