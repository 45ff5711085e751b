"""Synthetic Qwen3.5 text checkpoints: ``config.json`` + one ``model.safetensors``.

The tensor names and shapes are those of a Qwen3.5 text decoder as evie-core loads it
(crates/evie-core/src/model.rs:137-203, prefix ``model.language_model.``; conv weights ``[C, 1, K]``).
Every tensor is bf16. Matrices, the conv kernel, ``A_log`` and ``dt_bias`` are N(0, std) drawn in the order
``tensor_specs`` lists them from one ``torch.Generator`` seeded with ``seed``; norm gains are stored as 1.0
(so the ``1 + w`` norms have an effective gain of 2 and the gated norm a gain of 1).
"""
from __future__ import annotations

import json
import os
import struct

# Public Qwen3.5 text-model shapes (0.8B: 24 layers x 3584 neurons; 4B: 32 layers x 9216 neurons). Every fourth
# layer (index % 4 == 3) is gated full attention, the rest are Gated DeltaNet.
QWEN35_0_8B = dict(
    hidden_size=1024, intermediate_size=3584, num_hidden_layers=24, num_attention_heads=8, num_key_value_heads=2,
    head_dim=256, vocab_size=248320, rms_norm_eps=1e-6, linear_conv_kernel_dim=4, linear_key_head_dim=128,
    linear_num_key_heads=16, linear_num_value_heads=16, linear_value_head_dim=128, tie_word_embeddings=True,
    rope_parameters=dict(rope_theta=10_000_000.0, partial_rotary_factor=0.25),
)
QWEN35_4B = dict(
    hidden_size=2560, intermediate_size=9216, num_hidden_layers=32, num_attention_heads=16, num_key_value_heads=4,
    head_dim=256, vocab_size=248320, rms_norm_eps=1e-6, linear_conv_kernel_dim=4, linear_key_head_dim=128,
    linear_num_key_heads=16, linear_num_value_heads=32, linear_value_head_dim=128, tie_word_embeddings=True,
    rope_parameters=dict(rope_theta=10_000_000.0, partial_rotary_factor=0.25),
)


def text_config(base: dict, **over) -> dict:
    cfg = dict(base)
    cfg.update(over)
    n = cfg["num_hidden_layers"]
    every = cfg.pop("full_attention_interval", 4)
    cfg["layer_types"] = ["full_attention" if i % every == every - 1 else "linear_attention" for i in range(n)]
    cfg["model_type"] = "qwen3_5_text"
    return cfg


def tiny_config(**over) -> dict:
    """A small config with the same structure (used by the CPU tests and the smoke check)."""
    base = dict(
        hidden_size=128, intermediate_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
        head_dim=256, vocab_size=512, rms_norm_eps=1e-6, linear_conv_kernel_dim=4, linear_key_head_dim=128,
        linear_num_key_heads=2, linear_num_value_heads=4, linear_value_head_dim=128, tie_word_embeddings=True,
        rope_parameters=dict(rope_theta=10_000_000.0, partial_rotary_factor=0.25),
    )
    base.update(over)
    return text_config(base)


def tensor_specs(cfg: dict):
    """(name, shape, kind) in generation order; kind is 'normal' or 'ones'."""
    p = "model.language_model."
    d, n, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    hk, hv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
    dk, dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
    conv_dim = 2 * hk * dk + hv * dv
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    out = [(p + "embed_tokens.weight", (V, d), "normal")]
    for i, lt in enumerate(cfg["layer_types"]):
        L = f"{p}layers.{i}."
        out.append((L + "input_layernorm.weight", (d,), "ones"))
        if lt == "linear_attention":
            out += [
                (L + "linear_attn.in_proj_qkv.weight", (conv_dim, d), "normal"),
                (L + "linear_attn.in_proj_z.weight", (hv * dv, d), "normal"),
                (L + "linear_attn.in_proj_b.weight", (hv, d), "normal"),
                (L + "linear_attn.in_proj_a.weight", (hv, d), "normal"),
                (L + "linear_attn.conv1d.weight", (conv_dim, 1, cfg["linear_conv_kernel_dim"]), "normal"),
                (L + "linear_attn.A_log", (hv,), "normal"),
                (L + "linear_attn.dt_bias", (hv,), "normal"),
                (L + "linear_attn.norm.weight", (dv,), "ones"),
                (L + "linear_attn.out_proj.weight", (d, hv * dv), "normal"),
            ]
        else:
            out += [
                (L + "self_attn.q_proj.weight", (nh * hd * 2, d), "normal"),
                (L + "self_attn.k_proj.weight", (nkv * hd, d), "normal"),
                (L + "self_attn.v_proj.weight", (nkv * hd, d), "normal"),
                (L + "self_attn.o_proj.weight", (d, nh * hd), "normal"),
                (L + "self_attn.q_norm.weight", (hd,), "ones"),
                (L + "self_attn.k_norm.weight", (hd,), "ones"),
            ]
        out += [
            (L + "post_attention_layernorm.weight", (d,), "ones"),
            (L + "mlp.gate_proj.weight", (n, d), "normal"),
            (L + "mlp.up_proj.weight", (n, d), "normal"),
            (L + "mlp.down_proj.weight", (d, n), "normal"),
        ]
    out.append((p + "norm.weight", (d,), "ones"))
    return out


def write_checkpoint(path: str, cfg: dict, seed: int, std: float = 0.02, device: str = "cpu") -> str:
    """Writes ``config.json`` and ``model.safetensors`` under ``path`` (created). Returns ``path``."""
    import torch

    os.makedirs(path, exist_ok=True)
    specs = tensor_specs(cfg)
    header, off = {}, 0
    for name, shape, _ in specs:
        nbytes = 2
        for s in shape:
            nbytes *= s
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    header["__metadata__"] = {"format": "pt", "generator": f"torch seed={seed} std={std}"}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    gen = torch.Generator(device=device).manual_seed(seed)
    tmp = os.path.join(path, "model.safetensors.partial")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name, shape, kind in specs:
            if kind == "ones":
                t = torch.ones(shape, dtype=torch.bfloat16)
            else:
                t = (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)
            f.write(t.contiguous().view(torch.int16).cpu().numpy().tobytes())
    os.replace(tmp, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return path


def ensure_checkpoint(path: str, cfg: dict, seed: int, device: str = "cpu") -> str:
    """Writes the checkpoint unless an identical one (same config and seed) is already there. Processes sharing the
    path (one per GPU) serialise on an exclusive lock next to it: the first writes, the others find it complete."""
    import fcntl

    stamp = os.path.join(path, "SYNTHETIC")
    want = json.dumps({"cfg": cfg, "seed": seed, "device": device}, sort_keys=True)
    os.makedirs(os.path.dirname(os.path.abspath(path)) or ".", exist_ok=True)
    with open(os.path.abspath(path) + ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if os.path.exists(stamp) and os.path.exists(os.path.join(path, "model.safetensors")):
                with open(stamp) as f:
                    if f.read() == want:
                        return path
            if os.path.exists(stamp):
                os.unlink(stamp)
            write_checkpoint(path, cfg, seed, device=device)
            with open(stamp, "w") as f:
                f.write(want)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return path


def read_tensor(path: str, name: str):
    """One tensor of a checkpoint directory as a numpy array (bf16 widened to f32)."""
    import numpy as np

    for fn in sorted(os.listdir(path)):
        if not fn.endswith(".safetensors"):
            continue
        with open(os.path.join(path, fn), "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(n))
            if name not in header:
                continue
            h = header[name]
            s, e = h["data_offsets"]
            f.seek(8 + n + s)
            raw = f.read(e - s)
        if h["dtype"] == "BF16":
            return (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(h["shape"])
        if h["dtype"] == "F32":
            return np.frombuffer(raw, np.float32).reshape(h["shape"])
        raise ValueError(f"{name}: dtype {h['dtype']}")
    raise KeyError(name)
