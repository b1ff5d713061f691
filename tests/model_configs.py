"""Synthetic weights of the benchmark model configurations (architectures only; no checkpoint is
available offline).  Each generator yields (name, shape, dtype, init) in checkpoint order; build()
makes the tensors on a device, seeded per tensor (seed = tensor index)."""

from __future__ import annotations

import torch


def t5_3b_fp32():
    """3B fp32 encoder-decoder: 24 + 24 layers, d_model 2048, gated-GELU FFN 5120, 32 heads x 64,
    relative-position bias 32 buckets x 32 heads, vocab 32128, untied LM head (558 tensors,
    11.4 GB)."""
    d, ff, v = 2048, 5120, 32128
    f = torch.float32
    out = [("shared.weight", (v, d), f, "normal")]
    for i in range(24):
        p = f"encoder.block.{i}."
        out += [(p + f"layer.0.SelfAttention.{w}.weight", (d, d), f, "normal") for w in "qkvo"]
        if i == 0:
            out.append((p + "layer.0.SelfAttention.relative_attention_bias.weight", (32, 32), f, "normal"))
        out += [(p + "layer.0.layer_norm.weight", (d,), f, "ones"),
                (p + "layer.1.DenseReluDense.wi_0.weight", (ff, d), f, "normal"),
                (p + "layer.1.DenseReluDense.wi_1.weight", (ff, d), f, "normal"),
                (p + "layer.1.DenseReluDense.wo.weight", (d, ff), f, "normal"),
                (p + "layer.1.layer_norm.weight", (d,), f, "ones")]
    out.append(("encoder.final_layer_norm.weight", (d,), f, "ones"))
    for i in range(24):
        p = f"decoder.block.{i}."
        out += [(p + f"layer.0.SelfAttention.{w}.weight", (d, d), f, "normal") for w in "qkvo"]
        if i == 0:
            out.append((p + "layer.0.SelfAttention.relative_attention_bias.weight", (32, 32), f, "normal"))
        out.append((p + "layer.0.layer_norm.weight", (d,), f, "ones"))
        out += [(p + f"layer.1.EncDecAttention.{w}.weight", (d, d), f, "normal") for w in "qkvo"]
        out += [(p + "layer.1.layer_norm.weight", (d,), f, "ones"),
                (p + "layer.2.DenseReluDense.wi_0.weight", (ff, d), f, "normal"),
                (p + "layer.2.DenseReluDense.wi_1.weight", (ff, d), f, "normal"),
                (p + "layer.2.DenseReluDense.wo.weight", (d, ff), f, "normal"),
                (p + "layer.2.layer_norm.weight", (d,), f, "ones")]
    out += [("decoder.final_layer_norm.weight", (d,), f, "ones"), ("lm_head.weight", (v, d), f, "normal")]
    return out


def qwen_4b_fp8():
    """Mixed-precision 4B decoder: 36 layers, hidden 2560, intermediate 9728, 32 q / 8 kv heads of
    128, vocab 151936; linear weights float8_e4m3fn = clamp(N(0,1) * 16, +-448) with bf16
    per-128x128-block scales |N(0, 0.02)|; embeddings, LM head and norms bf16 (651 tensors,
    5.2 GB)."""
    h, inter, v, q, kv = 2560, 9728, 151936, 32 * 128, 8 * 128
    b, f8 = torch.bfloat16, torch.float8_e4m3fn
    out = [("model.embed_tokens.weight", (v, h), b, "normal")]

    def lin(name, o, i):
        return [(name + ".weight", (o, i), f8, "fp8"), (name + ".weight_scale_inv", (-(-o // 128), -(-i // 128)), b, "abs")]

    for i in range(36):
        p = f"model.layers.{i}."
        out += lin(p + "self_attn.q_proj", q, h) + lin(p + "self_attn.k_proj", kv, h)
        out += lin(p + "self_attn.v_proj", kv, h) + lin(p + "self_attn.o_proj", h, q)
        out += [(p + "self_attn.q_norm.weight", (128,), b, "normal"), (p + "self_attn.k_norm.weight", (128,), b, "normal")]
        out += lin(p + "mlp.gate_proj", inter, h) + lin(p + "mlp.up_proj", inter, h) + lin(p + "mlp.down_proj", h, inter)
        out += [(p + "input_layernorm.weight", (h,), b, "normal"), (p + "post_attention_layernorm.weight", (h,), b, "normal")]
    out += [("model.norm.weight", (h,), b, "normal"), ("lm_head.weight", (v, h), b, "normal")]
    return out


def whisper_1b5_fp16():
    """fp16 speech encoder-decoder: 32 + 32 layers, d_model 1280, FFN 5120, 20 heads, two input
    conv1d layers over 128 mel bins (kernel 3), vocab 51866, N(0, 0.02) (1259 tensors, 3.1 GB)."""
    d, ff, v = 1280, 5120, 51866
    f = torch.float16

    def attn(p):
        return [(p + "k_proj.weight", (d, d), f, "normal"), (p + "v_proj.weight", (d, d), f, "normal"),
                (p + "v_proj.bias", (d,), f, "normal"), (p + "q_proj.weight", (d, d), f, "normal"),
                (p + "q_proj.bias", (d,), f, "normal"), (p + "out_proj.weight", (d, d), f, "normal"),
                (p + "out_proj.bias", (d,), f, "normal")]

    def norm(p):
        return [(p + ".weight", (d,), f, "normal"), (p + ".bias", (d,), f, "normal")]

    def mlp(p):
        return [(p + "fc1.weight", (ff, d), f, "normal"), (p + "fc1.bias", (ff,), f, "normal"),
                (p + "fc2.weight", (d, ff), f, "normal"), (p + "fc2.bias", (d,), f, "normal")]

    out = [("model.encoder.conv1.weight", (d, 128, 3), f, "normal"), ("model.encoder.conv1.bias", (d,), f, "normal"),
           ("model.encoder.conv2.weight", (d, d, 3), f, "normal"), ("model.encoder.conv2.bias", (d,), f, "normal"),
           ("model.encoder.embed_positions.weight", (1500, d), f, "normal")]
    for i in range(32):
        p = f"model.encoder.layers.{i}."
        out += attn(p + "self_attn.") + norm(p + "self_attn_layer_norm") + mlp(p) + norm(p + "final_layer_norm")
    out += norm("model.encoder.layer_norm")
    out += [("model.decoder.embed_tokens.weight", (v, d), f, "normal"),
            ("model.decoder.embed_positions.weight", (448, d), f, "normal")]
    for i in range(32):
        p = f"model.decoder.layers.{i}."
        out += attn(p + "self_attn.") + norm(p + "self_attn_layer_norm") + attn(p + "encoder_attn.")
        out += norm(p + "encoder_attn_layer_norm") + mlp(p) + norm(p + "final_layer_norm")
    out += norm("model.decoder.layer_norm")
    return out


def build(spec, device) -> list[torch.Tensor]:
    out = []
    for idx, (_, shape, dtype, init) in enumerate(spec):
        g = torch.Generator(device=device).manual_seed(idx)
        if init == "ones":
            out.append(torch.ones(shape, dtype=dtype, device=device))
        elif init == "fp8":
            x = torch.randn(shape, generator=g, device=device) * 16
            out.append(x.clamp(-448, 448).to(dtype))
        elif init == "abs":
            out.append((torch.randn(shape, generator=g, device=device) * 0.02).abs().to(dtype))
        else:
            out.append((torch.randn(shape, generator=g, device=device) * 0.02).to(dtype))
    return out
