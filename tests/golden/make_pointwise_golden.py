"""Generate the golden vectors that pin the RMSNorm / RoPE / SwiGLU oracle.

The reference has no code for these kernels (README.md:16-18 lists them as
planned), so the pin is the Llama-family modules of the transformers package
in this image, run on CPU in the storage dtype:

    python tests/golden/make_pointwise_golden.py

Writes tests/golden/pointwise_golden.npz (small, committed): seeded inputs
and the outputs of
  * transformers.models.llama.modeling_llama.LlamaRMSNorm (fp16 and bf16;
    a fused residual case is the same module applied to rnd(x + residual)),
  * LlamaRotaryEmbedding + apply_rotary_pos_emb (NeoX pairing, theta 10000
    and 500000, explicit positions) on fp16 q/k, and the same on float32
    copies of them (a tighter pin: no fp16 rounding of cos/sin),
  * LlamaMLP's activation product act_fn(gate) * up with SiLU (fp16, bf16).
fp16 values are stored as float16, the rest as float32 (both exact).
"""
from __future__ import annotations

import os

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "pointwise_golden.npz")


def main() -> None:
    import transformers
    from transformers import LlamaConfig
    from transformers.models.llama import modeling_llama as ml

    g = torch.Generator().manual_seed(20240611)
    rec: dict[str, np.ndarray] = {"transformers_version": np.array(transformers.__version__)}

    def f32(t):
        return t.numpy() if t.dtype == torch.float16 else t.float().numpy()

    # RMSNorm: plain and on a residual sum, fp16 and bf16.
    for dt, name in ((torch.float16, "f16"), (torch.bfloat16, "bf16")):
        rows, hidden, eps = 4, 256, 1e-6
        x = (torch.randn(rows, hidden, generator=g) * 1.5).to(dt)
        res = torch.randn(rows, hidden, generator=g).to(dt)
        w = (1.0 + 0.25 * torch.randn(hidden, generator=g)).to(dt)
        norm = ml.LlamaRMSNorm(hidden, eps=eps).to(dt)
        with torch.no_grad():
            norm.weight.copy_(w)
            y = norm(x)
            s = x + res                      # storage-dtype add, as a residual stream does
            y_res = norm(s)
        rec[f"rms_{name}_x"], rec[f"rms_{name}_res"], rec[f"rms_{name}_w"] = f32(x), f32(res), f32(w)
        rec[f"rms_{name}_y"], rec[f"rms_{name}_s"], rec[f"rms_{name}_yres"] = f32(y), f32(s), f32(y_res)
        rec[f"rms_{name}_eps"] = np.array(eps)

    # RoPE (NeoX pairing): q [B, H_q, S, D], k [B, H_kv, S, D].
    for theta, tag in ((10000.0, "t1e4"), (500000.0, "t5e5")):
        B, Hq, Hkv, S, D = 1, 4, 2, 16, 64
        cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D,
                          rope_theta=theta, max_position_embeddings=4096)
        if getattr(cfg, "rope_parameters", None) is not None:
            cfg.rope_parameters["rope_theta"] = theta
        rot = ml.LlamaRotaryEmbedding(cfg)
        q = torch.randn(B, Hq, S, D, generator=g).to(torch.float16)
        k = torch.randn(B, Hkv, S, D, generator=g).to(torch.float16)
        pos = torch.randint(0, 2048, (B, S), generator=g)
        with torch.no_grad():
            cos, sin = rot(q, pos)
            qo, ko = ml.apply_rotary_pos_emb(q, k, cos, sin)
            cos32, sin32 = rot(q.float(), pos)
            qo32, ko32 = ml.apply_rotary_pos_emb(q.float(), k.float(), cos32, sin32)
        rec[f"rope_{tag}_q"], rec[f"rope_{tag}_k"] = f32(q), f32(k)
        rec[f"rope_{tag}_pos"] = pos.numpy().astype(np.int32)
        rec[f"rope_{tag}_qo"], rec[f"rope_{tag}_ko"] = f32(qo), f32(ko)
        rec[f"rope_{tag}_qo32"], rec[f"rope_{tag}_ko32"] = f32(qo32), f32(ko32)
        rec[f"rope_{tag}_inv_freq"] = rot.inv_freq.float().numpy()
        rec[f"rope_{tag}_theta"] = np.array(theta)

    # SwiGLU: act_fn(gate) * up as LlamaMLP applies it.
    for dt, name in ((torch.float16, "f16"), (torch.bfloat16, "bf16")):
        rows, inter = 4, 256
        cfg = LlamaConfig(hidden_size=64, intermediate_size=inter, hidden_act="silu")
        mlp = ml.LlamaMLP(cfg)
        gu = (torch.randn(rows, 2 * inter, generator=g) * 3.0).to(dt)
        with torch.no_grad():
            y = mlp.act_fn(gu[:, :inter]) * gu[:, inter:]
        rec[f"swiglu_{name}_gu"], rec[f"swiglu_{name}_y"] = f32(gu), f32(y)

    np.savez_compressed(OUT, **rec)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
