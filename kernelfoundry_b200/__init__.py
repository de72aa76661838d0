"""kernelfoundry_b200 -- B200-native (sm_100a) flash-attention forward.

A drop-in for the host launcher of sviraaj/kernelfoundry's flash-attention
kernel: fp16 Q/K/V [B, H, S, D] -> fp32 O, GQA/MQA, D in {16, 64, 128, 256},
prefill and decode.  The kernels live in lib/libkf_attn.so (C ABI:
include/kf_attn.h); this package is the Python host side.

  attention  torch-tensor API + the reference-compatible launcher
  multi_gpu  one-process-per-GPU sharding (batch / KV heads) and the
             cross-GPU split-KV decode (partials + NCCL all-gather + merge)
  pointwise  RMSNorm (plain / fused residual), RoPE, SwiGLU
             (C ABI: include/kf_pointwise.h)
  synth      seeded counter-based N(0,1) fp16 inputs generated on the GPU
             (C ABI: include/kf_synth.h)
  build      nvcc build of the library (sm_100a only)
"""
from ._lib import KFError, lib  # noqa: F401
from .attention import (  # noqa: F401
    combine_packed,
    combine_partials,
    device_error,
    flash_attn_fwd,
    flash_attn_paged,
    flash_attn_partial,
    launch_flash_attn,
    plan,
    workspace_bytes,
)

from .pointwise import fused_add_rms_norm, rms_norm, rope_, swiglu  # noqa: F401
from .synth import NormalStream, fill_normal_f16  # noqa: F401

__version__ = "0.1.0"
