"""Host-side argument handling shared by the decode and prefill entry points.

Mirrors what the reference's solution wrappers accept
(gdn/decode/solution/triton/kernel.py:85-135, gdn/prefill/solution/triton/kernel.py:272-347,
gdn/decode/solution/cuda/kernel.py:479-531): bf16 q/k/v, fp32 state or None,
gates in bf16 or fp32 (the reference's own tests pass fp32 a/b,
gdn/tests/test_correctness.py:221-223), cu_seqlens int32 or int64.
"""
from __future__ import annotations

import math

import torch

from . import _lib

HEAD_DIM = 128

_GATE_CODES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}
_INDEX_CODES = {torch.int32: _lib.DTYPE_I32, torch.int64: _lib.DTYPE_I64}


def require_cuda(name: str, t: torch.Tensor, device: torch.device) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got device {t.device}); "
                         "this operator has no CPU path")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def as_bf16(name: str, t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    return t.contiguous()


def as_gate(name: str, t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Gate/parameter tensors: bf16 or fp32 pass through, other floats go to fp32."""
    if t.dtype not in _GATE_CODES:
        if not t.dtype.is_floating_point:
            raise TypeError(f"{name} must be a floating tensor, got {t.dtype}")
        t = t.float()
    t = t.contiguous()
    return t, _GATE_CODES[t.dtype]


def as_index(name: str, t: torch.Tensor) -> tuple[torch.Tensor, int]:
    if t.dtype not in _INDEX_CODES:
        raise TypeError(f"{name} must be int32 or int64, got {t.dtype}")
    return t.contiguous(), _INDEX_CODES[t.dtype]


def resolve_scale(scale, head_dim: int = HEAD_DIM) -> float:
    """`scale=None` or 0.0 selects 1/sqrt(D) (gdn/decode/baseline/triton/kernel.py:52-53)."""
    if scale is None:
        return 1.0 / math.sqrt(head_dim)
    if isinstance(scale, torch.Tensor):
        scale = float(scale.item())
    scale = float(scale)
    if scale == 0.0:
        return 1.0 / math.sqrt(head_dim)
    return scale


def check_heads(HQ: int, HV: int, D: int) -> None:
    if D != HEAD_DIM:
        raise ValueError(f"head_size must be {HEAD_DIM}, got {D}")
    if HQ <= 0 or HV % HQ != 0:
        raise ValueError(f"num_v_heads ({HV}) must be a positive multiple of num_q_heads ({HQ})")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()
