"""Host-side rotary tables, uploaded once to the GPU.

The reference prepares cos/sin on the host per position
(experiments/lfm25_x8_model.py:23-30, `rotary(position)`; the older loop in
experiments/007_lfm25_npu_chat.py:49-57).  Its PyTorch path computes them
with Lfm2RotaryEmbedding (transformers modeling_lfm2.py:93-132): inverse
frequencies theta^(-2i/64) in fp32, phase = position * inv_freq duplicated to
64 lanes, cos/sin in fp32, cast to bf16.  The same torch CPU operations are
used here so that the table equals the one the reference path would produce;
a table is a model constant (like a weight), built once for all positions.
"""
from __future__ import annotations

import torch

HEAD_DIM = 64
THETA = 1.0e6


def rope_table(num_positions: int, head_dim: int = HEAD_DIM, theta: float = THETA,
               device: torch.device | str | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin as bf16 [num_positions, head_dim] for positions 0..num_positions-1."""
    if num_positions <= 0:
        raise ValueError("num_positions must be positive")
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))
    pos = torch.arange(num_positions, dtype=torch.int64).reshape(1, 1, -1).float()
    freqs = (inv_freq[None, :, None].float() @ pos).transpose(1, 2)[0]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = (emb.cos() * 1.0).to(torch.bfloat16)
    sin = (emb.sin() * 1.0).to(torch.bfloat16)
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos.contiguous(), sin.contiguous()
