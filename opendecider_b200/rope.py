"""RoPE cos/sin tables of Qwen3_5TextRotaryEmbedding (transformers models/qwen3_5/modeling_qwen3_5.py:85-155) for text
positions with partial_rotary_factor 1.0: inv_freq = 1 / theta^(arange(0, D, 2) / D) computed in fp32 on the CPU (as
the HF module builds its buffer), freqs = pos * inv_freq, emb = cat(freqs, freqs), cos/sin in fp32 then cast to the
activation dtype. Built once per backbone; od_qk_norm_rope indexes them by each token's position."""
from __future__ import annotations

import torch


def rope_tables(D: int, theta: float, n_pos: int, dtype=torch.bfloat16, device="cuda"):
    inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(dtype=torch.float) / D))
    pos = torch.arange(n_pos, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos().to(dtype).to(device).contiguous(), emb.sin().to(dtype).to(device).contiguous()
