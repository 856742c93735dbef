"""RoPE cos/sin tables.

Values follow the HF Granite rotary embedding the reference runs
(transformers models/granite/modeling_granite.py:338-365): fp32
``inv_freq = 1 / theta ** (arange(0, d, 2) / d)``, fp32 ``pos * inv_freq``,
``cos``/``sin`` in fp32, cast to bf16.  Since ``emb = cat(freqs, freqs)``, only
the first ``d/2`` columns are stored.  Computed once on the host CPU.
"""

from __future__ import annotations

import torch


def inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))


def rope_tables(head_dim: int, theta: float, max_pos: int):
    invf = inv_freq(head_dim, theta)  # [d/2] fp32
    pos = torch.arange(max_pos, dtype=torch.int64).float()
    # (inv_freq[:, None] @ pos[None, :]) in the reference: one fp32 product per entry
    freqs = (invf[None, :, None] @ pos[None, None, :]).transpose(1, 2)[0]  # [max_pos, d/2]
    return freqs.cos().to(torch.bfloat16).contiguous(), freqs.sin().to(torch.bfloat16).contiguous()
