"""Seeded synthetic weights and inputs for the decode workloads.

The reference measures on real audio with HF checkpoints; there is no network
here, so the workloads use random-init weights of the same architecture
(N(0, 0.02) matrices, RMSNorm weights 1, lm_head tied to the embedding) and
N(0, 1) audio-projector embeddings of the same shapes:

* ``b1``:  one stream, 300 audio embeddings + 20 random prompt token ids
  (T = 320), 128 greedy steps as K=8-step graph replays, cache 640;
* ``b48``: 48 streams with prompt lengths uniform in [300, 900] (right-padded
  to the longest), 128 greedy steps, cache 1040;
* ``verify``: one stream, KV cache of 600 positions, verify forwards of
  [last token + 8 random draft ids].
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .engine import GraniteDims

BF16 = torch.bfloat16
GRANITE_1B = GraniteDims()


def weight_shapes(d: GraniteDims):
    out = [("embed_tokens.weight", (d.vocab, d.hidden))]
    for i in range(d.layers):
        p = f"layers.{i}."
        out += [
            (p + "input_layernorm.weight", (d.hidden,)),
            (p + "self_attn.q_proj.weight", (d.n_q * d.head_dim, d.hidden)),
            (p + "self_attn.k_proj.weight", (d.n_kv * d.head_dim, d.hidden)),
            (p + "self_attn.v_proj.weight", (d.n_kv * d.head_dim, d.hidden)),
            (p + "self_attn.o_proj.weight", (d.hidden, d.n_q * d.head_dim)),
            (p + "post_attention_layernorm.weight", (d.hidden,)),
            (p + "mlp.gate_proj.weight", (d.inter, d.hidden)),
            (p + "mlp.up_proj.weight", (d.inter, d.hidden)),
            (p + "mlp.down_proj.weight", (d.hidden, d.inter)),
        ]
    out.append(("norm.weight", (d.hidden,)))
    return out


def make_weights(d: GraniteDims = GRANITE_1B, seed: int = 0, std: float = 0.02, device="cuda") -> dict:
    """N(0, std) bf16 matrices drawn on ``device`` from one seeded generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = {}
    for name, shape in weight_shapes(d):
        if len(shape) == 1:
            w[name] = torch.ones(shape, dtype=BF16, device=device)
        else:
            w[name] = (torch.randn(shape, generator=g, device=device) * std).to(BF16)
    return w


@dataclass
class DecodeInputs:
    inputs_embeds: torch.Tensor  # (B, T, H) bf16, CPU
    prompt_lengths: torch.Tensor  # (B,) int64, CPU
    T: int


def b1_inputs(embed: torch.Tensor, seed: int = 0, n_audio: int = 300, n_prompt: int = 20) -> DecodeInputs:
    """300 N(0,1) audio embeddings followed by the embeddings of 20 random
    prompt ids (merged before the x12 multiplier, as build_inputs_embeds does)."""
    g = torch.Generator().manual_seed(seed)
    audio = torch.randn(1, n_audio, embed.shape[1], generator=g).to(BF16)
    ids = torch.randint(0, embed.shape[0], (n_prompt,), generator=g)
    text = embed[ids.to(embed.device)].to("cpu", BF16).unsqueeze(0)
    emb = torch.cat([audio, text], dim=1)
    return DecodeInputs(emb, torch.tensor([emb.shape[1]]), emb.shape[1])


def batched_inputs(hidden: int, batch: int = 48, seed: int = 0, lo: int = 300, hi: int = 900) -> DecodeInputs:
    g = torch.Generator().manual_seed(seed)
    pl = torch.randint(lo, hi + 1, (batch,), generator=g)
    T = int(pl.max())
    emb = torch.randn(batch, T, hidden, generator=g).to(BF16)
    pos = torch.arange(T)[None, :]
    emb = emb * (pos < pl[:, None]).unsqueeze(-1).to(BF16)  # right padding: zero rows past T_b
    return DecodeInputs(emb, pl, T)
