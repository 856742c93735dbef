"""Oracle restatement (torch, CPU) of Starling's Granite greedy-decode path.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

This restates, op for op and rounding point for rounding point, what the
reference runs eagerly:

* one decode forward: ``FusedLLMMega._decode_step_eager``
  (src/starling/granite/llm_mega.py:493-589), whose glue ops are bit-equal to
  the HF Granite modules (tests/test_llm_mega.py:145-170);
* prefill: ``LLMMega.prefill`` (llm_mega.py:176-202) = ``GraniteModel.forward``
  (transformers models/granite/modeling_granite.py:380-445) over the prompt
  with a causal mask over the whole static cache;
* the static cache: ``StaticLayer.update`` (transformers cache_utils.py:308-335),
  i.e. ``index_copy_`` of the new K/V rows at the write slot;
* greedy loops: ``MultiStepLLMMega.generate`` (src/starling/granite/multistep.py:250-333),
  ``BatchedLLMMega.generate`` (src/starling/granite/batched.py:331-437) including
  the right-padding mask (batched.py:180-200) and per-stream RoPE offset
  (batched.py:373-380), and ``SpeculativeDecoder.generate``
  (src/starling/granite/speculative.py:318-567) with its verify mask
  (speculative.py:755-765).

Quantised weights (no counterpart in the reference) enter as the
reference-eager path with each ``nn.Linear`` replaced by the fp32 dequantised
weight: ``y = bf16(x.float() @ W_deq.T)``.
"""

from __future__ import annotations

import math
import os
from contextlib import contextmanager
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from . import quant_ref

BF16 = torch.bfloat16


# --------------------------------------------------------------------------- #
# dims
# --------------------------------------------------------------------------- #
@dataclass(frozen=True)
class Dims:
    hidden: int = 2048
    n_q: int = 16
    n_kv: int = 4
    head_dim: int = 128
    inter: int = 8192
    vocab: int = 100352
    layers: int = 40
    eps: float = 1e-5
    theta: float = 10000.0
    attn_mult: float = 0.0078125
    emb_mult: float = 12.0
    res_mult: float = 0.22
    logits_scaling: float = 8.0


# Granite multipliers come from src/starling/config.py:57-60.
GRANITE_1B_DIMS = Dims()
# Small model for golden fixtures: head_dim stays 128 (the kernels' head size),
# an odd vocabulary exercises the lm_head row tail.
TINY_DIMS = Dims(hidden=512, n_q=4, n_kv=2, head_dim=128, inter=1024, vocab=2051, layers=2)


# --------------------------------------------------------------------------- #
# synthetic weights (deterministic CPU generator, HF parameter names)
# --------------------------------------------------------------------------- #
def weight_shapes(d: Dims) -> list[tuple[str, tuple[int, ...]]]:
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


def make_weights(d: Dims, seed: int = 0, std: float = 0.02, norm_jitter: float = 0.0) -> dict:
    """N(0, std) bf16 matrices, RMSNorm weights 1 (+ optional jitter), tied lm_head.

    Generated in ``weight_shapes`` order from one ``torch.Generator(seed)`` so
    the same weights come out on any host running this torch build.
    """
    gen = torch.Generator().manual_seed(seed)
    w = {}
    for name, shape in weight_shapes(d):
        if len(shape) == 1:
            t = torch.ones(shape)
            if norm_jitter:
                t = t + norm_jitter * torch.randn(shape, generator=gen)
        else:
            t = torch.randn(shape, generator=gen) * std
        w[name] = t.to(BF16)
    return w


def weights_checksum(w: dict) -> float:
    return float(sum(t.float().double().sum().item() * (i + 1) for i, t in enumerate(w.values())))


# --------------------------------------------------------------------------- #
# linear layers (bf16 or dequantised)
# --------------------------------------------------------------------------- #
# Accumulation of the oracle's matmuls.  "bf16": what the reference runs (bf16
# matmuls accumulated in fp32 by the BLAS, in its order).  "f64": the same ops
# and rounding points with every matmul accumulated in float64 and rounded once
# to bf16 -- the most accurate result at each of the reference's rounding
# points, used by the tests to measure how far any accumulation order (the
# BLAS's, the CUDA kernels') sits from it.
ACCUMULATE = "bf16"


@contextmanager
def accumulate(mode: str):
    """Run the oracle's matmuls with ``mode`` ("bf16" or "f64") inside the block."""
    global ACCUMULATE
    assert mode in ("bf16", "f64")
    old, ACCUMULATE = ACCUMULATE, mode
    try:
        yield
    finally:
        ACCUMULATE = old


def _matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if ACCUMULATE == "f64":
        return torch.matmul(a.double(), b.double()).to(BF16)
    return torch.matmul(a, b)


class Linear:
    """``nn.Linear`` stand-in.  ``fmt == 'bf16'`` runs the bf16 matmul the
    reference runs; quantised formats run ``bf16(x.float() @ W_deq.T)``."""

    def __init__(self, w_bf16: torch.Tensor, fmt: str = "bf16"):
        self.fmt = fmt
        self.N, self.K = w_bf16.shape
        if fmt == "bf16":
            self.w = w_bf16
            self.parts = None
        else:
            parts = quant_ref.quantize(fmt, w_bf16.float().numpy())
            self.parts = parts
            self.w = torch.from_numpy(quant_ref.dequantize(fmt, parts))  # fp32

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if ACCUMULATE == "f64":  # every product and sum exact to ~2^-53, one rounding to bf16
            return F.linear(x.double(), self.w.double()).to(BF16)
        if self.fmt == "bf16":
            return F.linear(x, self.w)
        return F.linear(x.float(), self.w).to(BF16)


# --------------------------------------------------------------------------- #
# glue ops (transformers modeling_granite.py / starling llm_kernels.py)
# --------------------------------------------------------------------------- #
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """GraniteRMSNorm (modeling_granite.py:192-197); = llm_kernels._rmsnorm_kernel
    (llm_kernels.py:105-116): x*rsqrt(mean x^2 + eps) in fp32, round to bf16,
    then times the bf16 weight."""
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return w * (xf * torch.rsqrt(var + eps)).to(x.dtype)


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """silu in fp32 rounded to bf16, then times up in bf16 (llm_kernels.py:252-260)."""
    return F.silu(g) * u


def residual_scale(x: torch.Tensor, y: torch.Tensor, alpha: float) -> torch.Tensor:
    """x + bf16(alpha*y) (llm_kernels.py:306-313; modeling_granite.py:273-278)."""
    return x + y * alpha


def inv_freq(d: Dims) -> torch.Tensor:
    """Default RoPE inverse frequencies (modeling_granite.py:338-341)."""
    return 1.0 / (
        d.theta ** (torch.arange(0, d.head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / d.head_dim)
    )


def rope_cos_sin(d: Dims, position_ids: torch.Tensor):
    """GraniteRotaryEmbedding.forward (modeling_granite.py:353-365): fp32
    ``inv_freq (x) pos``, ``cat(freqs, freqs)``, cos/sin, cast to bf16.
    position_ids: (B, T) int64 -> cos, sin (B, T, head_dim) bf16."""
    invf = inv_freq(d)
    inv_exp = invf[None, :, None].float().expand(position_ids.shape[0], -1, 1)
    pos_exp = position_ids[:, None, :].float()
    freqs = (inv_exp @ pos_exp).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(BF16), emb.sin().to(BF16)


def rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """GQA expand (llm_mega.py:446-451)."""
    if n_rep == 1:
        return x
    B, n_kv, S, D = x.shape
    return x[:, :, None, :, :].expand(B, n_kv, n_rep, S, D).reshape(B, n_kv * n_rep, S, D)


# --------------------------------------------------------------------------- #
# model
# --------------------------------------------------------------------------- #
class OracleModel:
    """The decoder's weights as the oracle uses them.  Quantised formats are
    quantised and dequantised here (numpy); with ``workers`` > 1 the layers are
    built on a thread pool (numpy releases the GIL inside its array
    operations; each layer is independent, so the result is the same)."""

    def __init__(self, d: Dims, weights: dict, fmt: str = "bf16", workers: Optional[int] = None):
        self.d = d
        self.fmt = fmt
        self.embed = weights["embed_tokens.weight"]
        self.final_norm = weights["norm.weight"]
        if workers is None:
            workers = min(os.cpu_count() or 1, 16) if fmt != "bf16" and d.layers > 2 else 1
        if workers > 1:
            with ThreadPoolExecutor(workers) as ex:
                head = ex.submit(Linear, self.embed, fmt)
                self.layers = list(ex.map(lambda i: make_layer(d, weights, i, fmt), range(d.layers)))
                self.lm_head = head.result()
        else:
            self.layers = [make_layer(d, weights, i, fmt) for i in range(d.layers)]
            # lm_head is tied to the embedding.
            self.lm_head = Linear(self.embed, fmt)


class OracleCache:
    """StaticCache stand-in: per-layer K/V ``(B, n_kv, max_len, hd)`` bf16."""

    def __init__(self, d: Dims, B: int, max_len: int):
        self.max_len = max_len
        self.k = [torch.zeros(B, d.n_kv, max_len, d.head_dim, dtype=BF16) for _ in range(d.layers)]
        self.v = [torch.zeros(B, d.n_kv, max_len, d.head_dim, dtype=BF16) for _ in range(d.layers)]


def forward(
    m: OracleModel,
    cache: OracleCache,
    hidden: torch.Tensor,
    position_ids: torch.Tensor,
    slot0: int,
    mask: torch.Tensor,
) -> torch.Tensor:
    """One forward of T new tokens per stream on top of the cache.

    hidden: (B, T, H) bf16, already multiplied by the embedding multiplier.
    position_ids: (B, T) RoPE positions.  slot0: cache slot of token 0 (the
    ``cumulative_length`` of every layer).  mask: (B, 1|T, T, max_len) additive
    bf16 mask.  Returns logits (B, T, V) bf16 (already / logits_scaling),
    mirroring llm_mega.py:513-589.
    """
    d = m.d
    T = hidden.shape[1]
    cos, sin = rope_cos_sin(d, position_ids)
    cos4, sin4 = cos.unsqueeze(1), sin.unsqueeze(1)
    slots = torch.arange(T) + slot0
    for li, L in enumerate(m.layers):
        hidden = layer_forward(d, L, cache.k[li], cache.v[li], hidden, cos4, sin4, slots, mask)
    hidden = rmsnorm(hidden, m.final_norm, d.eps)
    return m.lm_head(hidden) / d.logits_scaling


def layer_forward(d: Dims, L: dict, kc: torch.Tensor, vc: torch.Tensor, hidden, cos4, sin4, slots, mask):
    """One decoder layer, the per-layer body of llm_mega.py:523-582."""
    B, T, _ = hidden.shape
    hd, n_q, n_kv = d.head_dim, d.n_q, d.n_kv
    residual = hidden
    normed = rmsnorm(hidden, L["in_norm"], d.eps)
    q = L["q"](normed).view(B, T, n_q, hd).transpose(1, 2)
    k = L["k"](normed).view(B, T, n_kv, hd).transpose(1, 2)
    v = L["v"](normed).view(B, T, n_kv, hd).transpose(1, 2)
    q = q * cos4 + rotate_half(q) * sin4
    k = k * cos4 + rotate_half(k) * sin4
    kc.index_copy_(2, slots, k)
    vc.index_copy_(2, slots, v)
    kr = repeat_kv(kc, n_q // n_kv)
    vr = repeat_kv(vc, n_q // n_kv)
    scores = _matmul(q, kr.transpose(2, 3)) * d.attn_mult
    scores = scores + mask
    attn = F.softmax(scores, dim=-1, dtype=torch.float32).to(BF16)
    ao = _matmul(attn, vr).transpose(1, 2).reshape(B, T, n_q * hd)
    ao = L["o"](ao)
    hidden = residual_scale(residual, ao, d.res_mult)
    residual = hidden
    normed = rmsnorm(hidden, L["post_norm"], d.eps)
    act = silu_mul(L["gate"](normed), L["up"](normed))
    return residual_scale(residual, L["down"](act), d.res_mult)


class DenseLinear(Linear):
    """Linear over an already dequantised fp32 weight (quantised formats)."""

    def __init__(self, w_f32: torch.Tensor, fmt: str):
        self.fmt = fmt
        self.N, self.K = w_f32.shape
        self.w = w_f32
        self.parts = None


def _fused_quant(ws: list, fmt: str) -> list:
    """Quantise the row-concatenation of ``ws`` as one tensor (the packed q|k|v
    and gate|up matrices share one nvfp4 tensor scale), dequantise, split."""
    w = torch.cat(ws, dim=0)
    deq = torch.from_numpy(quant_ref.dequantize(fmt, quant_ref.quantize(fmt, w.float().numpy())))
    return [DenseLinear(t.contiguous(), fmt) for t in deq.split([x.shape[0] for x in ws])]


def make_layer(d: Dims, weights: dict, i: int, fmt: str = "bf16") -> dict:
    p = f"layers.{i}."
    if fmt != "bf16":
        q, k, v = _fused_quant([weights[p + "self_attn.q_proj.weight"], weights[p + "self_attn.k_proj.weight"],
                                weights[p + "self_attn.v_proj.weight"]], fmt)
        gate, up = _fused_quant([weights[p + "mlp.gate_proj.weight"], weights[p + "mlp.up_proj.weight"]], fmt)
        return dict(
            in_norm=weights[p + "input_layernorm.weight"],
            post_norm=weights[p + "post_attention_layernorm.weight"],
            q=q, k=k, v=v, o=Linear(weights[p + "self_attn.o_proj.weight"], fmt),
            gate=gate, up=up, down=Linear(weights[p + "mlp.down_proj.weight"], fmt),
        )
    return dict(
        in_norm=weights[p + "input_layernorm.weight"],
        post_norm=weights[p + "post_attention_layernorm.weight"],
        q=Linear(weights[p + "self_attn.q_proj.weight"], fmt),
        k=Linear(weights[p + "self_attn.k_proj.weight"], fmt),
        v=Linear(weights[p + "self_attn.v_proj.weight"], fmt),
        o=Linear(weights[p + "self_attn.o_proj.weight"], fmt),
        gate=Linear(weights[p + "mlp.gate_proj.weight"], fmt),
        up=Linear(weights[p + "mlp.up_proj.weight"], fmt),
        down=Linear(weights[p + "mlp.down_proj.weight"], fmt),
    )


def make_layer_weights(d: Dims, seed: int = 0, std: float = 0.02) -> dict:
    """Weights of layer 0 only (the one-layer decode case), same generator
    order as :func:`make_weights` minus the embedding and final norm."""
    gen = torch.Generator().manual_seed(seed)
    w = {}
    for name, shape in weight_shapes(Dims(**{**d.__dict__, "layers": 1})):
        if not name.startswith("layers.0."):
            continue
        t = torch.ones(shape) if len(shape) == 1 else torch.randn(shape, generator=gen) * std
        w[name] = t.to(BF16)
    return w


def layer_step_case(d: Dims, seed: int = 0, past: int = 256, std: float = 0.02):
    """The one-layer decode case: layer-0 weights N(0, std), ``past`` cached
    positions of N(0,1) bf16 K/V, input hidden N(0,1) bf16 at position
    ``past``.  Returns (weights, k_cache, v_cache, x, position)."""
    w = make_layer_weights(d, seed, std)
    gen = torch.Generator().manual_seed(seed + 1)
    max_len = past + 1
    kc = torch.zeros(1, d.n_kv, max_len, d.head_dim, dtype=BF16)
    vc = torch.zeros(1, d.n_kv, max_len, d.head_dim, dtype=BF16)
    kc[:, :, :past] = torch.randn(1, d.n_kv, past, d.head_dim, generator=gen).to(BF16)
    vc[:, :, :past] = torch.randn(1, d.n_kv, past, d.head_dim, generator=gen).to(BF16)
    x = torch.randn(1, 1, d.hidden, generator=gen).to(BF16)
    return w, kc, vc, x, past


def layer_step(d: Dims, L: dict, kc, vc, x, position: int):
    """Run one decode step of one layer in place on (kc, vc); return hidden out."""
    pos = torch.tensor([[position]])
    cos, sin = rope_cos_sin(d, pos)
    max_len = kc.shape[2]
    valid = (torch.arange(max_len) <= position).view(1, -1)
    mask = decode_mask(1, max_len, valid)
    return layer_forward(d, L, kc, vc, x, cos.unsqueeze(1), sin.unsqueeze(1),
                         torch.tensor([position]), mask)


NEG = torch.finfo(BF16).min


def decode_mask(B: int, max_len: int, valid: torch.Tensor) -> torch.Tensor:
    """(B,1,1,max_len) additive mask; ``valid`` (B, max_len) bool."""
    m = torch.zeros(B, max_len, dtype=BF16)
    m.masked_fill_(~valid, NEG)
    return m.view(B, 1, 1, max_len)


def prefill_mask(B: int, T: int, max_len: int, prompt_lengths: Optional[torch.Tensor]) -> torch.Tensor:
    """Causal (+ right-padding) mask over the static cache, as
    ``create_causal_mask`` builds it for a StaticCache prefill."""
    q = torch.arange(T)[:, None]
    kpos = torch.arange(max_len)[None, :]
    valid = (kpos <= q).unsqueeze(0).expand(B, T, max_len)
    if prompt_lengths is not None:
        valid = valid & (kpos.unsqueeze(0) < prompt_lengths.view(B, 1, 1))
    m = torch.zeros(B, T, max_len, dtype=BF16)
    m.masked_fill_(~valid, NEG)
    return m.view(B, 1, T, max_len)


def embed_ids(m: OracleModel, ids: torch.Tensor) -> torch.Tensor:
    """``embed_tokens(ids) * 12`` in bf16 (llm_mega.py:514)."""
    return m.embed[ids] * m.d.emb_mult


# --------------------------------------------------------------------------- #
# decoders mirroring the reference's generate loops
# --------------------------------------------------------------------------- #
class OracleDecoder:
    def __init__(self, m: OracleModel, max_cache_len: int, B: int = 1):
        self.m = m
        self.B = B
        self.max_len = max_cache_len
        self.cache = OracleCache(m.d, B, max_cache_len)
        self.pos = 0

    # LLMMega.prefill (llm_mega.py:176-202); batched: batched.py:222-276
    def prefill(self, inputs_embeds: torch.Tensor, prompt_lengths: Optional[torch.Tensor] = None):
        B, T, _ = inputs_embeds.shape
        assert T < self.max_len
        hidden = inputs_embeds.to(BF16) * self.m.d.emb_mult
        pos_ids = torch.arange(T).unsqueeze(0).expand(B, T)
        mask = prefill_mask(B, T, self.max_len, prompt_lengths)
        logits = forward(self.m, self.cache, hidden, pos_ids, 0, mask)
        self.pos = T
        if prompt_lengths is None:
            last = logits[:, -1, :]
        else:
            last = logits[torch.arange(B), prompt_lengths.long() - 1, :]
        self.last_logits = last
        return last.argmax(dim=-1)

    def step(self, tokens: torch.Tensor, rope_pos: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
        """One decode step: tokens (B,), rope positions (B,), valid (B, max_len).
        Writes cache slot ``self.pos`` and returns logits (B, V)."""
        hidden = embed_ids(self.m, tokens.view(self.B, 1))
        mask = decode_mask(self.B, self.max_len, valid)
        logits = forward(self.m, self.cache, hidden, rope_pos.view(self.B, 1), self.pos, mask)
        self.pos += 1
        return logits[:, 0, :]

    # MultiStepLLMMega.generate (multistep.py:250-333) / LLMMega.generate
    # (llm_mega.py:250-324): greedy, stop at EOS or max_new_tokens.
    def generate(self, inputs_embeds: torch.Tensor, max_new_tokens: int, eos: int,
                 record_logits: bool = False):
        assert self.B == 1
        T = inputs_embeds.shape[1]
        if max_new_tokens > self.max_len - T + 1:
            raise ValueError("max_new_tokens would overflow the static KV cache")
        if max_new_tokens <= 0:
            return [], []
        tok = self.prefill(inputs_embeds)
        # The reference does not test the prefill token for EOS; decoding
        # starts regardless (llm_mega.py:288-319, multistep.py:286-328).
        out = [int(tok)]
        logs = [self.last_logits[0].clone()] if record_logits else []
        for i in range(max_new_tokens - 1):
            cur = T + i
            valid = (torch.arange(self.max_len) <= cur).view(1, -1)
            lg = self.step(torch.tensor([out[-1]]), torch.tensor([cur]), valid)
            if record_logits:
                logs.append(lg[0].clone())
            out.append(int(lg[0].argmax()))
            if out[-1] == eos:
                break
        return out, logs

    # BatchedLLMMega.generate (batched.py:331-437)
    def generate_batched(self, inputs_embeds, prompt_lengths, max_new_tokens, eos, pad):
        B, T, _ = inputs_embeds.shape
        pl = torch.full((B,), T, dtype=torch.long) if prompt_lengths is None else prompt_lengths.long()
        pad_offset = T - pl
        first = self.prefill(inputs_embeds, None if prompt_lengths is None else pl)
        gen = [[int(t)] for t in first]
        finished = [g[0] == eos for g in gen]
        nxt = torch.tensor([pad if finished[b] else gen[b][0] for b in range(B)])
        if max_new_tokens <= 1 or all(finished):
            return gen
        kpos = torch.arange(self.max_len)
        for i in range(max_new_tokens - 1):
            cur = T + i
            valid = (kpos[None, :] < pl[:, None]) | ((kpos >= T) & (kpos <= cur))[None, :]
            lg = self.step(nxt, cur - pad_offset, valid)
            new = lg.argmax(dim=-1)
            for b in range(B):
                if not finished[b]:
                    gen[b].append(int(new[b]))
                    if int(new[b]) == eos:
                        finished[b] = True
            nxt = torch.tensor([pad if finished[b] else int(new[b]) for b in range(B)])
            if all(finished):
                break
        return gen

    # SpeculativeDecoder._verify_forward (speculative.py:572-593) with the
    # causal verify mask of speculative.py:755-765; writes slots [start, start+L).
    def verify(self, ids: torch.Tensor, start_pos: int) -> torch.Tensor:
        L = ids.numel()
        hidden = embed_ids(self.m, ids.view(1, L))
        q = torch.arange(start_pos, start_pos + L)[:, None]
        valid = torch.arange(self.max_len)[None, :] <= q
        mask = torch.zeros(L, self.max_len, dtype=BF16)
        mask.masked_fill_(~valid, NEG)
        mask = mask.view(1, 1, L, self.max_len)
        pos_ids = torch.arange(start_pos, start_pos + L).view(1, L)
        return forward(self.m, self.cache, hidden, pos_ids, start_pos, mask)[0]


def speculative_generate(dec: OracleDecoder, inputs_embeds, draft: list[int], max_new_tokens: int,
                         eos: int, min_chunk=8, boundary_chunk=2, max_chunk=16):
    """SpeculativeDecoder.generate (speculative.py:318-567): verify loop with
    accept / correct / bonus, cache rewind, draft re-alignment, adaptive chunk
    size, then single-step fallback.  Returns (emitted, stats)."""
    P = inputs_embeds.shape[1]
    first = int(dec.prefill(inputs_embeds))
    emitted = [first]
    stats = dict(accepted=0, verify_forwards=0, decode_steps=0)
    if emitted[-1] == eos or len(emitted) >= max_new_tokens:
        return emitted, stats
    cache_pos = P
    draft_pos = 0
    chunk_size = min_chunk
    SEARCH_WIN, STUCK_LIMIT = 40, 8
    stuck = 0
    n = len(draft)
    while draft_pos < n and len(emitted) < max_new_tokens:
        before = draft_pos
        k = min(chunk_size, n - draft_pos, max_new_tokens - len(emitted), dec.max_len - cache_pos - 1)
        if k <= 0:
            break
        chunk = draft[draft_pos:draft_pos + k]
        ids = torch.tensor([emitted[-1]] + chunk)
        logits = dec.verify(ids, cache_pos)
        stats["verify_forwards"] += 1
        preds_all = logits[: k + 1].argmax(dim=-1).tolist()
        preds, bonus = preds_all[:k], preds_all[k]
        j = 0
        mismatch = full = stopped = False
        while j < k and preds[j] == chunk[j]:
            emitted.append(chunk[j])
            stats["accepted"] += 1
            if chunk[j] == eos:
                j += 1
                stopped = True
                break
            j += 1
        if not stopped:
            if j < k:
                emitted.append(preds[j])
                mismatch = True
                stopped = preds[j] == eos
            else:
                full = True
                emitted.append(bonus)
                stopped = bonus == eos
        if full:
            cache_pos += k + 1
            draft_pos += k
        elif mismatch:
            cache_pos += j + 1
            draft_pos += j
        else:
            cache_pos += j
            draft_pos += j
        last_val = emitted[-1]
        realigned = False
        if not stopped and draft_pos < n:
            for dd in range(draft_pos, min(draft_pos + SEARCH_WIN, n)):
                if draft[dd] == last_val:
                    draft_pos = dd + 1
                    stats["accepted"] += 1
                    realigned = True
                    break
        stuck = 0 if draft_pos > before else stuck + 1
        if stuck >= STUCK_LIMIT and not stopped and draft_pos < n:
            draft_pos = before + 1
            stuck = 0
        if not stopped:
            if full:
                chunk_size = min(chunk_size + 4, max_chunk)
            elif mismatch and j == 0 and not realigned:
                chunk_size = boundary_chunk
            else:
                chunk_size = min_chunk
        if stopped or len(emitted) >= max_new_tokens:
            return emitted, stats
    while len(emitted) < max_new_tokens:
        valid = (torch.arange(dec.max_len) <= cache_pos).view(1, -1)
        dec.pos = cache_pos
        lg = dec.step(torch.tensor([emitted[-1]]), torch.tensor([cache_pos]), valid)
        stats["decode_steps"] += 1
        tid = int(lg[0].argmax())
        emitted.append(tid)
        cache_pos += 1
        if tid == eos:
            break
    return emitted, stats
