"""Generate golden vectors by running the reference decoders on CPU.

Run where a checkout of the reference (sims1253/starling) is available,
with ``STARLING_REF`` naming its root directory:

    STARLING_REF=<reference checkout> python tests/golden/make_golden.py

It imports the reference's own ``LLMMega``, ``FusedLLMMega``,
``BatchedLLMMega`` and ``SpeculativeDecoder`` (src/starling/granite/*.py),
drives them eagerly on CPU (``capture=False``; ``torch.cuda.synchronize`` and
the CUDA-graph capture hooks stubbed out, ``FusedLLMMega``'s Triton glue
replaced by the torch ops it is bit-equal to, tests/test_llm_mega.py:145-170)
on a small random-init Granite model whose weights come from
``oracle.granite_ref.make_weights``, and saves the token ids and logits to
``tests/golden/*.pt``.  The files are small and committed; the reference
itself is not needed at test time.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
if not os.environ.get("STARLING_REF"):
    raise SystemExit("set STARLING_REF to the root of a reference checkout (it holds src/starling/)")
REF = Path(os.environ["STARLING_REF"]) / "src"
sys.path.insert(0, str(REF))

torch.cuda.synchronize = lambda *a, **k: None  # called unconditionally by the reference

from transformers import GraniteConfig, GraniteModel  # noqa: E402
from transformers.models.granite.modeling_granite import GraniteDecoderLayer  # noqa: E402
from transformers.cache_utils import StaticCache  # noqa: E402
from transformers.modeling_utils import local_torch_dtype  # noqa: E402

from starling.granite import llm_mega, batched, speculative  # noqa: E402

from oracle import granite_ref as gr  # noqa: E402

GOLDEN_STD = 0.2  # wide enough that greedy decoding does not collapse to one token
EOS = 100257


class _TorchGlue:
    """The torch ops the reference's Triton glue kernels equal bit-for-bit."""

    @staticmethod
    def fused_rmsnorm(x, w, eps):
        xf = x.float()
        var = xf.pow(2).mean(-1, keepdim=True)
        return w * (xf * torch.rsqrt(var + eps)).to(x.dtype)

    @staticmethod
    def fused_silu_mul(g, u):
        return torch.nn.functional.silu(g) * u

    @staticmethod
    def fused_residual_scale(x, y, a):
        return x + y * a


def hf_config(d: gr.Dims) -> GraniteConfig:
    cfg = GraniteConfig(
        hidden_size=d.hidden, intermediate_size=d.inter, num_hidden_layers=d.layers,
        num_attention_heads=d.n_q, num_key_value_heads=d.n_kv, head_dim=d.head_dim,
        vocab_size=d.vocab, rms_norm_eps=d.eps, rope_theta=d.theta,
        attention_multiplier=d.attn_mult, embedding_multiplier=d.emb_mult,
        residual_multiplier=d.res_mult, logits_scaling=d.logits_scaling,
        max_position_embeddings=4096, tie_word_embeddings=True,
    )
    cfg._attn_implementation = "eager"
    return cfg


def build_hf(d: gr.Dims, weights: dict):
    # Instantiate the way from_pretrained(torch_dtype=bf16) does: under a bf16
    # default dtype, so parameters are bf16 while the rotary inv_freq buffer,
    # computed with an explicit fp32 dtype, stays fp32.
    with local_torch_dtype(torch.bfloat16):
        lm = GraniteModel(hf_config(d)).eval()
    assert lm.rotary_emb.inv_freq.dtype == torch.float32
    missing, unexpected = lm.load_state_dict(weights, strict=False)
    assert not unexpected and all("rotary" in k for k in missing), (missing, unexpected)
    head = torch.nn.Linear(d.hidden, d.vocab, bias=False).to(torch.bfloat16)
    head.weight = lm.embed_tokens.weight  # tied
    return lm, head


def record_logits(dec):
    """Wrap ``_decode_step_eager`` to keep a copy of ``static_logits`` per step."""
    logs = []
    orig = dec._decode_step_eager

    def wrapped():
        orig()
        logs.append(dec.static_logits.reshape(-1, dec.static_logits.shape[-1]).clone())

    dec._decode_step_eager = wrapped
    return logs


def main():
    torch.set_grad_enabled(False)
    d = gr.TINY_DIMS
    weights = gr.make_weights(d, seed=0, std=GOLDEN_STD, norm_jitter=0.1)
    lm, head = build_hf(d, weights)
    gen = torch.Generator().manual_seed(1)
    T = 24
    emb = torch.randn(1, T, d.hidden, generator=gen).to(torch.bfloat16)
    max_len = 96
    n_new = 40

    # -- B=1: LLMMega (HF forward) and FusedLLMMega (fused loop) -------------
    dec = llm_mega.LLMMega(lm, head, max_cache_len=max_len, device="cpu")
    logs_hf = record_logits(dec)
    r_hf = dec.generate(emb, max_new_tokens=n_new, eos_token_id=EOS, capture=False)
    fdec = llm_mega.FusedLLMMega(lm, head, max_cache_len=max_len, device="cpu")
    fdec._k = _TorchGlue
    logs_f = record_logits(fdec)
    r_f = fdec.generate(emb, max_new_tokens=n_new, eos_token_id=EOS, capture=False)
    assert torch.equal(r_hf.ids, r_f.ids)
    # prefill logits (first token) via the reference's prefill
    pdec = llm_mega.LLMMega(lm, head, max_cache_len=max_len, device="cpu")
    T_ = emb.shape[1]
    pos_ids = torch.arange(T_).unsqueeze(0)
    out = pdec.lm(inputs_embeds=emb, position_ids=pos_ids, past_key_values=pdec.cache, use_cache=True)
    prefill_logits = (pdec.lm_head(out.last_hidden_state[:, -1:, :]) / 8.0).reshape(-1)

    b1 = dict(
        dims=d.__dict__, std=GOLDEN_STD, seed=0, norm_jitter=0.1,
        checksum=gr.weights_checksum(weights), inputs_embeds=emb, max_cache_len=max_len,
        max_new_tokens=n_new, ids=r_hf.ids[0], prefill_logits=prefill_logits,
        step_logits=torch.stack([x[0] for x in logs_f]),
    )
    torch.save(b1, HERE / "b1_greedy.pt")
    print("b1 ids", r_hf.ids[0].tolist())

    # -- batched with right padding (BatchedLLMMega, HF forward) -------------
    B = 3
    pl = torch.tensor([24, 17, 20])
    embB = torch.randn(B, T, d.hidden, generator=gen).to(torch.bfloat16)
    bdec = batched.BatchedLLMMega(lm, head, max_cache_len=max_len, max_batch_size=B, device="cpu")
    bdec.capture = lambda *a, **k: None  # keep _captured False -> eager step
    logs_b = record_logits(bdec)
    rb = bdec.generate(embB, prompt_lengths=pl, max_new_tokens=n_new, eos_token_id=EOS)
    bfd = batched.BatchedFusedLLMMega(lm, head, max_cache_len=max_len, max_batch_size=B, device="cpu")
    bfd._k = _TorchGlue
    bfd.capture = lambda *a, **k: None
    rbf = bfd.generate(embB, prompt_lengths=pl, max_new_tokens=n_new, eos_token_id=EOS)
    for a, b in zip(rb.ids_list, rbf.ids_list):
        assert torch.equal(a, b)
    torch.save(
        dict(inputs_embeds=embB, prompt_lengths=pl, max_cache_len=max_len, max_new_tokens=n_new,
             ids=[x.clone() for x in rb.ids_list], step_logits=torch.stack(logs_b[:4])),
        HERE / "batched_padded.pt",
    )
    print("batched ids", [x.tolist()[:12] for x in rb.ids_list])

    # -- speculative verify loop (SpeculativeDecoder, eager verify forward) ---
    greedy = r_hf.ids[0].tolist()
    draft = list(greedy[1:])
    # corrupt a few draft positions so accept / correct / re-align all run
    for i in (3, 4, 11, 20, 27):
        if i < len(draft):
            draft[i] = (draft[i] + 7) % d.vocab
    draft.insert(15, 5)
    sdec_llm = llm_mega.LLMMega(lm, head, max_cache_len=max_len, device="cpu")
    sdec_llm.capture = lambda *a, **k: None
    sd = speculative.SpeculativeDecoder(sdec_llm, lm.embed_tokens)
    rs = sd.generate(emb, draft, max_new_tokens=n_new, eos_token_id=EOS)
    torch.save(
        dict(inputs_embeds=emb, draft=draft, max_cache_len=max_len, max_new_tokens=n_new,
             ids=rs.ids[0], accepted=rs.accepted, verify_forwards=rs.verify_forwards,
             decode_steps=rs.decode_steps),
        HERE / "speculative.pt",
    )
    print("spec ids equal greedy:", rs.ids[0].tolist() == greedy, rs.accepted, rs.verify_forwards)

    # -- one Granite-1B-size decoder layer, 256 cached positions ----------------
    D = gr.GRANITE_1B_DIMS
    w, kc, vc, x, past = gr.layer_step_case(D, seed=0, past=256, std=0.02)
    cfg = hf_config(gr.Dims(**{**D.__dict__, "layers": 1}))
    with local_torch_dtype(torch.bfloat16):
        layer = GraniteDecoderLayer(cfg, 0).eval()
    layer.load_state_dict({k[len("layers.0."):]: v for k, v in w.items()})
    cache = StaticCache(config=cfg, max_cache_len=past + 1)
    # prime the static cache with the 256 past rows (lazy init via one update)
    cache.layers[0].lazy_initialization(kc[:, :, :1], vc[:, :, :1])
    cache.layers[0].keys.copy_(kc)
    cache.layers[0].values.copy_(vc)
    cache.layers[0].cumulative_length.fill_(past)
    from transformers.models.granite.modeling_granite import GraniteRotaryEmbedding
    with local_torch_dtype(torch.bfloat16):
        rot = GraniteRotaryEmbedding(cfg)
    pos = torch.tensor([[past]])
    cos, sin = rot(x, pos)
    mask = torch.zeros(1, 1, 1, past + 1, dtype=torch.bfloat16)
    y = layer(x, attention_mask=mask, position_ids=pos, past_key_values=cache, use_cache=True,
              position_embeddings=(cos, sin))
    torch.save(
        dict(seed=0, past=past, std=0.02, x=x, y=y.reshape(-1),
             k_new=cache.layers[0].keys[0, :, past].clone(), v_new=cache.layers[0].values[0, :, past].clone()),
        HERE / "layer_step.pt",
    )
    print("layer step y[:4]", y.reshape(-1)[:4])


if __name__ == "__main__":
    main()
