"""Granite LLM constants used by the decode path.

Same values as the reference's src/starling/config.py:46-60 (Granite-4.0-1b
decoder of granite-speech-4.1-2b) and its token ids (config.py:67-71).  The
synthetic decode workloads use the same multipliers with intermediate 8192 and
vocabulary 100352.
"""

LLM_HIDDEN_SIZE: int = 2048
LLM_NUM_LAYERS: int = 40
LLM_NUM_ATTN_HEADS: int = 16
LLM_NUM_KV_HEADS: int = 4
LLM_HEAD_DIM: int = 128
LLM_INTERMEDIATE_SIZE: int = 4096
LLM_VOCAB_SIZE: int = 100353
LLM_ROPE_THETA: float = 10000.0
LLM_RMS_NORM_EPS: float = 1e-5
LLM_ATTENTION_MULTIPLIER: float = 0.0078125
LLM_EMBEDDING_MULTIPLIER: float = 12.0
LLM_RESIDUAL_MULTIPLIER: float = 0.22
LLM_LOGITS_SCALING: float = 8.0

LLM_PAD_TOKEN_ID: int = 100256
LLM_BOS_TOKEN_ID: int = 100257
LLM_EOS_TOKEN_ID: int = 100257

LLM_LOGIT_ATOL: float = 0.05
"""Absolute logit tolerance of the reference's fused path (config.py:80)."""

WEIGHT_FORMATS = ("bf16", "fp8", "int8", "nvfp4")
