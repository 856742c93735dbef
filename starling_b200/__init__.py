"""starling_b200: a B200 (sm_100a) native implementation of Starling's Granite
LLM greedy-decode hot path behind the reference's Python decode API.

    from starling_b200 import MultiStepLLMMega, BatchedLLMMega, SpeculativeDecoder

The CUDA work is in ``libstarling_b200.so`` (C ABI: include/starling_b200.h),
loaded with ctypes; there is no CPU fallback.
"""

from .config import LLM_EOS_TOKEN_ID, LLM_PAD_TOKEN_ID  # noqa: F401
from .flags import OptFlags, flags, get_default_flags, set_default_flags  # noqa: F401


def __getattr__(name):
    # Lazy so that importing the package (e.g. for the quantiser on CPU) does
    # not require the CUDA library.
    if name in ("LLMMega", "FusedLLMMega", "GenerateResult", "BenchReport"):
        from . import llm_mega

        return getattr(llm_mega, name)
    if name == "MultiStepLLMMega":
        from .multistep import MultiStepLLMMega

        return MultiStepLLMMega
    if name in ("BatchedLLMMega", "BatchedFusedLLMMega", "BatchedGenerateResult"):
        from . import batched

        return getattr(batched, name)
    if name in ("SpeculativeDecoder", "SpecResult"):
        from . import speculative

        return getattr(speculative, name)
    if name in ("GraniteEngine", "GraniteDims"):
        from . import engine

        return getattr(engine, name)
    raise AttributeError(name)
