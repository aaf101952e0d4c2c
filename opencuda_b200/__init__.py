"""opencuda_b200: a B200-native batch compiler for OpenCUDA's CUDA-C subset.

The data-parallel phases of the reference pipeline (garrick247/opencuda:
preprocess -> lex -> parse -> optimize -> emit) run as sm_100a kernels over
whole batches of translation units; ``include/ocb.h`` is the C ABI.
"""
from .api import (Context, OcbError, TokenBatch, TextBatch, context, lex_batch,  # noqa: F401
                  preprocess_batch, parse_batch, optimize_batch, compile_batch,
                  pack_sources, TU_OK, TU_RAISES, TU_UNSUPPORTED, TU_OVERFLOW,
                  TU_TIMEOUT)

__version__ = "0.1.0"
