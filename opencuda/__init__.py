"""opencuda: a B200-native batch compiler for OpenCUDA's CUDA-C subset.

The data-parallel phases of the reference pipeline (garrick247/opencuda:
preprocess -> lex -> parse -> optimize -> emit) run as sm_100a kernels over
whole batches of translation units; ``include/ocb.h`` is the C ABI.

Drop-in surface: ``compile(src) -> ptx`` (the bytes of the reference CLI's
``--emit-ptx`` file), ``compile_batch(srcs, devices=...)`` and the CLI
``python -m opencuda X.cu --emit-ptx``.  The per-stage batch calls
(``lex_batch``, ``preprocess_batch``, ``parse_batch``, ``optimize_batch``)
live on ``Context`` and in ``opencuda.api``.
"""
from .api import (Context, OcbError, TokenBatch, TextBatch, context, lex_batch,  # noqa: F401
                  preprocess_batch, parse_batch, optimize_batch,
                  pack_sources, TU_OK, TU_RAISES, TU_UNSUPPORTED, TU_OVERFLOW,
                  TU_TIMEOUT)
from .compiler import (CompileError, Result, compile, compile_batch,  # noqa: F401,A004
                       resolve_includes, partition_lpt)

__version__ = "0.2.0"
