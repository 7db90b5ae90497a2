"""B200 (sm_100a) implementation of the fiber/ai EmbeddingGemma encoder hot path.

The compute lives in ``libfgemma.so`` (hand-written CUDA for sm_100a behind
the C ABI in ``include/fgemma.h``). This package holds its ctypes binding
(``_lib``), the host-side mirror of the reference's API — ``gemma`` for
``models/gemma`` (Load / Embed / embedBatch) and ``tensor`` for the tensor
operations the encoder calls — and the build step (``build``).
"""

__all__ = ["gemma", "tensor", "build"]
