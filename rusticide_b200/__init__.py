"""B200-native batched token sampler behind rusticide-sampling's API.

The product is librusticide_cuda.so (C ABI in include/rusticide_cuda.h); this
package is its Python host side: the ctypes binding, a mirror of the
reference's Sampler API, and the synthetic logit generator of the benchmark.
"""

from .sampler import (  # noqa: F401
    Engine,
    InvalidShape,
    NoValidTokens,
    Sampler,
    SamplingError,
    SamplingParams,
    TensorError,
    VocabOverflow,
    engine,
    extract_logits,
    row_error,
)

__all__ = [
    "Engine", "InvalidShape", "NoValidTokens", "Sampler", "SamplingError", "SamplingParams",
    "TensorError", "VocabOverflow", "engine", "extract_logits", "row_error",
]
