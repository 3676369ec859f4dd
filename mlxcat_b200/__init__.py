"""mlxcat_b200 -- B200-native (sm_100a) n-gram speculative-decode path of mlxcat.

The compute lives in ``libmlxcat_cuda.so`` (CUDA kernels + C ABI, see
``include/mlxcat_cuda.h``); this package is the host-side mirror of the
reference's Swift surface over that ABI.  The library is loaded by the first
object that needs it (``Context``, ``lib()``) and that call fails loudly when
it is missing: there is no CPU fallback.  Importing the package (for the
model and workload descriptions alone) maps no native code.
"""
from . import _abi
from ._abi import MlxcatError, lib
from .engine import (
    CONFIGS, LLAMA3_8B, QWEN3_4B, TINY, BatchKVCache, ContinuousBatchGenerator, Context,
    FinishReason, ModelConfig, Request, Response, SamplingParameters, Scheduler,
    SpeculativeDecodingConfiguration, SpeculativeDecodingStats, allowed_next_token_ids, speculative_token_masks,
)

__all__ = [
    "BatchKVCache", "CONFIGS", "ContinuousBatchGenerator", "Context", "FinishReason", "LLAMA3_8B",
    "MlxcatError", "ModelConfig", "QWEN3_4B", "Request", "Response", "SamplingParameters",
    "Scheduler", "SpeculativeDecodingConfiguration", "SpeculativeDecodingStats", "TINY", "allowed_next_token_ids",
    "lib", "speculative_token_masks",
]
