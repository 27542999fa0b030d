"""modelc_b200 -- B200-native (sm_100a) speculative-decoding step for modelc.

The compute path is ``libmodelc_cuda.so`` (hand-written CUDA, C ABI in
``include/modelc_cuda.h``); this package is a thin host binding of it.
"""
from ._lib import McError, lib, last_error  # noqa: F401
from .generate import (KV_FP32, KV_INT8, KV_MIXED, CacheLookup, GenerationConfig,  # noqa: F401
                       KvSnapshot, LlamaDraftModel, MlpDraftModel, NgramDraftModel,
                       PrefixCache, Session, forward_llama_cached, sample_rows,
                       speculative_generate, tp_unique_id)
from .model import (LLAMA2_70B, LLAMA3_8B, PRESETS, TINY, TINYLLAMA,  # noqa: F401
                    LlamaConfig, Linear, QTensor, Weights, quantize_int8_rows,
                    quantize_int8_tensor, synth_weights, synth_weights_torch)

__version__ = "0.1.0"
