"""qora-llm_b200: B200 (sm_100a) decode engine behind QORA's Q4 SmolLM3-3B forward step.

The compute lives in libqora_cuda.so (hand-written CUDA, C ABI in include/qora_cuda.h);
this package is the host-side mirror of the reference's Rust interface
(`load_model`, `empty_kv_cache`, `forward_decode_raw`, `raw_prefill`, greedy argmax)
over that ABI (engine.py), plus the `.qora` format tools (qora_format.py). There is no
CPU fallback: every compute call goes through the CUDA library and fails loudly if it
cannot be loaded.
"""
from . import abi, qora_format  # noqa: F401
from . import engine  # noqa: F401
from .engine import (DecodeWeights, KVCache, QoraError, empty_kv_cache,  # noqa: F401
                     forward_decode_raw, load_model, raw_prefill)

__all__ = ["abi", "qora_format", "engine", "DecodeWeights", "KVCache", "QoraError",
           "load_model", "empty_kv_cache", "forward_decode_raw", "raw_prefill"]
