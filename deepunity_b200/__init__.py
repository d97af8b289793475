"""deepunity_b200 -- B200 (sm_100a) implementation of DeepUnity's quantized llama
decode path behind a C ABI (libdeepunity_cuda.so, include/deepunity_cuda.h)."""
from ._lib import DUError, lib  # noqa: F401
from .llm import CONFIGS, KVQuant, LlamaConfig, LlamaForCausalLM, LLM, LLMQuant, LLMRegistry  # noqa: F401

__all__ = ["DUError", "lib", "CONFIGS", "KVQuant", "LlamaConfig", "LlamaForCausalLM", "LLM", "LLMQuant",
           "LLMRegistry"]
