"""Model zoo built on the sm_100a kernels: GPT-2 family and Llama-3 family."""

from .gpt import GPT, GPTConfig, gpt2_small, gpt2_xl, init_gpt2_
from .llama import Llama, LlamaConfig, init_llama_, llama3_8b

__all__ = ["GPT", "GPTConfig", "gpt2_small", "gpt2_xl", "init_gpt2_", "Llama", "LlamaConfig",
           "llama3_8b", "init_llama_"]
