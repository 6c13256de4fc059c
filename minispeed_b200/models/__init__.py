"""Model zoo built on the sm_100a kernels: GPT-2 family and Llama-3 family."""

from .gpt import GPT, GPTConfig, gpt2_small, gpt2_xl, init_gpt2_

__all__ = ["GPT", "GPTConfig", "gpt2_small", "gpt2_xl", "init_gpt2_"]
