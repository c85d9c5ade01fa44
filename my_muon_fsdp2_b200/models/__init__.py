from .encoder import SimpleTransformer, mlp_512_2048_512
from .gpt2 import GPT2LargeConfig, GPT2MediumConfig, GPT2SmallConfig, GPTConfig, GPTModel
from .llama import Llama, LlamaConfig, apply_fsdp

__all__ = ["Llama", "LlamaConfig", "apply_fsdp", "GPTModel", "GPTConfig", "GPT2SmallConfig", "GPT2MediumConfig",
           "GPT2LargeConfig", "SimpleTransformer", "mlp_512_2048_512"]
