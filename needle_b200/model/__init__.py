"""needle_b200 model glue: config, Llama/Qwen2 decoders and ModelRunner
(mirrors of needle's ``needle/model`` package on the B200 attention path)."""
from .config import ModelConfig, preset
from .llama import LlamaForCausalLM
from .qwen2 import Qwen2ForCausalLM
from .runner import ModelRunner, build_model

__all__ = ["ModelConfig", "preset", "LlamaForCausalLM", "Qwen2ForCausalLM", "ModelRunner",
           "build_model"]
