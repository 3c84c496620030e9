"""Qwen2 on the B200 attention path (mirror of ``needle/model/qwen2.py``).

Identical to Llama except for biases on the q/k/v projections
(``needle/model/qwen2.py:12-39``).
"""
from __future__ import annotations

from .llama import LlamaDecoderLayer, LlamaForCausalLM, LlamaModel


class Qwen2DecoderLayer(LlamaDecoderLayer):
    qkv_bias = True


class Qwen2Model(LlamaModel):
    layer_cls = Qwen2DecoderLayer


class Qwen2ForCausalLM(LlamaForCausalLM):
    model_cls = Qwen2Model
