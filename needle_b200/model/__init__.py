"""needle_b200 model glue: config, Llama/Qwen2 decoder, ModelRunner."""
