"""needle_b200: a B200 (sm_100a) attention hot path for the needle inference engine.

``needle_b200.ops`` wraps the C ABI of ``include/needle_b200.h`` (KV-cache
scatter, RoPE, paged split-K decode, prefill attention, fused residual +
RMSNorm); ``needle_b200.layers`` and ``needle_b200.model`` mirror needle's
``Attention`` / ``RMSNorm`` / ``RotaryEmbedding`` modules and its
``ModelRunner`` on top of those kernels.
"""
__version__ = "0.1.0"
