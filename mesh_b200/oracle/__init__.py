"""CPU fp32 oracle: a restatement of the reference host math, used as the correctness reference."""
from .tensor_ops import (  # noqa: F401
    matmul, silu, gelu, rms_norm, layer_norm, softmax, deterministic_sample_threshold,
    sample_token, sample_greedy, sample_tokens_device_semantics, embed_tokens, apply_rope,
)
from .forward import OracleWeights, LocalForwardPass  # noqa: F401
