from .llama import (
    PRESETS,
    Llama,
    LlamaConfig,
    flops_per_token,
    lm_loss,
    muon_and_adam_params,
    param_count,
    preset,
)

__all__ = [
    "PRESETS",
    "Llama",
    "LlamaConfig",
    "flops_per_token",
    "lm_loss",
    "muon_and_adam_params",
    "param_count",
    "preset",
]
