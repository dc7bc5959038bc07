"""Deterministic vLLM inference via fixed-point reductions, B200-native.

Drop-in for the reference plugin ``fxpr_vllm``: ``register()``,
``quantization="fixed_point_det"``, ``attention_backend="CUSTOM"``, the
``fxpr::*`` torch.library ops and the ``VLLM_FXP_*`` knobs. Every reduction
runs in hand-written sm_100a CUDA kernels (``_lib/libfxpr_b200.so``).
"""
