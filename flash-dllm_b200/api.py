"""Public API of flash_dllm_b200 (resolved lazily by the package shim)."""
from .ops import attn_cache, plan_cache_attention, qkv_rope_cache, rmsnorm, verify_attn, verify_qkv  # noqa: F401

__all__ = ["qkv_rope_cache", "verify_qkv", "rmsnorm", "plan_cache_attention", "attn_cache", "verify_attn"]
