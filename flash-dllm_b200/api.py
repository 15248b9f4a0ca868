"""Public API of flash_dllm_b200 (resolved lazily by the package shim)."""
from .checkpoint import from_pretrained, load_model, load_tokenizer  # noqa: F401
from .flash_cache import flash_fused_elastic_cache, install_into_reference  # noqa: F401
from .generate import generate_with_Flash_dLLM, get_rotary_embedding, make_blocks  # noqa: F401
from .model import LLaDAConfigB200, LLaDAModelB200  # noqa: F401
from .ops import attn_cache, plan_cache_attention, qkv_rope_cache, rmsnorm, verify_attn, verify_qkv  # noqa: F401

__all__ = ["from_pretrained", "load_model", "load_tokenizer", "flash_fused_elastic_cache", "install_into_reference", "generate_with_Flash_dLLM", "get_rotary_embedding",
           "make_blocks", "LLaDAConfigB200", "LLaDAModelB200", "qkv_rope_cache", "verify_qkv", "rmsnorm",
           "plan_cache_attention", "attn_cache", "verify_attn"]
