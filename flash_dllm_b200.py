"""Import name of the package whose sources live in ``flash-dllm_b200/``.

A directory name with a hyphen is not importable, so this module makes
itself the package: it points ``__path__`` at that directory (so
``import flash_dllm_b200.generate`` etc. resolve there).  Public names are
resolved lazily from ``flash_dllm_b200.api`` so that ``flash_dllm_b200.build``
can run before the shared library exists.
"""
import importlib as _importlib
import os as _os

__path__ = [_os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "flash-dllm_b200")]

_PUBLIC = ("flash_fused_elastic_cache", "generate_with_Flash_dLLM", "get_rotary_embedding", "make_blocks",
           "LLaDAModelB200", "LLaDAConfigB200", "install_into_reference", "qkv_rope_cache", "verify_qkv",
           "rmsnorm", "attn_cache", "verify_attn", "plan_cache_attention", "from_pretrained", "load_model",
           "load_tokenizer")


def __getattr__(name):
    # Only public names resolve lazily; anything else (submodules such as
    # ``_lib``) must fall through to the regular submodule import.
    if name not in _PUBLIC:
        raise AttributeError(name)
    api = _importlib.import_module("flash_dllm_b200.api")
    return getattr(api, name)
