"""The C-ABI library on the CPU (no GPU calls): it loads, exports every
function ``include/flashdllm_b200.h`` declares, the ctypes table mirrors the
header exactly, and the host-side queries and argument checks answer without
touching a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashdllm_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fdllm_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from flash_dllm_b200 import build
    if not os.path.exists(build.LIB):
        build.build()
    from flash_dllm_b200 import _lib
    return _lib


def test_header_declarations_are_exported(lib):
    names = _declared()
    assert len(names) >= 20
    raw = ctypes.CDLL(lib.LIB_PATH)
    for n in names:
        assert hasattr(raw, n), f"{n} declared in the header but not exported"


def test_ctypes_table_mirrors_the_header(lib):
    assert sorted(lib.SIGNATURES) == _declared()


def test_host_side_queries_and_checks(lib):
    L = lib.lib()
    assert b"sm_100a" in L.fdllm_version()
    assert L.fdllm_error_string(8).decode().startswith("request exceeds")
    assert L.fdllm_error_string(0) == b"ok"
    assert L.fdllm_attn_plan_capacity(512, 8) == 512 // 64 + 8
    assert L.fdllm_attn_plan_bytes(512, 8) >= 4 * (8 + 16 * 8 + 3 * 8)
    # scores workspace: a 64-bit accumulator row and a counter per sequence
    assert L.fdllm_attn_workspace_bytes(16, 32, 896) >= 16 * 896 * 8 + 16 * 4
    assert L.fdllm_error_string(9).decode().startswith("attention-score column sum out of range")
    # invalid arguments are refused before anything is launched
    assert L.fdllm_attn_cache(None, None, None, None, None, 1, None, 1.0, 4096, 0, 896, 7168, 0.1, 1, None, 0,
                              None, 0, None) == 1
    assert L.fdllm_qkv_rope_cache(None, None, None, None, None, None, None, None, None, None, 64, 4000, 32, 512,
                                  None, 0, None) == 1
    assert L.fdllm_qkv_set_plan(1, 96, 1, 0, -1) == 1  # tile width 96 is not a plan
    assert L.fdllm_qkv_set_plan(-1, 0, 0, 0, -1) == 0
    assert L.fdllm_gemm_set_plan(192, 0, 0, -1, 0) == 1
    assert L.fdllm_gemm_set_plan(0, 0, 0, -1, 0) == 0
    assert L.fdllm_gemm_bf16(None, None, None, None, 64, 100, 4096, 100, 0, None, 0, None) == 1  # 100 % 32 != 0
