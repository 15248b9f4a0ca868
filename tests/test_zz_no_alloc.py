"""The no-allocation QKV entry point (fdllm_qkv_rope_cache_noalloc).

Callers that cannot allocate device memory -- an embedding runtime whose
device memory belongs to another component, or a plugin that may not call
cudaMalloc once loaded -- use this variant: it takes its split-K scratch from
a fixed array inside the library instead of a caller workspace.  This test
calls it through the C ABI twice in a row and compares each result with the
regular entry point's, within the tolerance the other QKV tests use, and
checks that a request needing more scratch than the array holds is refused.
The array's counter / flag region is zeroed on entry of every call that uses
it, so calls of different kinds (split-K counters, CTA-pair handoff flags)
can follow one another on the same array; a mixed sequence checks that.
The file is collected last so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _inputs(n_rows, d_model, n_slots, seed):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    x = torch.randn(n_rows, d_model, generator=g).bfloat16().to(dev)
    w = [(torch.randn(d_model, d_model, generator=g) * 0.02).bfloat16().to(dev) for _ in range(3)]
    pos = torch.randperm(n_slots, generator=g)[:n_rows].to(dev)
    kc = torch.randn(n_slots, d_model, generator=g).bfloat16().to(dev)
    vc = torch.randn(n_slots, d_model, generator=g).bfloat16().to(dev)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    f = torch.einsum("i,j->ij", torch.arange(n_slots, dtype=torch.float32), inv)
    sin, cos = torch.cat([f, f], -1).sin().to(dev), torch.cat([f, f], -1).cos().to(dev)
    return x, w, pos, kc, vc, sin, cos


def _noalloc(lib, x, w, pos, sin, cos, q, kc, vc, n_heads):
    return lib.fdllm_qkv_rope_cache_noalloc(
        x.data_ptr(), w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(), pos.data_ptr(), sin.data_ptr(),
        cos.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), x.shape[0], x.shape[1], n_heads, kc.shape[0],
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("n_rows", [64, 256])
def test_noalloc_matches_workspace_entry_point_twice(n_rows, qkv_plan):
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status, lib
    qkv_plan(impl=0)  # the stream-K GEMM: its flags and per-CTA partial sums live in the array
    d_model, n_slots = 4096, 512
    n_heads = d_model // 128
    x, w, pos, kc0, vc0, sin, cos = _inputs(n_rows, d_model, n_slots, seed=11)
    q_ref = torch.empty_like(x)
    k_ref, v_ref = kc0.clone(), vc0.clone()
    ops.qkv_rope_cache(x, *w, pos, sin, cos, q_ref, k_ref, v_ref, n_heads)
    check_device_status()
    for it in range(2):  # the scratch keeps the last call's contents; a second call must still be right
        q = torch.empty_like(x)
        kc, vc = kc0.clone(), vc0.clone()
        assert _noalloc(lib(), x, w, pos, sin, cos, q, kc, vc, n_heads) == 0
        check_device_status()
        assert _rel(q, q_ref) <= TOL, (it, _rel(q, q_ref))
        assert _rel(kc[pos], k_ref[pos]) <= TOL
        assert _rel(vc[pos], v_ref[pos]) <= TOL


@pytest.mark.parametrize("impl", [0, 1])
def test_noalloc_mixed_calls_share_the_array(impl, qkv_plan):
    """Calls of different kinds on the one array, each compared with the
    workspace entry point: with the stream-K GEMM 64, 256 and 64 rows; with
    the earlier kernels a 64-row split-K call, a 256-row CTA-pair call and a
    64-row call again."""
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status, lib
    qkv_plan(impl=impl, splits=3 if impl else 0)
    d_model, n_slots = 4096, 512
    n_heads = d_model // 128
    for k, n_rows in enumerate((64, 256, 64)):
        x, w, pos, kc0, vc0, sin, cos = _inputs(n_rows, d_model, n_slots, seed=20 + k)
        q_ref = torch.empty_like(x)
        k_ref, v_ref = kc0.clone(), vc0.clone()
        ops.qkv_rope_cache(x, *w, pos, sin, cos, q_ref, k_ref, v_ref, n_heads)
        check_device_status()
        q = torch.empty_like(x)
        kc, vc = kc0.clone(), vc0.clone()
        assert _noalloc(lib(), x, w, pos, sin, cos, q, kc, vc, n_heads) == 0
        check_device_status()
        assert _rel(q, q_ref) <= TOL, (n_rows, _rel(q, q_ref))
        assert _rel(kc[pos], k_ref[pos]) <= TOL
        assert _rel(vc[pos], v_ref[pos]) <= TOL


def test_noalloc_refuses_requests_beyond_its_scratch(qkv_plan):
    from flash_dllm_b200._lib import lib
    qkv_plan(impl=1, splits=4, pair=0)  # the earlier single-CTA kernel, 256 rows x 4 K-splits: ~50 MB > 24 MiB
    x, w, pos, kc, vc, sin, cos = _inputs(256, 4096, 512, seed=12)
    q = torch.empty_like(x)
    k_before = kc.clone()
    assert _noalloc(lib(), x, w, pos, sin, cos, q, kc, vc, 32) == 8  # FDLLM_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert torch.equal(kc, k_before)  # nothing was launched
