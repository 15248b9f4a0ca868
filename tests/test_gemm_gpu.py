"""GPU parity of the stream-K tcgen05 GEMM (fdllm_gemm_bf16, fdllm_gemm_swiglu)
against a plain torch fp32 reference of the same op on the same bf16 inputs:
out = bf16(a @ w.T (+ residual)) and the SwiGLU product with the reference's
bf16 rounding points (gate and up rounded, silu rounded, product rounded).
Tolerance: max |cuda - ref| / max |ref| <= 2e-2 (bf16 outputs); in practice
the difference is the fp32 summation order, about one bf16 ulp.  The GEMM
sums stream-K pieces in a fixed order, so results repeat bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


@pytest.fixture
def gemm_plan():
    from flash_dllm_b200 import ops
    yield ops.set_gemm_plan
    ops.set_gemm_plan()


def _ab(rows, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(rows, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    return a, w, g


@pytest.mark.parametrize("rows,n,k,plan", [
    (64, 4096, 4096, {}),               # attn_out, one sequence per GPU
    (64, 4096, 12288, {}),              # ff_out, one sequence per GPU (many pieces per tile)
    (20, 4096, 12288, {"ksub": 1}),     # M = 64 UMMAs with rows in two of the four TMEM lane quarters
    (49, 512, 1024, {"bn": 256}),       # ... a row quarter cut inside, 256-column tiles
    (512, 4096, 12288, {}),             # ff_out, eight sequences
    (512, 4096, 4096, {"pair": 0, "bn": 128}),  # single CTAs above 128 rows
    (256, 2048, 2048, {"ksub": 1}),            # CTA pairs, one 64-K box per stage
    (64, 1024, 512, {"pair": 1}),              # CTA pairs with the second CTA's rows all outside A
    (300, 1024, 512, {}),               # partial m-tile
    (1, 256, 64, {}),
    (130, 160, 256, {}),                # partial n-tile (160 = 128 + 32 columns)
    (200, 1024, 1024, {"grid": 7}),     # few CTAs: long ranges, pieces of several tiles
    (96, 2048, 2048, {"grid": 1}),      # one CTA: no pieces at all
    (300, 512, 256, {"grid": 2}),       # more m-tiles than CTAs: one group, m-tiles innermost
    (512, 4096, 4096, {"pair": 0, "dp": 1}),  # one whole tile per CTA (128 tiles)
    (512, 4096, 4096, {"dp": 1}),       # CTA pairs, one whole tile each
    (384, 4096, 4096, {}),              # short K, 96 tiles of 128: single CTAs, stream-K (no whole tiles)
    (448, 4096, 4096, {}),              # ... 128 tiles: one whole tile per CTA
    (100, 4096, 1024, {"grid": 30}),    # several contributors per tile, more than fit the ring
    (256, 2048, 2048, {"pair": 0, "bn": 256, "ksub": 1}),
    (64, 2048, 2048, {"bn": 256, "ksub": 2}),
    # CTA pairs, whole-tile waves after a stream-K region: owners whose
    # fix-up is not their last segment read the partials from the workspace
    (512, 12288, 4096, {}),             # QKV width, eight sequences: 22 split tiles + one wave of 74 pairs
    (512, 12288, 4096, {"dp": 2}),      # ... all tiles stream-K
    (200, 2048, 1024, {"grid": 3}),     # 2 split tiles over 3 pairs, then 2 waves
    (100, 2048, 1024, {"grid": 5, "pair": 0}),  # single CTAs (always all stream-K): 16 tiles over 5 CTAs
    (50, 2048, 1024, {"grid": 6, "ksub": 1}),   # ... M = 64 accumulators
])
@pytest.mark.parametrize("residual", [False, True])
def test_gemm_matches_torch(rows, n, k, plan, residual, gemm_plan):
    from flash_dllm_b200 import ops
    from flash_dllm_b200._lib import check_device_status
    gemm_plan(**plan)
    a, w, g = _ab(rows, n, k, rows + n + k)
    res = torch.randn(rows, n, device="cuda", generator=g).bfloat16() if residual else None
    y = ops.linear(a, w, res)
    check_device_status()
    ref = a.float() @ w.float().T
    if residual:
        ref = ref + res.float()
    assert _rel(y, ref.bfloat16()) <= TOL
    y2 = ops.linear(a, w, res)
    assert torch.equal(y, y2)  # fixed summation order


def test_gemm_strided_output_and_lm_head_width(gemm_plan):
    """Output written into a wider buffer (row stride > columns), and the
    LM-head width (126464 columns = 494 tiles of 256) on a few rows."""
    from flash_dllm_b200 import ops
    a, w, g = _ab(40, 512, 1024, 3)
    buf = torch.zeros(40, 768, device="cuda", dtype=torch.bfloat16)
    ops.linear(a, w, out=buf[:, 128:640])
    assert _rel(buf[:, 128:640], (a.float() @ w.float().T).bfloat16()) <= TOL
    assert not buf[:, :128].any() and not buf[:, 640:].any()
    a, w, _ = _ab(256, 126464, 4096, 4)
    y = ops.linear(a, w)
    ref = a[:64].float() @ w.float().T  # a row subset keeps the reference cheap
    assert _rel(y[:64], ref.bfloat16()) <= TOL


@pytest.mark.parametrize("rows,h,k,plan", [
    (64, 12288, 4096, {}),              # LLaDA-8B MLP, one sequence per GPU
    (512, 12288, 4096, {}),             # eight sequences
    (37, 512, 256, {"bn": 256}),
    (50, 2048, 1024, {"ksub": 1}),      # M = 64 UMMAs, several pieces per tile
    (200, 1024, 512, {"grid": 5}),
    (200, 1024, 512, {"pair": 0}),
    (64, 12288, 4096, {"dp": 2}),       # the explicit all-stream-K schedule on single CTAs
    (300, 2048, 1024, {"grid": 3}),     # pairs, two m-tiles: split tiles then waves
])
def test_gemm_swiglu_matches_torch(rows, h, k, plan, gemm_plan):
    from flash_dllm_b200 import ops
    from flash_dllm_b200._lib import check_device_status
    gemm_plan(**plan)
    g = torch.Generator(device="cuda").manual_seed(rows + h)
    a = torch.randn(rows, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * h, k, device="cuda", generator=g) * 0.05).bfloat16()
    y = ops.linear_swiglu(a, w)
    check_device_status()
    gate = (a.float() @ w[:h].float().T).bfloat16()
    up = (a.float() @ w[h:].float().T).bfloat16()
    ref = torch.nn.functional.silu(gate.float()).bfloat16().float() * up.float()
    assert _rel(y, ref) <= TOL
    assert torch.equal(y, ops.linear_swiglu(a, w))
