"""GPU parity of the fused QKV + RoPE + cache-scatter kernel (tcgen05) and of
RMSNorm against the CPU oracle (reference kernel semantics, fp32 on
bf16-rounded inputs).  Tolerance: max |cuda - oracle| / max |oracle| <= 2e-2
(bf16 outputs; the bound stated for Q/K/V)."""
import pytest
import torch

from oracle import flash_cache_oracle as fco

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _rotary(n_slots, theta=500000.0, dim=128):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    f = torch.einsum("i,j->ij", torch.arange(n_slots, dtype=torch.float32), inv)
    p = torch.cat([f, f], -1)
    return p.sin(), p.cos()


def _case(n_rows, d_model, n_slots, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n_rows, d_model, generator=g).bfloat16()
    w = [(torch.randn(d_model, d_model, generator=g) * 0.02).bfloat16() for _ in range(3)]
    pos = torch.randperm(n_slots, generator=g)[:n_rows].to(torch.int64)
    kc = torch.randn(n_slots, d_model, generator=g).bfloat16()
    vc = torch.randn(n_slots, d_model, generator=g).bfloat16()
    sin, cos = _rotary(n_slots)
    return x, w, pos, kc, vc, sin, cos


def _oracle(x, w, pos, kc, vc, sin, cos, n_heads):
    q = torch.zeros(x.shape, dtype=torch.float32)
    k2, v2 = kc.float().clone(), vc.float().clone()
    bt = torch.tensor([[0, 0, 0, x.shape[0]]])
    fco.qkv_proj_cache(x.float(), q, k2, v2, pos, bt, w[0].float(), w[1].float(), w[2].float(), sin, cos,
                       n_heads, x.shape[0])
    return q, k2, v2


@pytest.mark.parametrize("n_rows,d_model,n_slots,plan", [
    (64, 4096, 512, {}),                                     # BASELINE config 1 shape
    (1, 256, 64, {}),
    (129, 256, 512, {}),
    (512, 4096, 1024, {}),
    (256, 4096, 1024, {}),
    (384, 4096, 2176, {}),                                   # BASELINE config 5 cache step (4 seqs x 96 rows)
    (64, 4096, 512, {"impl": 0}),                            # the stream-K GEMM at every row count
    (1, 256, 64, {"impl": 0}),
    (300, 512, 1024, {"impl": 0, "gemm": {"pair": 0, "bn": 256}}),
    (300, 512, 1024, {"impl": 0, "gemm": {"pair": 1, "ksub": 1}}),
    (64, 4096, 512, {"impl": 0, "gemm": {"bn": 256}}),
    (200, 1024, 512, {"impl": 0, "gemm": {"grid": 3}}),      # long ranges: several pieces, several tiles
    (64, 4096, 512, {"impl": 1, "splits": 3}),               # the earlier kernels: split-K
    (64, 4096, 512, {"impl": 1, "bn": 64, "splits": 1}),
    (59, 256, 256, {"impl": 1, "splits": 2}),
    (300, 512, 1024, {"impl": 1, "bn": 64}),
    (256, 4096, 1024, {"impl": 1}),                          # CTA-pair stream-K kernel (129-256 rows)
    (300, 512, 1024, {"impl": 1, "pair": 1}),                # ... forced: a half-empty 256-row block
    (512, 4096, 1024, {"impl": 1, "pair": 1}),               # ... forced: partial tiles, owner fix-ups
])
def test_qkv_rope_cache_matches_oracle(n_rows, d_model, n_slots, plan, qkv_plan):
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status
    plan = dict(plan)
    gemm = plan.pop("gemm", {})
    qkv_plan(**plan)
    ops.set_gemm_plan(**gemm)
    n_heads = d_model // 128
    x, w, pos, kc, vc, sin, cos = _case(n_rows, d_model, n_slots, seed=n_rows + d_model)
    dev = torch.device("cuda")
    q = torch.empty(n_rows, d_model, dtype=torch.bfloat16, device=dev)
    kd, vd = kc.to(dev), vc.to(dev)
    ops.qkv_rope_cache(x.to(dev), *(t.to(dev) for t in w), pos.to(dev), sin.to(dev), cos.to(dev), q, kd, vd,
                       n_heads)
    check_device_status()
    qo, ko, vo = _oracle(x, w, pos, kc, vc, sin, cos, n_heads)
    assert _rel(q, qo) <= TOL
    assert _rel(kd[pos.to(dev)], ko[pos]) <= TOL
    assert _rel(vd[pos.to(dev)], vo[pos]) <= TOL
    untouched = torch.ones(n_slots, dtype=torch.bool)
    untouched[pos] = False
    assert torch.equal(kd.cpu()[untouched], kc[untouched])
    assert torch.equal(vd.cpu()[untouched], vc[untouched])


@pytest.mark.parametrize("n_rows,d_model", [(64, 1024), (200, 1024), (512, 4096), (256, 4096), (64, 4096)])
def test_verify_qkv_matches_oracle(n_rows, d_model):
    """512 x 4096 is the config-4 verify forward on one GPU (8 sequences x 64
    rows), 256 the CTA-pair path (config 5), 64 one sequence per GPU."""
    import flash_dllm_b200.ops as ops
    n_slots = 512
    n_heads = d_model // 128
    x, w, pos, kc, vc, sin, cos = _case(n_rows, d_model, n_slots, seed=7 + n_rows)
    pos = torch.randint(0, n_slots, (n_rows,), generator=torch.Generator().manual_seed(3))  # repeats allowed
    dev = torch.device("cuda")
    q, k, v = (torch.empty(n_rows, d_model, dtype=torch.bfloat16, device=dev) for _ in range(3))
    ops.verify_qkv(x.to(dev), *(t.to(dev) for t in w), pos.to(dev), sin.to(dev), cos.to(dev), q, k, v, n_heads)
    q1, k1, v1 = (torch.zeros(n_rows, d_model) for _ in range(3))
    bt = torch.tensor([[0, 0, 0, n_rows]], dtype=torch.int32)
    fco.verify_qkv_proj(x.float(), q1, k1, v1, pos, w[0].float(), w[1].float(), w[2].float(), sin, cos, bt,
                        n_heads, n_rows)
    assert _rel(q, q1) <= TOL and _rel(k, k1) <= TOL and _rel(v, v1) <= TOL


def test_qkv_bad_slot_is_reported_not_written():
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import FdllmError, check_device_status
    d_model, n_slots, n_rows = 256, 64, 8
    x, w, pos, kc, vc, sin, cos = _case(n_rows, d_model, n_slots, seed=1)
    pos[3] = n_slots + 5  # out of range: the kernel skips the row and records the error
    dev = torch.device("cuda")
    q = torch.empty(n_rows, d_model, dtype=torch.bfloat16, device=dev)
    kd, vd = kc.to(dev), vc.to(dev)
    ops.qkv_rope_cache(x.to(dev), *(t.to(dev) for t in w), pos.to(dev), sin.to(dev), cos.to(dev), q, kd, vd, 2)
    with pytest.raises(FdllmError):
        check_device_status()
    check_device_status()  # cleared
    ok = torch.ones(n_rows, dtype=torch.bool)
    ok[3] = False
    _, ko, _ = _oracle(x[ok], w, pos[ok], kc, vc, sin, cos, 2)
    assert _rel(kd[pos[ok].to(dev)], ko[pos[ok]]) <= TOL


@pytest.mark.parametrize("rows,dim", [(1, 4096), (77, 4096), (5, 256)])
def test_rmsnorm_matches_reference_rounding(rows, dim):
    import flash_dllm_b200.ops as ops
    g = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, dim, generator=g) * 3).bfloat16()
    w = (1 + 0.1 * torch.randn(dim, generator=g)).bfloat16()
    y = ops.rmsnorm(x.cuda(), w.cuda(), 1e-5)
    ref = fco.rms_norm(x, w, 1e-5)
    # identical rounding points; the fp32 sum order differs, so allow ~1 bf16 ulp
    assert _rel(y, ref) <= 8e-3


def test_split_k_workspace_reuse_across_shapes(qkv_plan):
    """Split-K calls with different tile counts share one workspace: a call
    with few tiles must not leave partial sums where a later call with more
    tiles keeps its counters (all 96 head tiles of d_model 4096 checked)."""
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status
    qkv_plan(impl=1, splits=3)
    dev = torch.device("cuda")
    for n_rows, d_model, n_slots in ((64, 1024, 256), (64, 4096, 512), (200, 1024, 512), (64, 4096, 512)):
        n_heads = d_model // 128
        x, w, pos, kc, vc, sin, cos = _case(n_rows, d_model, n_slots, seed=n_rows * 7 + d_model)
        q = torch.empty(n_rows, d_model, dtype=torch.bfloat16, device=dev)
        kd, vd = kc.to(dev), vc.to(dev)
        ops.qkv_rope_cache(x.to(dev), *(t.to(dev) for t in w), pos.to(dev), sin.to(dev), cos.to(dev), q, kd, vd,
                           n_heads)
        check_device_status()
        qo, ko, vo = _oracle(x, w, pos, kc, vc, sin, cos, n_heads)
        assert _rel(q, qo) <= TOL and _rel(kd[pos.to(dev)], ko[pos]) <= TOL and _rel(vd[pos.to(dev)], vo[pos]) <= TOL
