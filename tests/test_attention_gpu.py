"""GPU parity of the block-table attention (Flash-Cache, fused masked +
tracked rows with the attention-score accumulation) and of the Flash-Verify
attention against the CPU oracle (the reference kernels' semantics, bf16
inputs, P rounded to bf16 like the reference).  Outputs: max |cuda - oracle| /
max |oracle| <= 2e-2; accumulated scores: <= 1e-3 (fp32 sums of the same
bf16 products in a different order).  The scores must also be bit-identical
from one run to the next (order-independent fixed-point sums)."""
import numpy as np
import pytest
import torch

import cases
from oracle import decode_oracle as do
from oracle import flash_cache_oracle as fco

pytestmark = pytest.mark.gpu
TOL = 2e-2
SCORE_TOL = 1e-3


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _tiles(j, k_end, start, n, bm):
    return [(j, k_end, s, min(s + bm, start + n)) for s in range(start, start + n, bm)]


def _cache_inputs(k_ends, masked, tracked, d_model, lmax, bm, seed):
    g = torch.Generator().manual_seed(seed)
    B = len(k_ends)
    rows_m, rows_t, acc = [], [], 0
    for j in range(B):
        if masked[j]:
            rows_m += _tiles(j, k_ends[j], acc, masked[j], bm)
            acc += masked[j]
    for j in range(B):
        if tracked[j]:
            rows_t += _tiles(j, k_ends[j], acc, tracked[j], bm)
            acc += tracked[j]
    n_rows = acc
    q = torch.randn(n_rows, d_model, generator=g).bfloat16()
    kc = torch.randn(B * lmax, d_model, generator=g).bfloat16()
    vc = torch.randn(B * lmax, d_model, generator=g).bfloat16()
    mb = torch.tensor(rows_m, dtype=torch.int64).reshape(-1, 4)
    tb = torch.tensor(rows_t, dtype=torch.int64).reshape(-1, 4)
    return q, kc, vc, mb, tb, n_rows


def _run_cache(q, kc, vc, mb, tb, n_rows, lmax, bm, n_heads, B, kv_splits=0, scores=True, page_table=None,
               sc0=None):
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status
    dev = torch.device("cuda")
    scale = 1.0 / 128 ** 0.5
    qd, kd, vd = q.to(dev), kc.to(dev), vc.to(dev)
    o = torch.zeros_like(qd)
    sc = None
    if scores:
        sc = torch.zeros(B * lmax, dtype=torch.float32, device=dev) if sc0 is None else sc0.to(dev).clone()
    plan, cap = ops.plan_cache_attention(mb.to(dev), tb.to(dev), n_rows, B, bm, lmax, dev)
    pt = None if page_table is None else page_table.to(dev).to(torch.int32).contiguous()
    ops.attn_cache(qd, o, kd, vd, plan, cap, sc, 1.0 / (bm * n_heads), n_heads, lmax, scale, kv_splits,
                   page_table=pt)
    check_device_status()
    return o, sc


def _oracle_cache(q, kc, vc, mb, tb, lmax, bm, n_heads, B):
    scale = 1.0 / 128 ** 0.5
    o = torch.zeros(q.shape)
    S = torch.zeros((bm, n_heads, B, lmax))
    if mb.shape[0]:
        fco.cache_attention(q, o, kc, vc, mb, lmax, n_heads, bm, scale, 128, S)
    if tb.shape[0]:
        fco.cache_attention(q, o, kc, vc, tb, lmax, n_heads, bm, scale, 128, None)
    return o, S.mean((0, 1)).view(-1)


def test_cache_attention_golden_case():
    c = cases.cache_case()
    q = c["xn"].bfloat16()
    kc, vc = c["k_cache"].bfloat16(), c["v_cache"].bfloat16()
    o, sc = _run_cache(q, kc, vc, c["masked_blocks"], c["tracked_blocks"], q.shape[0], cases.LMAX,
                       cases.BLOCK_M, cases.N_HEADS, 2)
    oo, so = _oracle_cache(q, kc, vc, c["masked_blocks"], c["tracked_blocks"], cases.LMAX, cases.BLOCK_M,
                           cases.N_HEADS, 2)
    assert _rel(o, oo) <= TOL
    assert _rel(sc, so) <= SCORE_TOL


@pytest.mark.parametrize("kv_splits", [0, 1, 3, 8])  # 3 runs as 2 (cluster merge: 1, 2, 4, 8)
def test_cache_attention_config2_shape(kv_splits):
    """BASELINE config 2 shape: 8 sequences, k_end uniform in [256,1024] step
    32, 32 masked rows + 0..32 refresh rows each, 32 heads x 128."""
    rs = np.random.RandomState(5)
    B, bm, lmax, H = 8, 32, 1024, 32
    k_ends = [int(x) for x in rs.choice(np.arange(256, 1025, 32), B)]
    tracked = [int(x) for x in rs.randint(0, 33, B)]
    tracked[2] = 0
    q, kc, vc, mb, tb, n = _cache_inputs(k_ends, [bm] * B, tracked, H * 128, lmax, bm, seed=11)
    o, sc = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B, kv_splits)
    oo, so = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL
    assert _rel(sc, so) <= SCORE_TOL


def _config2(seed=5):
    """BASELINE config 2's generator: 8 sequences, k_end uniform over
    {256, 288, ..., 1024}, 32 masked rows + a refresh count uniform in
    [0, 32] per sequence, Q/K/V ~ N(0, 1), 32 heads x 128, and the block
    table's storage as a seeded permutation of 64-token pages."""
    rs = np.random.RandomState(seed)
    B, bm, lmax, H = 8, 32, 1024, 32
    k_ends = [int(x) for x in rs.choice(np.arange(256, 1025, 32), B)]
    tracked = [int(x) for x in rs.randint(0, 33, B)]
    pps = lmax // 64
    page_table = torch.from_numpy(rs.permutation(B * pps).reshape(B, pps).astype(np.int32))
    return B, bm, lmax, H, k_ends, tracked, page_table


@pytest.mark.parametrize("kv_splits", [0, 1, 4])
def test_cache_attention_config2_paged(kv_splits):
    """BASELINE config 2 as stated: the keys of every sequence sit in 64-token
    pages scattered by a seeded permutation; the oracle gathers the pages back
    to the reference's contiguous per-sequence regions."""
    B, bm, lmax, H, k_ends, tracked, pt = _config2()
    q, kc, vc, mb, tb, n = _cache_inputs(k_ends, [bm] * B, tracked, H * 128, lmax, bm, seed=12)
    # kc / vc are the physical paged storage (B * lmax rows = all pages)
    o, sc = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B, kv_splits, page_table=pt)
    kcc = fco.pages_to_contiguous(kc, pt, lmax)
    vcc = fco.pages_to_contiguous(vc, pt, lmax)
    oo, so = _oracle_cache(q, kcc, vcc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL
    assert _rel(sc, so) <= SCORE_TOL


def test_scores_are_reproducible():
    """The same forward three times and twice more with the keys split over a
    cluster gives bit-identical attn_scores: the column sums are added as
    integers (2^-32 fixed point), exact in any order, so neither the order in
    which CTAs finish nor the key split changes a score, and refresh decisions
    taken from them do not vary run to run.  Scores accumulate on top of
    earlier values, as across layers."""
    B, bm, lmax, H, k_ends, tracked, _ = _config2(seed=6)
    q, kc, vc, mb, tb, n = _cache_inputs(k_ends, [bm] * B, tracked, H * 128, lmax, bm, seed=13)
    sc0 = torch.randn(B * lmax, generator=torch.Generator().manual_seed(2))
    runs = [_run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B, ks, sc0=sc0) for ks in (1, 1, 1, 4, 4)]
    for o, sc in runs[1:3]:
        assert torch.equal(sc, runs[0][1])
        assert torch.equal(o, runs[0][0])
    assert torch.equal(runs[3][1], runs[0][1]) and torch.equal(runs[4][1], runs[0][1])
    oo, so = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(runs[0][1] - sc0.cuda(), so) <= SCORE_TOL


def test_out_of_range_scores_are_reported():
    """A masked-row column sum beyond the fixed-point range (|sum| >= 2^24;
    here queries scaled by 1e5) is reported as FDLLM_ERR_RANGE after the
    call, the output rows are still written, and the score workspace is
    zeroed again so the next call is exact."""
    from flash_dllm_b200._lib import FdllmError
    B, bm, lmax, H, k_ends, tracked, _ = _config2(seed=4)
    q, kc, vc, mb, tb, n = _cache_inputs(k_ends, [bm] * B, tracked, H * 128, lmax, bm, seed=15)
    with pytest.raises(FdllmError) as e:
        _run_cache((q.float() * 1e5).bfloat16(), kc, vc, mb, tb, n, lmax, bm, H, B, 1)
    assert e.value.code == 9
    o, sc = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B, 1)
    oo, so = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL and _rel(sc, so) <= SCORE_TOL


def test_cache_attention_config5_shape():
    """BASELINE config 5's first step on one GPU: 4 sequences of 1536 prompt
    + 512 generated tokens (2176-slot caches, reference rounding), 32 masked
    rows and ~2000 tracked rows each (every decoded and future slot is
    refreshed), with scores; 32 heads x 128."""
    B, bm, lmax, H = 4, 32, 2176, 32
    k_ends = [2176, 2176, 2048, 2176]
    tracked = [2000, 1984, 1900, 2016]
    q, kc, vc, mb, tb, n = _cache_inputs(k_ends, [bm] * B, tracked, H * 128, lmax, bm, seed=15)
    o, sc = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B)
    oo, so = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL
    assert _rel(sc, so) <= SCORE_TOL


def test_cache_attention_prefill_rows_and_no_scores():
    """Hundreds of tracked rows per sequence (the first decode step) -> several
    work items per sequence; the score output may be omitted."""
    B, bm, lmax, H = 2, 32, 768, 4
    q, kc, vc, mb, tb, n = _cache_inputs([768, 640], [bm, bm], [600, 300], H * 128, lmax, bm, seed=3)
    o, _ = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B, scores=False)
    oo, _ = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL


def test_cache_attention_block128_masked_spans_items():
    B, bm, lmax, H = 2, 128, 512, 2
    q, kc, vc, mb, tb, n = _cache_inputs([384, 512], [bm, 100], [200, 17], H * 128, lmax, bm, seed=4)
    o, sc = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B)
    oo, so = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL
    assert _rel(sc, so) <= SCORE_TOL


@pytest.mark.parametrize("kv_splits", [1, 2])
def test_cache_attention_growing_logits_and_nan_tail(kv_splits):
    """Key ranges that end inside a 64-key tile, logits that keep growing
    along the keys (the running max moves by far more than 2^8 several times),
    and NaN cache rows past every sequence's key range (never read as keys,
    zero-probability rows must not leak into the output)."""
    B, bm, lmax, H = 3, 32, 384, 2
    k_ends = [77, 200, 333]
    q, kc, vc, mb, tb, n = _cache_inputs(k_ends, [bm, bm, 20], [5, 40, 0], H * 128, lmax, bm, seed=8)
    grow = (1.0 + torch.arange(lmax, dtype=torch.float32) / 20.0).repeat(B)[:, None]
    kc = (kc.float() * grow).bfloat16()
    for j, ke in enumerate(k_ends):
        kc[j * lmax + ke:(j + 1) * lmax] = float("nan")
        vc[j * lmax + ke:(j + 1) * lmax] = float("nan")
    o, sc = _run_cache(q, kc, vc, mb, tb, n, lmax, bm, H, B, kv_splits)
    assert torch.isfinite(o).all()
    oo, so = _oracle_cache(q, kc, vc, mb, tb, lmax, bm, H, B)
    assert _rel(o, oo) <= TOL
    sc_valid = torch.cat([sc.cpu()[j * lmax:j * lmax + ke] for j, ke in enumerate(k_ends)])
    so_valid = torch.cat([so[j * lmax:j * lmax + ke] for j, ke in enumerate(k_ends)])
    assert _rel(sc_valid, so_valid) <= SCORE_TOL


def test_malformed_table_is_reported():
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import FdllmError, check_device_status
    dev = torch.device("cuda")
    mb = torch.tensor([[0, 999, 0, 16]], dtype=torch.int64, device=dev)  # k_end > seqlen_max
    plan, cap = ops.plan_cache_attention(mb, None, 16, 1, 16, 256, dev)
    with pytest.raises(FdllmError):
        check_device_status()
    assert int(plan[0]) == 0  # empty plan: the attention kernel does nothing


def _verify_inputs(s_list, n_keys, d_model, lmax, bm, seed):
    rs = np.random.RandomState(seed)
    g = torch.Generator().manual_seed(seed)
    bm2 = 2 * bm
    q_pos, k_pos, rows, masks = [], [], [], []
    acc_q = acc_k = 0
    for j, (s, nk) in enumerate(zip(s_list, n_keys)):
        perm = rs.permutation(lmax) + j * lmax
        t = bm2 - 2 * s
        q_pos.append(np.concatenate([perm[:t], perm[t:t + s], perm[t:t + s]]))
        k_pos.append(perm[t + s: t + s + nk])
        rows.append((acc_k, acc_k + nk, acc_q, acc_q + bm2))
        masks.append(do.verify_mask(bm, s))
        acc_q += bm2
        acc_k += nk
    B = len(s_list)
    n = acc_q
    return dict(
        q1=torch.randn(n, d_model, generator=g).bfloat16(), k1=torch.randn(n, d_model, generator=g).bfloat16(),
        v1=torch.randn(n, d_model, generator=g).bfloat16(),
        kc=torch.randn(B * lmax, d_model, generator=g).bfloat16(),
        vc=torch.randn(B * lmax, d_model, generator=g).bfloat16(),
        pos_k=torch.from_numpy(np.concatenate(k_pos).astype(np.int64)),
        blocks=torch.tensor(rows, dtype=torch.int32), mask=torch.cat(masks, 0))


def _check_verify(v, bm, H, kv_splits=0):
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status
    dev = torch.device("cuda")
    scale = 1.0 / 128 ** 0.5
    d = {k: t.to(dev) for k, t in v.items()}
    o = torch.zeros_like(d["q1"])
    ops.verify_attn(d["q1"], d["k1"], d["v1"], o, d["kc"], d["vc"], d["pos_k"], d["mask"], d["blocks"], 2 * bm, H,
                    scale, kv_splits)
    check_device_status()
    oo = torch.zeros(v["q1"].shape)
    fco.verify_attention(v["q1"], v["k1"], v["v1"], oo, v["kc"], v["vc"], v["pos_k"], v["mask"], v["blocks"], H,
                         2 * bm, scale, 64)
    assert _rel(o, oo) <= TOL


def test_verify_attention_golden_case():
    c = cases.verify_case()
    v = dict(q1=c["xn"].bfloat16(), k1=(c["xn"] * 0.5).bfloat16(), v1=(c["xn"] * -0.7).bfloat16(),
             kc=c["k_cache"].bfloat16(), vc=c["v_cache"].bfloat16(), pos_k=c["pos_k"], blocks=c["blocks"],
             mask=c["attn_mask"])
    _check_verify(v, cases.BLOCK_M, cases.N_HEADS)


@pytest.mark.parametrize("kv_splits", [0, 1, 4, 8])
def test_verify_attention_config4_shape(kv_splits):
    """bm 32 -> 64 verify rows per sequence, 8 sequences, 32 heads, ~830
    gathered cache keys each, varied draft counts S (0..16)."""
    rs = np.random.RandomState(9)
    s_list = [0, 16, 3, 8, 1, 16, 12, 5]
    n_keys = [int(896 - 64 + s + rs.randint(-20, 1)) - s for s in s_list]
    v = _verify_inputs(s_list, n_keys, 32 * 128, 896, 32, seed=21)
    _check_verify(v, 32, 32, kv_splits)


def _verify_inputs_generate_style(seqs, d_model, lmax, bm, seed):
    """Verify inputs laid out the way the decode loop builds them: for each
    sequence (nd decoded slots, s drafts, seqlen_k) the verify rows are the
    t = 2 bm - 2 s most recent decoded slots, the s draft slots and the same s
    slots again (mask views); the keys are the other decoded slots in their
    refresh order (score-sorted: a permutation, or still in slot order) and
    then the run of future slots [nd + s, seqlen_k).  Long runs of consecutive
    cache rows make most 64-key tiles load by TMA; the permuted prefixes are
    gathered."""
    rs = np.random.RandomState(seed)
    g = torch.Generator().manual_seed(seed)
    bm2 = 2 * bm
    q_pos, k_pos, rows, masks = [], [], [], []
    acc_q = acc_k = 0
    n_run_tiles = n_tiles = 0
    for j, (nd, s, seqlen_k, sorted_prefix) in enumerate(seqs):
        t = bm2 - 2 * s
        order = np.arange(nd) if sorted_prefix else rs.permutation(nd)  # full_pos[j, :nd]
        base = j * lmax
        q_slots = np.concatenate([order[nd - t:nd], np.arange(nd, nd + s), np.arange(nd, nd + s)]) + base
        keys = np.concatenate([order[:nd - t], np.arange(nd + s, seqlen_k)]) + base
        q_pos.append(q_slots)
        k_pos.append(keys)
        rows.append((acc_k, acc_k + len(keys), acc_q, acc_q + bm2))
        masks.append(do.verify_mask(bm, s))
        for k0 in range(0, len(keys), 64):
            tile = keys[k0:k0 + 64]
            n_tiles += 1
            n_run_tiles += int(len(tile) == 64 and np.all(np.diff(tile) == 1))
        acc_q += bm2
        acc_k += len(keys)
    B = len(seqs)
    n = acc_q
    v = dict(
        q1=torch.randn(n, d_model, generator=g).bfloat16(), k1=torch.randn(n, d_model, generator=g).bfloat16(),
        v1=torch.randn(n, d_model, generator=g).bfloat16(),
        kc=torch.randn(B * lmax, d_model, generator=g).bfloat16(),
        vc=torch.randn(B * lmax, d_model, generator=g).bfloat16(),
        pos_k=torch.from_numpy(np.concatenate(k_pos).astype(np.int64)),
        blocks=torch.tensor(rows, dtype=torch.int32), mask=torch.cat(masks, 0))
    return v, n_run_tiles, n_tiles


@pytest.mark.parametrize("kv_splits", [0, 1, 4, 8])
def test_verify_attention_config4_generate_layout(kv_splits):
    """Config 4 verify forward (8 sequences x 64 rows, 896-slot caches, 32
    heads) with the key lists the decode loop builds: most 64-key tiles are
    runs of consecutive cache rows (the TMA branch), the rest are gathered."""
    seqs = [(256, 16, 896, True), (300, 0, 896, True), (417, 3, 896, False), (512, 8, 896, True),
            (640, 16, 896, False), (288, 12, 896, True), (700, 1, 896, True), (830, 16, 896, False)]
    v, runs, tiles = _verify_inputs_generate_style(seqs, 32 * 128, 896, 32, seed=31)
    assert runs >= tiles // 2  # the layout exercises the TMA-run branch
    _check_verify(v, 32, 32, kv_splits)
