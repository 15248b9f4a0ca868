"""GPU parity of the decode bookkeeping kernels against the oracle's decision
functions (restating llada/generate.py).  Integer decisions are compared
bit-exactly given identical probabilities / scores, including ties (the
oracle sorts stably, like the kernels); fp64 probabilities to 1e-12."""
import numpy as np
import pytest
import torch

from oracle import decode_oracle as do

pytestmark = pytest.mark.gpu


def test_row_stats_matches_fp64_softmax_with_ties():
    import flash_dllm_b200.ops as ops
    g = torch.Generator().manual_seed(0)
    R, V = 37, 126464
    logits = (torch.randn(R, V, generator=g) * 3).bfloat16()
    logits[0, 5] = logits[0, 77] = 40.0      # tie at the maximum: lowest id wins
    logits[1] = 0.0                          # all equal
    tok = torch.randint(0, V, (R,), generator=g)
    p, am, pt = ops.row_stats(logits.cuda(), tok.cuda())
    po, amo = do.confidence(logits)
    pto = do.token_prob(logits, tok)
    assert torch.equal(am.cpu(), amo)
    assert int(am[0]) == 5 and int(am[1]) == 0
    assert torch.allclose(p.cpu(), po, rtol=1e-12, atol=0)
    assert torch.allclose(pt.cpu(), pto, rtol=1e-12, atol=1e-300)


@pytest.mark.parametrize("vocab,pad,scale,shift", [
    (126464, 0, 3.0, 0.0),      # 16-byte loads, every logit through the bf16 exp table
    (1000, 0, 3.0, 0.0),        # vocabulary a multiple of 8, small
    (1001, 7, 3.0, 0.0),        # odd vocabulary and padded row stride: single-logit loads
    (4096, 0, 300.0, 0.0),      # maximum beyond 512: fp64 exp path for the whole row
    (4096, 0, 3.0, 600.0),      # ... at a large offset
    (4096, 0, -1.0, 0.0),       # table for most logits, fp64 exp for outliers at -700 and -inf
])
def test_row_stats_load_paths(vocab, pad, scale, shift):
    """Every load / exponential path of the row pass against the fp64
    softmax: vectorised and single-logit loads, the bf16 exp table and the
    fp64 exp for magnitudes above 512."""
    import flash_dllm_b200.ops as ops
    g = torch.Generator().manual_seed(vocab + pad)
    R = 19
    full = (torch.randn(R, vocab + pad, generator=g) * abs(scale) + shift).bfloat16()
    if scale < 0:
        full[:, ::97] = -700.0
        full[:, 5::211] = float("-inf")
    logits = full[:, :vocab]
    tok = torch.randint(0, vocab, (R,), generator=g)
    p, am, pt = ops.row_stats(full.cuda()[:, :vocab], tok.cuda())
    po, amo = do.confidence(logits.contiguous())
    pto = do.token_prob(logits.contiguous(), tok)
    assert torch.equal(am.cpu(), amo)
    assert torch.allclose(p.cpu(), po, rtol=1e-12, atol=0)
    assert torch.allclose(pt.cpu(), pto, rtol=1e-12, atol=1e-300)


def _accept_case(seed, B, bm, L):
    rs = np.random.RandomState(seed)
    rows, info, window, eos_known, lens = [], [], [], [], []
    off = 0
    for j in range(B):
        n = bm if j % 3 else max(1, bm - 5)   # some windows cut short
        nd = rs.randint(0, L - n)
        slots = j * L + nd + np.arange(n)
        # probabilities with repeated values (ties) and some above the threshold
        p = rs.choice([0.05, 0.5, 0.9, 0.95, 0.95, 0.2], n)
        pred = j * L + nd + rs.randint(0, n + 1)
        info.append((off, n, j * L + nd, pred))
        eos_known.append(j % 2)
        rows.append(p)
        window.append(slots)
        lens.append(n)
        off += n
    return (np.concatenate(rows), np.concatenate(window), np.array(info, np.int64), np.array(eos_known, np.int32),
            lens)


@pytest.mark.parametrize("min_keep,with_draft", [(1, False), (1, True), (2, False)])
def test_window_accept_matches_oracle(min_keep, with_draft):
    import flash_dllm_b200.ops as ops
    B, bm, L, eos_id, thr = 9, 32, 256, 7, 0.9
    p, window, info, eos_known, lens = _accept_case(3, B, bm, L)
    rs = np.random.RandomState(4)
    tok = rs.randint(0, 10, p.shape[0]).astype(np.int64)
    dev = torch.device("cuda")
    full_pos = torch.arange(B * L, device=dev).reshape(B, L)
    fp_ref = full_pos.cpu().clone()
    x = torch.full((B * L,), -1, dtype=torch.int64, device=dev)
    x_ref = x.cpu().clone()
    xd = torch.full((B * L,), -1, dtype=torch.int64, device=dev) if with_draft else None
    keep, length, eos = ops.window_accept(torch.from_numpy(p).to(dev), torch.from_numpy(tok).to(dev),
                                          torch.from_numpy(window).to(dev), torch.from_numpy(info).to(dev),
                                          torch.from_numpy(eos_known).to(dev), L, thr, min_keep, eos_id, full_pos,
                                          x, xd)
    for j in range(B):
        off, n, at, pred = (int(v) for v in info[j])
        pj = torch.from_numpy(p[off:off + n]).clone()
        slots = torch.from_numpy(window[off:off + n])
        tail = slots >= pred
        if eos_known[j]:
            pj[tail] = 0
        order = do.sort_desc_stable(pj)
        k = min(do.accept_count(pj, thr, min_keep), n)
        assert int(keep[j]) == k
        assert int(length[j]) == (n - int(tail.sum()) if eos_known[j] else n)
        nd = at % L
        fp_ref[j, nd:nd + n] = slots[order]
        x_ref[slots[order][:k]] = torch.from_numpy(tok[off:off + n])[order][:k]
        committed = slots[order][:k][torch.from_numpy(tok[off:off + n])[order][:k] == eos_id]
        assert int(eos[j]) == (int(committed.max()) if committed.numel() else -1)
    assert torch.equal(full_pos.cpu(), fp_ref)
    assert torch.equal(x.cpu(), x_ref)
    if with_draft:
        assert torch.equal(xd.cpu()[torch.from_numpy(window)], torch.from_numpy(tok))


def test_verify_accept_matches_oracle():
    import flash_dllm_b200.ops as ops
    rs = np.random.RandomState(8)
    B, gamma, eos_id = 10, 0.8, 3
    s_list = [0, 16, 5, 1, 16, 9, 2, 16, 7, 4]
    info, p, toks, slots = [], [], [], []
    off = 0
    for j, s in enumerate(s_list):
        pv = rs.choice([1.0, 0.99, 0.95, 0.9, 0.5], s)
        pred = 1000 * j + rs.randint(0, 20)
        info.append((off, s, 0, pred))
        p.append(pv)
        toks.append(rs.randint(0, 6, s))
        slots.append(1000 * j + np.arange(s) * 2)
        off += s
    eos_known = np.array([j % 2 for j in range(B)], np.int32)
    p, toks, slots = (np.concatenate(a) for a in (p, toks, slots))
    dev = torch.device("cuda")
    x = torch.full((10000,), -1, dtype=torch.int64, device=dev)
    keep, eos = ops.verify_accept(torch.from_numpy(p).to(dev), torch.from_numpy(toks).to(dev),
                                  torch.from_numpy(slots).to(dev), torch.from_numpy(np.array(info)).to(dev),
                                  torch.from_numpy(eos_known).to(dev), gamma, eos_id, x)
    xr = torch.full((10000,), -1, dtype=torch.int64)
    for j, s in enumerate(s_list):
        off, _, _, pred = info[j]
        pv = torch.from_numpy(p[off:off + s]).clone()
        sl = torch.from_numpy(slots[off:off + s])
        if eos_known[j]:
            pv[sl >= pred] = 0
        k = do.verify_keep(pv, gamma)
        assert int(keep[j]) == k, j
        tk = torch.from_numpy(toks[off:off + s])
        xr[sl[:k]] = tk[:k]
        e = sl[:k][tk[:k] == eos_id]
        assert int(eos[j]) == (int(e.max()) if e.numel() else -1)
    assert torch.equal(x.cpu(), xr)


@pytest.mark.parametrize("n_max", [40, 896, 2176])
def test_refresh_sort_matches_stable_oracle(n_max):
    import flash_dllm_b200.ops as ops
    rs = np.random.RandomState(n_max)
    B, L = 5, max(n_max, 64) + 64
    scores = rs.choice([-1.5, 0.0, -0.0, 0.25, 3.0], B * L).astype(np.float32)
    scores[::7] = rs.standard_normal(len(scores[::7]))
    full_pos = np.stack([j * L + rs.permutation(L) for j in range(B)]).astype(np.int64)
    counts = np.array([n_max, 0, 1, n_max // 2, rs.randint(2, n_max)], np.int64)
    dev = torch.device("cuda")
    fp = torch.from_numpy(full_pos).to(dev)
    ops.refresh_sort(fp, torch.from_numpy(counts).to(dev), torch.from_numpy(scores).to(dev))
    ref = torch.from_numpy(full_pos).clone()
    sc = torch.from_numpy(scores)
    for j in range(B):
        n = int(counts[j])
        head = ref[j, :n]
        ref[j, :n] = head[do.refresh_order(sc[head])]
    assert torch.equal(fp.cpu(), ref)


def _host_verify_build(act, s_a, nd_a, sk_a, pred_a, bm, L, full_pos, x, x_draft):
    """The Flash-Verify inputs built on the host with numpy, the way the
    decode loop built them before (a batched restatement of
    llada/generate.py:254-292): the reference for fdllm_verify_build."""
    from oracle.decode_oracle import verify_mask
    act, s_a, nd_a, sk_a, pred_a = (np.asarray(v, np.int64) for v in (act, s_a, nd_a, sk_a, pred_a))
    t_a = 2 * bm - 2 * s_a
    base = act * L + nd_a
    P = np.arange(2 * bm, dtype=np.int64)[None, :]
    T, S = t_a[:, None], s_a[:, None]
    qi = (base[:, None] + np.where(P < T + S, P - T, P - T - S)).reshape(-1)
    flags = ((P >= T) & (P < T + S)).reshape(-1)
    lidx = np.flatnonzero((P >= T + S).reshape(-1))
    lens = np.maximum(np.stack([nd_a - t_a, sk_a - nd_a - s_a], 1), 0)
    starts = np.stack([base - nd_a, base + s_a], 1)
    ki = np.concatenate([np.arange(a, a + n) for a, n in zip(starts.reshape(-1), lens.reshape(-1))]
                        + [np.zeros(0, np.int64)])
    nk = lens.sum(1)
    k_end = np.cumsum(nk)
    q0 = np.arange(len(act), dtype=np.int64) * 2 * bm
    vrows = np.stack([k_end - nk, k_end, q0, q0 + 2 * bm], 1).astype(np.int32)
    info2 = np.stack([np.cumsum(s_a) - s_a, s_a, np.zeros_like(s_a), pred_a], 1)
    flat = full_pos.reshape(-1)
    qpos = flat[qi]
    xv = np.where(flags, x_draft[qpos], x[qpos])
    mask = np.concatenate([np.asarray(verify_mask(bm, int(s)).numpy(), bool) for s in s_a])
    return qpos, xv, mask, flat[ki], flat[qi[flags]], lidx, vrows, info2


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_verify_build_matches_host_build(seed):
    """fdllm_verify_build against the host build on random decode states
    (active slot subsets, 0 .. bm/2 drafts, decoded counts near and far from
    the key range end, permuted slot orders): every output bit-exact."""
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status
    rng = np.random.default_rng(seed)
    B, L, bm = 8, 512, 32
    full_pos = np.stack([rng.permutation(L) + j * L for j in range(B)]).astype(np.int64)
    x = rng.integers(0, 126464, B * L).astype(np.int64)
    x_draft = rng.integers(0, 126464, B * L).astype(np.int64)
    act = sorted(rng.choice(B, size=int(rng.integers(1, B + 1)), replace=False).tolist())
    s_a = rng.integers(0, bm // 2 + 1, len(act))
    s_a[0] = 0
    sk_a = rng.choice([384, 448, 512], len(act))
    nd_a = np.array([int(rng.integers(2 * bm, sk - s)) for sk, s in zip(sk_a, s_a)])
    pred_a = rng.integers(256, L, len(act))
    ref = _host_verify_build(act, s_a, nd_a, sk_a, pred_a, bm, L, full_pos, x, x_draft)
    t_a = 2 * bm - 2 * s_a
    nk = np.maximum(nd_a - t_a, 0) + np.maximum(sk_a - nd_a - s_a, 0)
    seq = np.stack([np.asarray(act), s_a, nd_a, sk_a, pred_a, np.cumsum(nk) - nk, np.cumsum(s_a) - s_a,
                    np.zeros_like(s_a)], 1).astype(np.int64)
    dev = torch.device("cuda")
    got = ops.verify_build(torch.from_numpy(seq).to(dev), int(nk.sum()), int(s_a.sum()), bm,
                           torch.from_numpy(full_pos).to(dev), torch.from_numpy(x).to(dev),
                           torch.from_numpy(x_draft).to(dev))
    check_device_status()
    for name, r, g in zip(("qpos", "x_verify", "mask", "kpos", "draft_slots", "lidx", "vblocks", "info2"), ref, got):
        assert np.array_equal(g.cpu().numpy(), np.asarray(r)), name


def _host_cache_build(act, masked, tracked, seqlen_k, nd, pred, bm, L, full_pos, x):
    """The Flash-Cache inputs built on the host, the way the decode loop built
    them before (restating llada/generate.py:52-58, 146-163, 439-465): masked
    rows of all sequences first, then the tracked rows, in tiles of bm rows;
    the reference for fdllm_cache_build."""
    m_rows, t_rows, acc, m_lens = [], [], 0, []

    def tiles(rows, j, start, n):
        for s0 in range(start, start + n, bm):
            rows.append((j, seqlen_k[j], s0, min(s0 + bm, start + n)))

    for j in act:
        n = sum(max(0, b - a) for a, b in masked[j])
        m_lens.append(n)
        if n:
            tiles(m_rows, j, acc, n)
            acc += n
    r_m = acc
    for j in act:
        n = sum(max(0, b - a) for a, b in tracked[j])
        if n:
            tiles(t_rows, j, acc, n)
            acc += n
    idx = [j * L + p for rs in (masked, tracked) for j in act for a, b in rs[j] for p in range(a, b)]
    flat = full_pos.reshape(-1)
    qpos = flat[np.asarray(idx, np.int64)]
    info, off = [], 0
    for k, j in enumerate(act):
        info.append((off, m_lens[k], j * L + nd[j], pred[j]))
        off += m_lens[k]
    return (np.asarray(m_rows + t_rows, np.int64).reshape(-1, 4), qpos, x[qpos], np.asarray(info, np.int64), r_m,
            len(m_rows), len(t_rows))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_cache_build_matches_host_build(seed):
    """fdllm_cache_build against the host build on random decode states: a
    freshly loaded slot (tracked = the prompt and the tail, a prefill-sized
    row set), continuing slots (masked window, a tracked window on either
    side), empty ranges and finished slots; every output bit-exact."""
    import flash_dllm_b200.ops as ops
    from flash_dllm_b200._lib import check_device_status
    rng = np.random.default_rng(seed)
    B, L, bm = 8, 512, 32
    full_pos = np.stack([rng.permutation(L) + j * L for j in range(B)]).astype(np.int64)
    x = rng.integers(0, 126464, B * L).astype(np.int64)
    act = sorted(rng.choice(B, size=int(rng.integers(1, B + 1)), replace=False).tolist())
    masked, tracked, seqlen_k, nd, pred = {}, {}, {}, {}, {}
    for i, j in enumerate(act):
        sk = int(rng.choice([384, 448, 512]))
        seqlen_k[j], pred[j] = sk, int(rng.integers(256, L))
        if i == 0:  # just loaded: prompt p, masked window after it, tracked = the rest
            p = int(rng.integers(40, 200))
            nd[j], masked[j], tracked[j] = p, ((p, p + bm),), ((0, p), (p + bm, max(sk, p + bm)))
        else:
            d = int(rng.integers(bm, sk - bm))
            t0 = max(0, d - int(rng.integers(0, 3)) * bm)
            t1 = min(sk, d + bm * int(rng.integers(1, 3)))
            nd[j], masked[j] = d, ((d, min(d + bm, L)),)
            tracked[j] = ((t0, d), (min(d + bm, L), max(t1, min(d + bm, L))))
    ref_tab, ref_q, ref_x, ref_info, r_m, n_m, n_t = _host_cache_build(act, masked, tracked, seqlen_k, nd, pred, bm, L,
                                                                      full_pos, x)
    # the decode loop's per-sequence scalars (flash-dllm_b200/generate.py)
    seq = np.zeros((len(act), 16), np.int64)
    for k, j in enumerate(act):
        seq[k, 0:4] = (j, seqlen_k[j], nd[j], pred[j])
        rs = list(masked[j][:1]) + [(0, 0)] * (1 - len(masked[j][:1])) + list(tracked[j][:2]) \
            + [(0, 0)] * (2 - len(tracked[j][:2]))
        for c, (a, b) in zip((4, 6, 8), rs):
            seq[k, c:c + 2] = (a, max(0, b - a))
    m_n, t_n = seq[:, 5], seq[:, 7] + seq[:, 9]
    m_tl, t_tl = -(-m_n // bm), -(-t_n // bm)
    seq[:, 10] = np.cumsum(m_n) - m_n
    seq[:, 11] = m_n.sum() + np.cumsum(t_n) - t_n
    seq[:, 12] = np.cumsum(m_tl) - m_tl
    seq[:, 13] = m_tl.sum() + np.cumsum(t_tl) - t_tl
    assert (int(m_tl.sum()), int(t_tl.sum()), int(m_n.sum())) == (n_m, n_t, r_m)
    dev = torch.device("cuda")
    tab, qpos, xq, info = ops.cache_build(torch.from_numpy(seq).to(dev), int(m_n.sum() + t_n.sum()), n_m + n_t, bm,
                                          torch.from_numpy(full_pos).to(dev), torch.from_numpy(x).to(dev))
    check_device_status()
    assert np.array_equal(tab.cpu().numpy(), ref_tab)
    assert np.array_equal(qpos.cpu().numpy(), ref_q)
    assert np.array_equal(xq.cpu().numpy(), ref_x)
    assert np.array_equal(info.cpu().numpy(), ref_info)
