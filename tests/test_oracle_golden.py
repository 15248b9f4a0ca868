"""The CPU oracle reproduces the reference's own outputs (golden fixtures made
by ``tests/golden/make_golden.py`` from the reference kernels under Triton's
interpreter and the reference decode loop).  CPU only."""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import decode_oracle as do
from oracle import flash_cache_oracle as fco
from oracle import tiny_model as tm

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# fp32 vs fp32 with a different summation order: the reference kernels run
# in Triton's interpreter (numpy) and the oracle in torch.
TOL = 2e-5


def _load(name):
    return np.load(os.path.join(HERE, name))


def _close(a, b, tol=TOL):
    a = torch.as_tensor(np.asarray(a), dtype=torch.float32)
    b = torch.as_tensor(np.asarray(b), dtype=torch.float32)
    err = (a - b).abs().max().item()
    scale = max(b.abs().max().item(), 1e-6)
    assert err / scale <= tol, f"max abs err {err} (scale {scale})"


def _cache_run():
    c = cases.cache_case()
    H, bm = cases.N_HEADS, cases.BLOCK_M
    q = torch.zeros_like(c["xn"])
    kc, vc = c["k_cache"].clone(), c["v_cache"].clone()
    qb = torch.cat([c["masked_blocks"], c["tracked_blocks"]])
    fco.qkv_proj_cache(c["xn"], q, kc, vc, c["pos"], qb, c["wq"], c["wk"], c["wv"], c["sin"], c["cos"], H, bm)
    att = torch.zeros_like(c["xn"])
    S = torch.zeros((bm, H, 2, cases.LMAX))
    scale = 1.0 / cases.HEAD_DIM ** 0.5
    fco.cache_attention(q, att, kc, vc, c["masked_blocks"], cases.LMAX, H, bm, scale, 128, S)
    fco.cache_attention(q, att, kc, vc, c["tracked_blocks"], cases.LMAX, H, bm, scale, 128, None)
    return c, q, kc, vc, att, S


def test_qkv_rope_cache_matches_reference_kernel():
    g = _load("kernels_fp32.npz")
    c, q, kc, vc, _, _ = _cache_run()
    _close(q, g["q"])
    _close(kc[c["pos"]], g["k_rows"])
    _close(vc[c["pos"]], g["v_rows"])


def test_cache_attention_and_scores_match_reference_kernels():
    g = _load("kernels_fp32.npz")
    _, _, _, _, att, S = _cache_run()
    _close(att, g["att"])
    _close(S, g["S"])


def test_verify_kernels_match_reference():
    g = _load("kernels_fp32.npz")
    v = cases.verify_case()
    H, bm2 = cases.N_HEADS, 2 * cases.BLOCK_M
    q1, k1, v1, o = (torch.zeros_like(v["xn"]) for _ in range(4))
    fco.verify_qkv_proj(v["xn"], q1, k1, v1, v["pos"], v["wq"], v["wk"], v["wv"], v["sin"], v["cos"],
                        v["blocks"], H, bm2)
    fco.verify_attention(q1, k1, v1, o, v["k_cache"], v["v_cache"], v["pos_k"], v["attn_mask"], v["blocks"],
                         H, bm2, 1.0 / cases.HEAD_DIM ** 0.5, 64)
    _close(q1, g["vq1"])
    _close(k1, g["vk1"])
    _close(v1, g["vv1"])
    _close(o, g["vo"])


def _oracle_block():
    _, w = cases.gen_weights()
    m = tm.TinyLLaDA(tm.TinyConfig(**cases.GEN_CFG), w)
    return m.layers[2]


def test_layer_driver_matches_reference():
    g = _load("layer_fp32.npz")
    blk = _oracle_block()
    c = cases.cache_case()
    blk.k_cache, blk.v_cache = c["k_cache"].clone(), c["v_cache"].clone()
    scores = torch.zeros(2 * cases.LMAX)
    qb = torch.cat([c["masked_blocks"], c["tracked_blocks"]])
    positions = [c["pos"], torch.tensor([], dtype=torch.int32), [c["sin"], c["cos"]], [], scores, []]
    lengths = [[-1, -1], None, c["masked_blocks"], c["tracked_blocks"], qb, [0, 1], 2, cases.LMAX,
               cases.BLOCK_M, 128, None, False]
    y = fco.flash_fused_elastic_cache(blk, c["xn"], 2, positions, lengths).squeeze(0)
    _close(y, g["cache_out"])
    _close(scores, g["cache_scores"])
    _close(blk.k_cache[c["pos"]], g["cache_k_rows"])
    v = cases.verify_case()
    blk.k_cache, blk.v_cache = v["k_cache"].clone(), v["v_cache"].clone()
    positions = [v["pos"], v["pos_k"], [v["sin"], v["cos"]], [], torch.zeros(2 * cases.LMAX), v["attn_mask"]]
    lengths = [[-1, -1], v["blocks"], None, torch.tensor([], dtype=torch.int32), None, [0, 1], 2,
               cases.LMAX, cases.BLOCK_M, 128, None, True]
    y = fco.flash_fused_elastic_cache(blk, v["xn"], 2, positions, lengths).squeeze(0)
    _close(y, g["verify_out"])


def _unpack(g, prefix, key):
    lens = g[f"{prefix}_{key}_len"]
    flat = g[f"{prefix}_{key}"]
    out, o = [], 0
    for n in lens:
        out.append(flat[o:o + n])
        o += n
    return out


@pytest.mark.parametrize("verify", [False, True])
def test_decode_loop_matches_reference_trajectory(verify):
    """Every forward's query tokens and slots, the step counts and the
    decoded tokens of the oracle loop equal the reference loop's."""
    path = os.path.join(HERE, "generate_fp32.npz")
    tag = "verify" if verify else "cache"
    if not os.path.exists(path) or f"{tag}_x" not in np.load(path).files:
        pytest.skip("generate fixture not built")
    g = np.load(path)
    _, w = cases.gen_weights()
    assert abs(float(g["weights_checksum"]) - tm.weights_checksum(w)) < 1e-3 * float(g["weights_checksum"])
    model = tm.TinyLLaDA(tm.TinyConfig(**cases.GEN_CFG), w)
    rec = []

    def fwd(x_query, lengths, positions):
        v = bool(lengths[11])
        rec.append((v, x_query.reshape(-1).clone(), positions[0].reshape(-1).to(torch.long).clone(),
                    positions[1].reshape(-1).to(torch.long).clone() if v else torch.zeros(0, dtype=torch.long)))
        return model.forward(x_query, lengths, positions)

    prompts = cases.gen_prompts()
    n = len(prompts)
    responses, n_steps = [""] * n, [0] * n
    responses, num_tokens, max_num_tokens = do.generate(
        fwd, model.layers, model.cfg.n_layers, model.cfg.d_model, cases.HEAD_DIM, model.cfg.rope_theta,
        torch.float32, prompts, list(cases.GEN_PROMPT_LENS), cases.GEN_BATCH, responses, n_steps,
        verify=verify, gen_length=cases.GEN_LEN[verify], **cases.GEN_KW)
    xs, qs, ks = (_unpack(g, tag, k) for k in ("x", "qpos", "kpos"))
    assert len(rec) == len(xs)
    for i, (v, x, qp, kp) in enumerate(rec):
        assert v == bool(g[f"{tag}_verify"][i]), i
        np.testing.assert_array_equal(x.numpy(), xs[i], err_msg=f"forward {i} tokens")
        np.testing.assert_array_equal(qp.numpy(), qs[i], err_msg=f"forward {i} query slots")
        np.testing.assert_array_equal(kp.numpy(), ks[i], err_msg=f"forward {i} key slots")
    assert n_steps == g[f"{tag}_n_steps"].tolist()
    assert [num_tokens, max_num_tokens] == g[f"{tag}_num_tokens"].tolist()
    resp = np.concatenate([np.array([int(t) for t in r.split()], np.int64) for r in responses])
    np.testing.assert_array_equal(resp, g[f"{tag}_resp"])


def test_block_tables_and_rope_match_reference_helpers():
    """make_blocks / get_rotary_embedding restatements for a ragged case
    (generate.py:44-58)."""
    b = do.make_blocks(1, [10, 300], 40, 77, 16)
    assert b.tolist() == [[1, 300, 40, 56], [1, 300, 56, 72], [1, 300, 72, 77]]
    sin, cos = do.get_rotary_embedding(8, 128, 500000.0)
    s2, c2 = cases.rotary(8)
    assert torch.equal(sin, s2) and torch.equal(cos, c2)
    assert sin.shape == (8, 128) and torch.equal(sin[:, :64], sin[:, 64:])


def test_verify_mask_structure():
    m = do.verify_mask(4, 2)  # bm=4: T=4, S=2
    assert m.shape == (8, 8)
    assert not m[:4, 4:6].any() and m[:4, 6:].all()
    assert m[4:6, 4:6].tolist() == [[True, False], [True, True]]
    assert m[4:6, 6:8].tolist() == [[False, True], [False, False]]
    assert m[6:8, 4:6].tolist() == [[False, False], [True, False]]
    assert m[6:8, 6:8].tolist() == [[True, True], [False, True]]
    assert do.verify_mask(4, 0).all()
