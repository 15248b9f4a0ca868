"""Seeded inputs shared by the golden-fixture generator and the tests.

Every input comes from ``numpy.random.RandomState`` (whose stream numpy keeps
stable across versions), so fixtures only need to store outputs.  Shapes are
small: d_model 256 = 2 heads x 128, block_length 16, two sequences.
"""
from __future__ import annotations

import numpy as np
import torch

D_MODEL = 256
N_HEADS = 2
HEAD_DIM = 128
BLOCK_M = 16
LMAX = 256
THETA = 500000.0


def rotary(seq_len: int, dim: int = HEAD_DIM, theta: float = THETA):
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    freqs = torch.einsum("i , j -> i j", torch.arange(seq_len, dtype=torch.float32), inv_freq)
    pos = torch.cat((freqs, freqs), dim=-1)
    return pos.sin(), pos.cos()


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype)


def cache_case(seed: int = 0):
    """Flash-Cache forward inputs: 2 sequences (k_end 200 and 180), 16 masked
    rows each, then 20 + 7 tracked rows (ragged last tiles).  Returns a dict
    of CPU tensors (fp32 activations, int64 tables/slots)."""
    rs = np.random.RandomState(seed)
    k_end = [200, 180]
    masked = [16, 16]
    tracked = [20, 7]
    pos = []
    slot_sets = []
    for j in range(2):
        slots = rs.permutation(k_end[j])[: masked[j] + tracked[j]] + j * LMAX
        slot_sets.append(slots)
    for j in range(2):
        pos.append(slot_sets[j][: masked[j]])
    for j in range(2):
        pos.append(slot_sets[j][masked[j]:])
    pos = np.concatenate(pos).astype(np.int64)
    nq = len(pos)
    rows_m, rows_t = [], []
    acc = 0
    for j in range(2):
        for s in range(0, masked[j], BLOCK_M):
            rows_m.append((j, k_end[j], acc + s, acc + min(s + BLOCK_M, masked[j])))
        acc += masked[j]
    for j in range(2):
        for s in range(0, tracked[j], BLOCK_M):
            rows_t.append((j, k_end[j], acc + s, acc + min(s + BLOCK_M, tracked[j])))
        acc += tracked[j]
    sin, cos = rotary(LMAX)
    return {
        "xn": _t(rs.standard_normal((nq, D_MODEL))),
        "wq": _t(rs.standard_normal((D_MODEL, D_MODEL)) * 0.05),
        "wk": _t(rs.standard_normal((D_MODEL, D_MODEL)) * 0.05),
        "wv": _t(rs.standard_normal((D_MODEL, D_MODEL)) * 0.05),
        "k_cache": _t(rs.standard_normal((2 * LMAX, D_MODEL))),
        "v_cache": _t(rs.standard_normal((2 * LMAX, D_MODEL))),
        "pos": torch.from_numpy(pos),
        "masked_blocks": torch.tensor(rows_m, dtype=torch.int64),
        "tracked_blocks": torch.tensor(rows_t, dtype=torch.int64),
        "sin": sin.repeat(2, 1),
        "cos": cos.repeat(2, 1),
        "k_end": k_end,
    }


def verify_case(seed: int = 1):
    """Flash-Verify inputs: 2 sequences of 2*16 rows; sequence 0 has S=6
    drafts (T=20), sequence 1 has S=0 (T=32).  Keys are gathered slot lists
    whose lengths (150, 97) are not multiples of the 64-key tile."""
    from oracle.decode_oracle import verify_mask  # local import: tests only
    rs = np.random.RandomState(seed)
    bm2 = 2 * BLOCK_M
    s_list = [6, 0]
    n_keys = [150, 97]
    q_pos, k_pos, rows, masks = [], [], [], []
    acc_q = acc_k = 0
    for j in range(2):
        perm = rs.permutation(LMAX)[: 200] + j * LMAX
        s = s_list[j]
        t = bm2 - 2 * s
        tracked = perm[:t]
        drafts = perm[t:t + s]
        q_pos.append(np.concatenate([tracked, drafts, drafts]))
        k_pos.append(perm[t + s: t + s + n_keys[j]])
        rows.append((acc_k, acc_k + n_keys[j], acc_q, acc_q + bm2))
        masks.append(verify_mask(BLOCK_M, s))
        acc_q += bm2
        acc_k += n_keys[j]
    sin, cos = rotary(LMAX)
    nq = acc_q
    return {
        "xn": _t(rs.standard_normal((nq, D_MODEL))),
        "wq": _t(rs.standard_normal((D_MODEL, D_MODEL)) * 0.05),
        "wk": _t(rs.standard_normal((D_MODEL, D_MODEL)) * 0.05),
        "wv": _t(rs.standard_normal((D_MODEL, D_MODEL)) * 0.05),
        "k_cache": _t(rs.standard_normal((2 * LMAX, D_MODEL))),
        "v_cache": _t(rs.standard_normal((2 * LMAX, D_MODEL))),
        "pos": torch.from_numpy(np.concatenate(q_pos).astype(np.int64)),
        "pos_k": torch.from_numpy(np.concatenate(k_pos).astype(np.int64)),
        "blocks": torch.tensor(rows, dtype=torch.int32),
        "attn_mask": torch.cat(masks, 0),
        "sin": sin.repeat(2, 1),
        "cos": cos.repeat(2, 1),
    }


# Tiny end-to-end decode setup (the reference generate_with_Flash_dLLM on a
# random-init 3-layer LLaDA); init_std 0.1 / head_std 0.5 give multi-token
# accepts, verify accepts and EOS events within a few dozen steps.
GEN_CFG = dict(d_model=256, n_heads=2, n_layers=3, mlp_hidden_size=512, vocab_size=512,
               rope_theta=THETA, rms_norm_eps=1e-5, init_std=0.1, head_std=0.5)
GEN_SEED = 0
GEN_EOS_SCALE = 1.5
GEN_KW = dict(block_length=16, mask_id=511, threshold=0.9, gamma=0.8, track_num=1, mask_num=2, eos_id=510)
# Per-mode generation length.  With verify=True the reference indexes a full
# ``block_length`` window (generate.py:215) and raises when the masked window
# is cut short by the end of the slot buffer; gen 96 keeps prompt+gen in
# [114, 128) so the buffer is 256 slots and the window never reaches its end
# (gen 32 hits that case).  verify=False handles short windows and keeps
# gen 32, whose run does reach the end of the buffer.
GEN_LEN = {False: 32, True: 96}
GEN_PROMPT_LENS = [20, 28, 24]
GEN_BATCH = 2


def gen_weights():
    from oracle import tiny_model as tm
    cfg = tm.TinyConfig(**GEN_CFG)
    w = tm.make_weights(cfg, GEN_SEED)
    w["model.transformer.ff_out.weight"][GEN_KW["eos_id"]] *= GEN_EOS_SCALE
    return cfg, w


def gen_prompts():
    rs = np.random.RandomState(1)
    return [torch.tensor(rs.randint(0, 500, size=L)) for L in GEN_PROMPT_LENS]
