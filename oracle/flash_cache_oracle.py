"""CPU restatement of the reference's fused Flash-Cache / Flash-Verify layer.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Everything here runs
in torch on the CPU.  Arithmetic is fp32; tensors that the reference keeps in
the model dtype (bf16 on the GPU) are rounded to that dtype at the same points
the reference stores them, so a bf16 call of this module reproduces the
reference's rounding points and an fp32 call reproduces its fp32 behaviour
(which is what ``TRITON_INTERPRET=1`` runs).

Reference file: ``llada/flash_cache_triton.py`` (VILA-Lab/Flash-dLLM).  Each
function cites the lines it restates.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch

NEG_INF = float("-inf")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float32)


def rope_rotate(acc: torch.Tensor, sin_rows: torch.Tensor, cos_rows: torch.Tensor) -> torch.Tensor:
    """Half-split rotary embedding on fp32 accumulators.

    ``rq1 = q1*cos1 - q2*sin1``, ``rq2 = q2*cos2 + q1*sin2`` where ``1``/``2``
    are the first/second 64 lanes of the 128-wide head
    (flash_cache_triton.py:84-93).  ``acc`` is (rows, heads, head_dim); the
    sin/cos rows are (rows, head_dim) fp32 and are shared by all heads.
    """
    half = acc.shape[-1] // 2
    a1, a2 = acc[..., :half], acc[..., half:]
    s = sin_rows[:, None, :]
    c = cos_rows[:, None, :]
    r1 = a1 * c[..., :half] - a2 * s[..., :half]
    r2 = a2 * c[..., half:] + a1 * s[..., half:]
    return torch.cat([r1, r2], dim=-1)


def _tile_rows(block_row: Sequence[int], block_m: int) -> range:
    """Rows one program instance covers: ``[q_s, q_s+BLOCK_M) & [.., q_e)``
    (flash_cache_triton.py:37-45, 124-131, 273-282)."""
    q_s, q_e = int(block_row[2]), int(block_row[3])
    return range(q_s, min(q_e, q_s + block_m))


def _project_rows(xn, wq, wk, wv, rows, pos, sin, cos, n_heads):
    """fp32 Q/K/V projection + RoPE of ``rows`` (flash_cache_triton.py:55-93)."""
    idx = torch.as_tensor(list(rows), dtype=torch.long)
    x = _f32(xn[idx])
    hd = x.shape[1] // n_heads
    q = (x @ _f32(wq).T).view(-1, n_heads, hd)
    k = (x @ _f32(wk).T).view(-1, n_heads, hd)
    v = (x @ _f32(wv).T).view(-1, n_heads, hd)
    p = pos[idx].to(torch.long)
    s_rows, c_rows = _f32(sin[p]), _f32(cos[p])
    rq = rope_rotate(q, s_rows, c_rows)
    rk = rope_rotate(k, s_rows, c_rows)
    return idx, p, rq.reshape(len(idx), -1), rk.reshape(len(idx), -1), v.reshape(len(idx), -1)


def qkv_proj_cache(xn, q_out, k_cache, v_cache, pos, block_table, wq, wk, wv, sin, cos,
                   n_heads: int, block_m: int) -> None:
    """K1 ``_flash_qkv_proj_cache_fwd`` (flash_cache_triton.py:15-100).

    For every block-table row ``(seq, k_end, q_s, q_e)`` and every head:
    Q/K/V of query rows ``[q_s, min(q_e, q_s+block_m))`` from the RMS-normed
    hidden states, RoPE on Q and K with the sin/cos row of the row's flat cache
    slot ``pos[r]``; Q is stored at query row ``r`` and K/V are scattered to
    cache row ``pos[r]``.  Outputs are rounded to the output tensors' dtype.
    """
    for row in block_table.tolist():
        rows = _tile_rows(row, block_m)
        if len(rows) == 0:
            continue
        idx, p, rq, rk, v = _project_rows(xn, wq, wk, wv, rows, pos, sin, cos, n_heads)
        q_out[idx] = rq.to(q_out.dtype)
        k_cache[p] = rk.to(k_cache.dtype)
        v_cache[p] = v.to(v_cache.dtype)


def verify_qkv_proj(xn, q1, k1, v1, pos, wq, wk, wv, sin, cos, block_table,
                    n_heads: int, block_m: int) -> None:
    """K4 ``_flash_verify_qkv_proj_fwd`` (flash_cache_triton.py:255-338).

    Same math as K1 for the verify rows (tile height ``2*block_length``) but
    Q, K and V all go to row-indexed scratch; the cache is not written.
    """
    for row in block_table.tolist():
        rows = _tile_rows(row, block_m)
        if len(rows) == 0:
            continue
        idx, _, rq, rk, v = _project_rows(xn, wq, wk, wv, rows, pos, sin, cos, n_heads)
        q1[idx] = rq.to(q1.dtype)
        k1[idx] = rk.to(k1.dtype)
        v1[idx] = v.to(v1.dtype)


class _Online:
    """Running (max, log-sum-exp, accumulator) exactly as the reference keeps
    it (flash_cache_triton.py:138-176): scale applied after the raw dot,
    natural ``exp``, P cast to the value dtype before the PV product."""

    def __init__(self, rows: int, heads: int, hd: int):
        self.m = torch.full((rows, heads), NEG_INF)
        self.lse = torch.full((rows, heads), NEG_INF)
        self.acc = torch.zeros(rows, heads, hd)

    def update(self, qk_scaled: torch.Tensor, v: torch.Tensor, p_dtype) -> None:
        # qk_scaled: (rows, heads, n); v: (n, heads, hd) fp32
        m_ij = torch.maximum(qk_scaled.max(dim=-1).values, self.m)
        p = torch.exp(qk_scaled - m_ij[..., None])
        l_ij = p.sum(dim=-1)
        self.acc = self.acc * torch.exp(self.m - m_ij)[..., None]
        p = p.to(p_dtype).to(torch.float32)
        self.acc = self.acc + torch.einsum("rhn,nhd->rhd", p, v)
        self.lse = m_ij + torch.log(torch.exp(self.lse - m_ij) + l_ij)
        self.m = m_ij

    def finish(self) -> torch.Tensor:
        return self.acc * torch.exp(self.m - self.lse)[..., None]


def cache_attention(q, o, k_cache, v_cache, block_table, seqlen_max: int, n_heads: int,
                    block_m: int, softmax_scale: float, block_n: int = 128,
                    S: Optional[torch.Tensor] = None) -> None:
    """K2 ``_flash_masked_attention_fwd`` (S given) and K3
    ``_flash_tracked_attention_fwd`` (S None) -- flash_cache_triton.py:103-252.

    Rows ``[q_s, min(q_e, q_s+block_m))`` of block row ``(seq, k_end, q_s,
    q_e)`` attend to cache rows ``[seq*seqlen_max, seq*seqlen_max + k_end)``
    in BLOCK_N tiles with the reference's online softmax.  When ``S`` is given
    (shape ``(block_m, heads, batch, seqlen_max)``) the raw, unscaled QK logit
    of every (row, head, key) is written to ``S[row - q_s, head, seq, key]``
    (flash_cache_triton.py:155-158).
    """
    hd = q.shape[1] // n_heads
    for row in block_table.tolist():
        b, k_end = int(row[0]), int(row[1])
        rows = _tile_rows(row, block_m)
        if len(rows) == 0:
            continue
        idx = torch.as_tensor(list(rows), dtype=torch.long)
        Q = _f32(q[idx]).view(-1, n_heads, hd)
        st = _Online(len(idx), n_heads, hd)
        base = b * seqlen_max
        for n0 in range(0, k_end, block_n):
            n1 = min(n0 + block_n, k_end)
            K = _f32(k_cache[base + n0: base + n1]).view(-1, n_heads, hd)
            V = _f32(v_cache[base + n0: base + n1]).view(-1, n_heads, hd)
            qk = torch.einsum("rhd,nhd->rhn", Q, K)
            if S is not None:
                S[0:len(idx), :, b, n0:n1] = qk
            st.update(qk * softmax_scale, V, v_cache.dtype)
        o[idx] = st.finish().reshape(len(idx), -1).to(o.dtype)


def pages_to_contiguous(cache: torch.Tensor, page_table: torch.Tensor, seqlen_max: int,
                        page: int = 64) -> torch.Tensor:
    """Gather a paged cache back into the reference's contiguous layout.

    Key ``n`` of sequence ``b`` lives at row ``page_table[b, n // page] * page
    + n % page`` of ``cache``; the result holds it at row ``b * seqlen_max +
    n``, which is where ``cache_attention`` (the reference kernels,
    ``start_n = batch_id * SEQLEN_MAX``, flash_cache_triton.py:122, 202) reads
    it.  The reference has no page table; this is the oracle of the paged
    variant."""
    B = page_table.shape[0]
    n = torch.arange(seqlen_max)
    rows = page_table.long()[:, n // page] * page + (n % page)[None, :]
    return cache[rows.reshape(-1)].reshape(B * seqlen_max, cache.shape[1])


def verify_attention(q1, k1, v1, o, k_cache, v_cache, pos_k, attn_mask, block_table,
                     n_heads: int, block_m: int, softmax_scale: float, block_n: int = 64) -> None:
    """K5 ``_flash_verify_attention_fwd`` (flash_cache_triton.py:341-428).

    Program ``pid`` handles verify block row ``(k_s, k_e, q_s, q_e)``: its
    ``block_m`` (= 2*block_length) rows attend to (a) cache rows gathered
    through ``pos_k[k_s:k_e]`` and (b) the block's own fresh K/V under the
    boolean mask ``attn_mask[pid*block_m:(pid+1)*block_m, :block_m]`` and the
    row-validity mask ``q_s + j < q_e``.  Part (b) reuses the running max of
    part (a) without re-stabilising (flash_cache_triton.py:416), exactly like
    the reference; with no cache keys that is ``exp(x - (-inf))`` and the
    reference yields non-finite rows.
    """
    hd = q1.shape[1] // n_heads
    for pid, row in enumerate(block_table.tolist()):
        k_s, k_e, q_s, q_e = (int(v) for v in row)
        nvalid = max(0, min(q_e - q_s, block_m))
        if nvalid == 0:
            continue
        idx_all = torch.arange(q_s, q_s + block_m)
        valid = idx_all < q_e

        def rows_of(t):
            out = torch.zeros(block_m, t.shape[1])
            out[:nvalid] = _f32(t[q_s:q_s + nvalid])
            return out.view(block_m, n_heads, hd)
        Q, K1, V1 = rows_of(q1), rows_of(k1), rows_of(v1)
        st = _Online(block_m, n_heads, hd)
        for n0 in range(k_s, k_e, block_n):
            n1 = min(n0 + block_n, k_e)
            sl = pos_k[n0:n1].to(torch.long)
            K = _f32(k_cache[sl]).view(-1, n_heads, hd)
            V = _f32(v_cache[sl]).view(-1, n_heads, hd)
            qk = torch.einsum("rhd,nhd->rhn", Q, K) * softmax_scale
            st.update(qk, V, v_cache.dtype)
        mask = attn_mask[pid * block_m:(pid + 1) * block_m, :block_m].to(torch.bool)
        qk1 = torch.einsum("rhd,nhd->rhn", Q, K1) * softmax_scale
        bias = torch.zeros(block_m, block_m)
        bias[:, ~valid] = NEG_INF
        bias[~mask] = NEG_INF
        qk1 = qk1 + bias[:, None, :]
        p1 = torch.exp(qk1 - st.m[..., None])
        l_ij = p1.sum(dim=-1)
        p1 = p1.to(v1.dtype).to(torch.float32)
        st.acc = st.acc + torch.einsum("rhn,nhd->rhd", p1, V1)
        st.lse = st.m + torch.log(torch.exp(st.lse - st.m) + l_ij)
        out = st.finish().reshape(block_m, -1)
        o[q_s:q_s + nvalid] = out[:nvalid].to(o.dtype)


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """``RMSLayerNorm.forward`` (llada/model/modeling_llada.py:389-403):
    fp32 normalise, cast back to the input dtype, then ``weight * x`` in that
    dtype."""
    og = x.dtype
    xf = _f32(x)
    var = xf.pow(2).mean(-1, keepdim=True)
    y = (xf * torch.rsqrt(var + eps)).to(og)
    if weight is not None:
        y = (_f32(weight) * _f32(y)).to(og)
    return y


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``nn.Linear`` without bias: fp32 accumulate, output in x's dtype."""
    return (_f32(x) @ _f32(w).T).to(x.dtype)


def flash_fused_elastic_cache(block, x: torch.Tensor, block_idx: int, positions: List, lengths: List,
                              softmax_scale: Optional[float] = None) -> torch.Tensor:
    """Layer driver ``flash_fused_elastic_cache`` (flash_cache_triton.py:462-638).

    ``block`` is any object with ``config.d_model``, ``config.n_heads``,
    ``attn_norm``/``ff_norm`` (callables), ``q_proj.weight``/``k_proj.weight``/
    ``v_proj.weight``/``attn_out``/``ff_proj``/``up_proj``/``ff_out``
    (weights) and the per-layer ``k_cache``/``v_cache`` -- the same attributes
    the reference reads from its ``LLaDALlamaBlock``.  ``positions`` and
    ``lengths`` are the reference's lists (generate.py:196-197, 299-300).
    """
    query_pos_flat, key_pos_flat, rotary_emb_pos, _info, attn_scores, attn_mask = positions
    (_start_layer, query_verify_blocks, query_masked_blocks, query_tracked_blocks, query_blocks,
     active_batch, _num_active, max_length, block_m, _block_n, _elastic, verify) = lengths
    d_model = block.config.d_model
    n_heads = block.config.n_heads
    head_dim = d_model // n_heads
    softmax_scale = softmax_scale or (1.0 / math.sqrt(head_dim))
    batch_size = len(active_batch)

    x_normed = block.attn_norm(x)
    att = torch.empty_like(x)
    q = torch.empty_like(x)
    sin, cos = rotary_emb_pos
    wq, wk, wv = block.q_proj.weight, block.k_proj.weight, block.v_proj.weight
    if verify:
        k1 = torch.empty_like(x)
        v1 = torch.empty_like(x)
        verify_qkv_proj(x_normed, q, k1, v1, query_pos_flat, wq, wk, wv, sin, cos,
                        query_verify_blocks, n_heads, 2 * block_m)
        verify_attention(q, k1, v1, att, block.k_cache, block.v_cache, key_pos_flat, attn_mask,
                         query_verify_blocks, n_heads, 2 * block_m, softmax_scale, block_n=64)
    else:
        S = torch.zeros((block_m, n_heads, batch_size, max_length), dtype=torch.float32)
        if query_blocks.shape[0] > 0:
            qkv_proj_cache(x_normed, q, block.k_cache, block.v_cache, query_pos_flat, query_blocks,
                           wq, wk, wv, sin, cos, n_heads, block_m)
        if query_masked_blocks.shape[0] > 0:
            cache_attention(q, att, block.k_cache, block.v_cache, query_masked_blocks, max_length,
                            n_heads, block_m, softmax_scale, 128, S)
        if query_tracked_blocks.shape[0] > 0:
            cache_attention(q, att, block.k_cache, block.v_cache, query_tracked_blocks, max_length,
                            n_heads, block_m, softmax_scale, 128, None)
        if block_idx > 1:
            attn_scores += S.mean((0, 1)).view(-1)

    att = linear(att, block.attn_out.weight)
    x = x + att
    og_x = x
    h = block.ff_norm(x)
    a, u = linear(h, block.ff_proj.weight), linear(h, block.up_proj.weight)
    a = torch.nn.functional.silu(a) * u
    a = linear(a, block.ff_out.weight)
    return (og_x + a).unsqueeze(0)
