"""Torch-facing wrappers of the C ABI (one function per entry point).

Each wrapper checks dtypes/shapes/devices, passes raw pointers and the
current CUDA stream to ``libflashdllm_b200.so`` and raises on a non-zero
status.  Workspaces come from :class:`Workspace`, a per-device buffer that
grows on demand and is zero-filled when (re)allocated (the kernels leave
their counters at zero after every call).
"""
from __future__ import annotations

import functools
from typing import Dict, Optional, Tuple

import torch

from . import _lib
from ._lib import call, ptr

BF16 = torch.bfloat16


class Workspace:
    """Grow-only zero-initialised device scratch, one per (device, tag).

    Buffers that were outgrown stay allocated (in ``_retired``): a captured
    CUDA graph may still hold their addresses."""

    _bufs: Dict[Tuple[int, str], torch.Tensor] = {}
    _retired: list = []

    @classmethod
    def get(cls, device: torch.device, nbytes: int, tag: str = "main") -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
        buf = cls._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("workspace must be sized by an eager call before graph capture")
            size = max(nbytes, 1 << 20)
            if buf is not None:
                size = max(size, int(buf.numel() * 1.5))
                cls._retired.append(buf)
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            cls._bufs[key] = buf
        return buf

    @classmethod
    def clear(cls) -> None:
        cls._bufs.clear()
        cls._retired.clear()

    @classmethod
    def rezero(cls) -> None:
        """Zero every live buffer in place (after a device error left
        counters or flags set); addresses are kept."""
        for buf in cls._bufs.values():
            buf.zero_()


_lib.on_device_error(Workspace.rezero)


def set_qkv_plan(impl: int = -1, bn: int = 0, splits: int = 0, ksub: int = 0, pair: int = -1) -> None:
    """Override the QKV kernel's plan (tuning and tests): impl 0 is the
    stream-K GEMM, 1 the earlier whole-tile kernels with their bn / splits /
    ksub / pair knobs, -1 automatic; no arguments restore the automatic
    plan."""
    call("fdllm_qkv_set_plan", impl, bn, splits, ksub, pair)


def set_gemm_plan(bn: int = 0, ksub: int = 0, grid: int = 0, pair: int = -1, dp: int = 0) -> None:
    """Override the stream-K GEMM's tile width, ring stage depth, grid,
    CTA-pair mode and tile schedule (dp 1: one whole tile per CTA, 2: all
    tiles split stream-K; tuning and tests); no arguments restore the
    automatic plan."""
    call("fdllm_gemm_set_plan", bn, ksub, grid, pair, dp)


def linear(a: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16(a @ w.T (+ residual)) on the stream-K tcgen05 GEMM (fp32 sum,
    one rounding, as torch.addmm).  ``a`` may be a row-strided view."""
    if a.dim() != 2 or a.dtype != BF16 or not a.is_cuda or a.stride(1) != 1:
        raise ValueError("a must be a 2-D CUDA bf16 tensor with unit column stride")
    _check(w, "w", BF16, 2)
    n_rows, k = a.shape
    if w.shape[1] != k:
        raise ValueError(f"shapes {tuple(a.shape)} x {tuple(w.shape)}^T do not match")
    n = w.shape[0]
    if a.stride(0) != k and n_rows > 1:
        a = a.contiguous()
    if residual is not None:
        _check(residual, "residual", BF16, 2)
        if residual.shape != (n_rows, n):
            raise ValueError("residual must be [rows, n]")
    y = torch.empty(n_rows, n, dtype=BF16, device=a.device) if out is None else out
    nbytes = _lib.lib().fdllm_gemm_workspace_bytes(n_rows, n, k, 0)
    ws = Workspace.get(a.device, nbytes, "gemm")
    call("fdllm_gemm_bf16", ptr(a), ptr(w), ptr(y), ptr(residual), n_rows, n, k, y.stride(0),
         residual.stride(0) if residual is not None else 0, ptr(ws), ws.numel(), _stream())
    return y


def linear_swiglu(a: torch.Tensor, w_gate_up: torch.Tensor) -> torch.Tensor:
    """bf16(silu(a @ W_gate.T)) * (a @ W_up.T) with ``w_gate_up`` the
    [gate; up] stacked weight [2H, K]; one stream-K GEMM, gate/up never
    leave the tensor memory."""
    _check(a, "a", BF16, 2)
    _check(w_gate_up, "w_gate_up", BF16, 2)
    n_rows, k = a.shape
    if w_gate_up.shape[1] != k or w_gate_up.shape[0] % 2:
        raise ValueError("w_gate_up must be [2H, K]")
    h = w_gate_up.shape[0] // 2
    y = torch.empty(n_rows, h, dtype=BF16, device=a.device)
    nbytes = _lib.lib().fdllm_gemm_workspace_bytes(n_rows, 2 * h, k, 1)
    ws = Workspace.get(a.device, nbytes, "gemm")
    call("fdllm_gemm_swiglu", ptr(a), ptr(w_gate_up), ptr(y), n_rows, h, k, y.stride(0), ptr(ws), ws.numel(),
         _stream())
    return y


def _check(t: torch.Tensor, name: str, dtype=None, dim=None) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if dim is not None and t.dim() != dim:
        raise ValueError(f"{name} must be {dim}-D, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _stream_public() -> int:
    return torch.cuda.current_stream().cuda_stream


def _stream_raw() -> int:
    return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())


# torch's current stream on the current device (the capture stream while a
# CUDA graph is being captured).  The raw lookup avoids ~15 us of Python in
# torch.cuda.current_stream() per kernel call; a torch without it gets the
# public call.
_stream = _stream_raw if hasattr(torch._C, "_cuda_getCurrentRawStream") and hasattr(torch._C, "_cuda_getDevice") \
    else _stream_public


@functools.lru_cache(maxsize=None)
def _sm_count(index: int) -> int:
    return torch.cuda.get_device_properties(index).multi_processor_count


def auto_kv_splits(items: int, n_heads: int, max_keys: int, device: torch.device) -> int:
    """Key splits for the attention launch.  The kernel runs one CTA per SM
    with two work items per CTA; a split count S (1, 2 or 4) runs each pair
    of items on a cluster of S CTAs, one key slice each, merged in
    distributed shared memory.  Split only while the grid still fits one wave
    and every slice keeps at least two 64-key tiles.  Clusters of 8 are left
    to explicit requests: they measured 2-4 x slower than 4 (one sequence
    over 640-896 keys: 37.5 vs 14.4-15.7 us)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    sms = _sm_count(idx)
    ctas = max(1, (items + 1) // 2) * n_heads
    s = 1
    while s < 4 and 2 * s * ctas <= sms and max_keys // (2 * s) >= 128:
        s *= 2
    return s


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _check(x, "x", BF16, 2)
    _check(weight, "weight", BF16, 1)
    y = torch.empty_like(x) if out is None else out
    call("fdllm_rmsnorm", ptr(x), ptr(weight), ptr(y), x.shape[0], x.shape[1], float(eps), _stream())
    return y


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    """(y, h) = (x + residual, RMSNorm(x + residual)) in one pass."""
    _check(x, "x", BF16, 2)
    _check(residual, "residual", BF16, 2)
    _check(weight, "weight", BF16, 1)
    y = torch.empty_like(x)
    h = torch.empty_like(x)
    call("fdllm_add_rmsnorm", ptr(x), ptr(residual), ptr(weight), ptr(y), ptr(h), x.shape[0], x.shape[1],
         float(eps), _stream())
    return y, h


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """bf16(silu(gate)) * up for [rows, cols] tensors; gate/up may be the
    column halves of one stacked GEMM output (same row stride, unit column
    stride), read in place."""
    if gate.shape != up.shape or gate.dim() != 2:
        raise ValueError("gate and up must be 2-D of the same shape")
    for t, name in ((gate, "gate"), (up, "up")):
        if t.dtype != BF16 or not t.is_cuda or t.stride(1) != 1:
            raise ValueError(f"{name} must be a CUDA bf16 tensor with unit column stride")
    if gate.stride(0) != up.stride(0):
        raise ValueError("gate and up must share a row stride")
    out = torch.empty(gate.shape, dtype=BF16, device=gate.device)
    call("fdllm_swiglu", ptr(gate), ptr(up), ptr(out), gate.shape[0], gate.shape[1],
         gate.stride(0) if gate.shape[0] > 1 else gate.shape[1], _stream())
    return out


def _qkv(entry: str, xn, wq, wk, wv, pos, sin, cos, q_out, k_out, v_out, n_heads: int) -> None:
    for t, n in ((xn, "xn"), (wq, "wq"), (wk, "wk"), (wv, "wv"), (q_out, "q_out"), (k_out, "k_out"),
                 (v_out, "v_out")):
        _check(t, n, BF16, 2)
    _check(pos, "pos", torch.int64, 1)
    _check(sin, "rope_sin", torch.float32, 2)
    _check(cos, "rope_cos", torch.float32, 2)
    n_rows, d_model = xn.shape
    if pos.shape[0] < n_rows:
        raise ValueError("pos shorter than the query rows")
    # slots index the RoPE tables, and the cache rows when K/V are scattered
    n_slots = sin.shape[0] if entry == "fdllm_verify_qkv" else min(sin.shape[0], k_out.shape[0])
    nbytes = _lib.lib().fdllm_qkv_workspace_bytes(n_rows, d_model, n_heads)
    ws = Workspace.get(xn.device, nbytes, "qkv")
    call(entry, ptr(xn), ptr(wq), ptr(wk), ptr(wv), ptr(pos), ptr(sin), ptr(cos), ptr(q_out), ptr(k_out),
         ptr(v_out), n_rows, d_model, n_heads, n_slots, ptr(ws), ws.numel(), _stream())


def qkv_rope_cache(xn, wq, wk, wv, pos, sin, cos, q_out, k_cache, v_cache, n_heads: int) -> None:
    """Q -> ``q_out`` rows, RoPE'd K and V -> ``k_cache/v_cache[pos[r]]``."""
    _qkv("fdllm_qkv_rope_cache", xn, wq, wk, wv, pos, sin, cos, q_out, k_cache, v_cache, n_heads)


def verify_qkv(xn, wq, wk, wv, pos, sin, cos, q_out, k_out, v_out, n_heads: int) -> None:
    """Q, K, V of the verify rows, all row-indexed (no cache write)."""
    _qkv("fdllm_verify_qkv", xn, wq, wk, wv, pos, sin, cos, q_out, k_out, v_out, n_heads)


def _table(t: Optional[torch.Tensor], dtype) -> Tuple[Optional[torch.Tensor], int]:
    if t is None or t.numel() == 0:
        return None, 0
    if t.dtype != dtype:
        t = t.to(dtype)
    t = t.contiguous()
    if t.dim() != 2 or t.shape[1] != 4:
        raise ValueError(f"block table must be (n, 4), got {tuple(t.shape)}")
    return t, t.shape[0]


def plan_cache_attention(masked_blocks, tracked_blocks, n_rows: int, batch_size: int, block_m: int,
                         seqlen_max: int, device: torch.device) -> Tuple[torch.Tensor, int]:
    """Device work list for :func:`attn_cache`; returns (plan, capacity)."""
    mb, nm = _table(masked_blocks, torch.int64)
    tb, nt = _table(tracked_blocks, torch.int64)
    cap = _lib.lib().fdllm_attn_plan_capacity(n_rows, batch_size)
    nbytes = _lib.lib().fdllm_attn_plan_bytes(n_rows, batch_size)
    plan = torch.empty(nbytes // 4, dtype=torch.int32, device=device)
    call("fdllm_plan_cache_attention", ptr(mb), nm, ptr(tb), nt, n_rows, batch_size, block_m, seqlen_max,
         ptr(plan), nbytes, _stream())
    return plan, cap


def attn_cache(q, o, k_cache, v_cache, plan: torch.Tensor, capacity: int, attn_scores, score_scale: float,
               n_heads: int, seqlen_max: int, softmax_scale: float, kv_splits: int = 0,
               items_hint: int = 0, page_table: Optional[torch.Tensor] = None) -> None:
    """Masked + tracked attention over the cache, optional fused score
    accumulation.  ``items_hint`` estimates the plan's real item count (the
    capacity is an upper bound) for the automatic key split.  ``page_table``
    (int32 [batch, pages_per_seq]) maps key n of sequence b to cache row
    ``page_table[b, n // 64] * 64 + n % 64``; without it sequence b owns rows
    ``[b * seqlen_max, b * seqlen_max + k_end)``."""
    for t, n in ((q, "q"), (o, "o"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, n, BF16, 2)
    if attn_scores is not None:
        _check(attn_scores, "attn_scores", torch.float32)
    pps = 0
    if page_table is not None:
        _check(page_table, "page_table", torch.int32, 2)
        pps = page_table.shape[1]
    d_model = q.shape[1]
    if kv_splits <= 0:
        kv_splits = auto_kv_splits(items_hint if items_hint > 0 else capacity, n_heads, seqlen_max, q.device)
    ws, nws = None, 0
    if attn_scores is not None:
        nbytes = _lib.lib().fdllm_attn_workspace_bytes(capacity, n_heads, seqlen_max)
        ws = Workspace.get(q.device, nbytes, "attn")
        nws = ws.numel()
    call("fdllm_attn_cache", ptr(q), ptr(o), ptr(k_cache), ptr(v_cache), ptr(plan), capacity, ptr(attn_scores),
         float(score_scale), d_model, n_heads, seqlen_max, k_cache.shape[0], float(softmax_scale), kv_splits,
         ptr(page_table), pps, ptr(ws), nws, _stream())


def verify_attn(q1, k1, v1, o, k_cache, v_cache, pos_k, attn_mask, verify_blocks, block_rows: int, n_heads: int,
                softmax_scale: float, kv_splits: int = 0, max_keys: Optional[int] = None) -> None:
    """Flash-Verify attention (gathered cache keys + masked in-block keys)."""
    for t, n in ((q1, "q1"), (k1, "k1"), (v1, "v1"), (o, "o"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, n, BF16, 2)
    vb, nb = _table(verify_blocks, torch.int32)
    if nb == 0:
        return
    if pos_k is not None and pos_k.numel() > 0:
        pos_k = pos_k.to(torch.int64).contiguous()
        n_pos = pos_k.numel()
    else:
        pos_k, n_pos = None, 0
    mask = attn_mask.contiguous()
    if mask.dtype not in (torch.bool, torch.uint8):
        mask = mask.to(torch.bool)
    if mask.shape[0] < nb * block_rows or mask.shape[1] != block_rows:
        raise ValueError(f"attn_mask must be ({nb}*{block_rows}, {block_rows}), got {tuple(mask.shape)}")
    d_model = q1.shape[1]
    items = nb * ((block_rows + 63) // 64)
    if kv_splits <= 0:
        kv_splits = auto_kv_splits(items, n_heads, max_keys if max_keys is not None else n_pos // nb, q1.device)
    call("fdllm_verify_attn", ptr(q1), ptr(k1), ptr(v1), ptr(o), ptr(k_cache), ptr(v_cache), ptr(pos_k), n_pos,
         ptr(mask), ptr(vb), nb, block_rows, q1.shape[0], d_model, n_heads, k_cache.shape[0], float(softmax_scale),
         kv_splits, None, 0, _stream())


# ------------------------------------------------------------- decoding --

def row_stats(logits: torch.Tensor, tokens: Optional[torch.Tensor] = None):
    """fp64 softmax max-probability and first argmax of each logit row, and
    the probability of ``tokens[r]`` when given -> (p_max, argmax, p_tok)."""
    if logits.dim() != 2 or logits.dtype != BF16 or logits.stride(1) != 1:
        raise ValueError("logits must be a 2-D bf16 tensor with unit column stride")
    n, v = logits.shape
    dev = logits.device
    p = torch.empty(n, dtype=torch.float64, device=dev)
    am = torch.empty(n, dtype=torch.int64, device=dev)
    pt = None
    if tokens is not None:
        tokens = tokens.to(torch.int64).contiguous()
        pt = torch.empty(n, dtype=torch.float64, device=dev)
    call("fdllm_row_stats", ptr(logits), logits.stride(0), n, v, ptr(tokens), ptr(p), ptr(am), ptr(pt), _stream())
    return p, am, pt


def window_accept(p, tok, window, seq_info, eos_known, lmax: int, threshold: float, min_keep: int, eos_id: int,
                  full_pos, x, x_draft=None):
    """Batched confidence acceptance; ``seq_info`` int64 (B, 4) = (row offset,
    window length, flat full_pos index of num_decoded, predicted_length).
    Returns device (keep int32, length_num int32, eos_slot int64)."""
    b = seq_info.shape[0]
    dev = p.device
    keep = torch.empty(b, dtype=torch.int32, device=dev)
    length = torch.empty(b, dtype=torch.int32, device=dev)
    eos = torch.empty(b, dtype=torch.int64, device=dev)
    call("fdllm_window_accept", ptr(p), ptr(tok), ptr(window), ptr(seq_info), ptr(eos_known), b,
         full_pos.shape[0], lmax,
         float(threshold), int(min_keep), int(eos_id), ptr(full_pos), ptr(x), ptr(x_draft), ptr(keep), ptr(length),
         ptr(eos), _stream())
    return keep, length, eos


def verify_accept(p, draft_tok, draft_slot, seq_info, eos_known, gamma: float, eos_id: int, x):
    """Batched Flash-Verify acceptance scan -> device (keep int32, eos_slot int64)."""
    b = seq_info.shape[0]
    dev = seq_info.device
    keep = torch.empty(b, dtype=torch.int32, device=dev)
    eos = torch.empty(b, dtype=torch.int64, device=dev)
    call("fdllm_verify_accept", ptr(p), ptr(draft_tok), ptr(draft_slot), ptr(seq_info), ptr(eos_known), b,
         x.numel(), float(gamma), int(eos_id), ptr(x), ptr(keep), ptr(eos), _stream())
    return keep, eos


def cache_build(seq: torch.Tensor, n_rows: int, n_tiles: int, bm: int, full_pos: torch.Tensor, x: torch.Tensor,
                out=None):
    """Flash-Cache forward inputs from per-sequence scalars (``seq`` int64
    [n, 16], see fdllm_cache_build) -> device (block tables int64
    [n_tiles, 4], query slots, query tokens, window-acceptance rows [n, 4]);
    ``out`` = (tables, query slots, query tokens) to write into."""
    _check(seq, "seq", torch.int64, 2)
    _check(full_pos, "full_pos", torch.int64, 2)
    n, dev = seq.shape[0], seq.device
    i64 = dict(dtype=torch.int64, device=dev)
    if out is None:
        tables = torch.empty(n_tiles, 4, **i64)
        qpos, xq = torch.empty(n_rows, **i64), torch.empty(n_rows, **i64)
    else:
        tables, qpos, xq = out
        if tables.shape != (n_tiles, 4) or qpos.numel() != n_rows or xq.numel() != n_rows:
            raise ValueError("cache_build: output buffers of the wrong size")
    seq_info = torch.empty(n, 4, **i64)
    call("fdllm_cache_build", ptr(seq), n, bm, full_pos.shape[1], x.numel(), ptr(full_pos), ptr(x), ptr(tables),
         ptr(qpos), ptr(xq), ptr(seq_info), _stream())
    return tables, qpos, xq, seq_info


def verify_build(seq: torch.Tensor, n_keys: int, n_drafts: int, bm: int, full_pos: torch.Tensor, x: torch.Tensor,
                 x_draft: torch.Tensor, out=None):
    """Flash-Verify forward inputs from per-sequence scalars (``seq`` int64
    [n, 8], see fdllm_verify_build) -> device (qpos, x_verify, mask bool
    [n * 2bm, 2bm], key slots, draft slots, logit rows, verify blocks int32
    [n, 4], acceptance rows int64 [n, 4]); ``out`` = (qpos, x_verify, mask,
    key slots, logit rows, verify blocks) to write into."""
    _check(seq, "seq", torch.int64, 2)
    _check(full_pos, "full_pos", torch.int64, 2)
    n, dev, r = seq.shape[0], seq.device, 2 * bm
    i64 = dict(dtype=torch.int64, device=dev)
    dslot = torch.empty(n_drafts, **i64)
    if out is None:
        qpos, xv = torch.empty(n * r, **i64), torch.empty(n * r, **i64)
        mask = torch.empty(n * r, r, dtype=torch.bool, device=dev)
        kpos, lidx = torch.empty(n_keys, **i64), torch.empty(n_drafts, **i64)
        vblocks = torch.empty(n, 4, dtype=torch.int32, device=dev)
    else:
        qpos, xv, mask, kpos, lidx, vblocks = out
        if (qpos.numel() != n * r or xv.numel() != n * r or tuple(mask.shape) != (n * r, r) or kpos.numel() != n_keys
                or lidx.numel() != n_drafts or tuple(vblocks.shape) != (n, 4)):
            raise ValueError("verify_build: output buffers of the wrong size")
    info2 = torch.empty(n, 4, **i64)
    call("fdllm_verify_build", ptr(seq), n, bm, full_pos.shape[1], x.numel(), ptr(full_pos), ptr(x), ptr(x_draft),
         ptr(qpos), ptr(xv), ptr(mask), ptr(kpos), ptr(dslot), ptr(lidx), ptr(vblocks), ptr(info2), _stream())
    return qpos, xv, mask, kpos, dslot, lidx, vblocks, info2


def refresh_sort(full_pos: torch.Tensor, counts: torch.Tensor, scores: torch.Tensor) -> None:
    """In place: full_pos[j, :counts[j]] ordered by ascending score (stable)."""
    _check(full_pos, "full_pos", torch.int64, 2)
    _check(scores, "scores", torch.float32)
    counts = counts.to(torch.int64).contiguous()
    call("fdllm_refresh_sort", ptr(full_pos), full_pos.shape[0], full_pos.shape[1], ptr(counts), ptr(scores),
         scores.numel(), _stream())
