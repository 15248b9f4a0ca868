"""Drop-in replacement of the reference's fused layer operator.

``flash_fused_elastic_cache(self, x, block_idx, positions, lengths,
softmax_scale=None)`` has the signature, argument meaning and side effects of
``llada/flash_cache_triton.py:462-638``: ``self`` is a LLaMA-style LLaDA
block (``config.d_model/n_heads``, ``attn_norm``, ``q_proj/k_proj/v_proj``,
``attn_out``, ``ff_norm``, ``ff_proj``, ``up_proj``, ``act``, ``ff_out``,
``dropout`` and the per-layer ``k_cache``/``v_cache`` set by the decode
driver); ``positions``/``lengths`` are the driver's lists; the caches and
``attn_scores`` are updated in place; the return value is the block output
``(1, Nq, d_model)``.

The attention half runs on this package's sm_100a kernels: RMSNorm, the
tcgen05 QKV + RoPE + cache-scatter GEMM (or its verify variant), and one
fused masked + tracked attention pass (or the verify attention).  The
reference's ``S`` tensor and ``attn_scores += S.mean((0, 1))`` become an
in-kernel accumulation.  After attention the projections can run on the
package's stream-K tcgen05 GEMM with fused epilogues: ``attn_out`` with the
residual add, ``ff_proj``/``up_proj`` as one GEMM over the stacked
``ffup_weight`` whose epilogue forms bf16(silu(gate)) * up (the gate and up
activations never reach HBM), and ``ff_out`` with the residual add.
Each projection runs on the GEMM that measured faster at its row count
(``use_own``): this package's for the stacked MLP projection up to 256
rows; cuBLAS (``addmm``, residual in its epilogue too) for
``attn_out``, ``ff_out``, the LM head and the MLP above 256 rows: in the
full decode step those measured faster (this package's kernels are faster
alone at several of those shapes).  The
environment variable ``FDLLM_OWN_GEMMS`` (a comma list of ``attn_out``,
``mlp``, ``ff_out``, ``lm_head``, ``all`` or ``none``) forces the choice for
comparisons (``lm_head``: the model's LM head, in ``model.py``).
"""
from __future__ import annotations

import math
import os

import torch

from . import ops


def _own_gemms():
    v = os.environ.get("FDLLM_OWN_GEMMS")
    names = ("attn_out", "mlp", "ff_out", "lm_head")
    if v is None:
        return None
    on = {x.strip() for x in v.split(",")}
    return {n: (n in on or "all" in on) for n in names}


OWN_GEMMS = _own_gemms()

# Rows up to which this package's GEMM is used, per projection, chosen by
# alternating full-step runs on one B200 (generated tokens/s; kernel timings
# taken alone ranked several of these the other way: back-to-back launches
# of one of this package's kernels overlap each launch's prologue and first
# weight loads with the tail of the one before, which the step's neighbours
# do not allow, and the config-4 step runs at the power cap).  Config 4
# (512-row forwards): cuBLAS for attn_out, the MLP projection and the LM head
# 449.4 / 448.7 vs 439.1 / 439.0 with this package's attn_out (kernel alone
# 24.6 vs 25.5 us) and MLP + SwiGLU (84.7 vs 77.1 + 10.3 us); config 3
# (64-row forwards): cuBLAS attn_out and ff_out with this package's MLP
# 227.2 / 227.3 vs 217.1 / 221.3 with this package's ff_out and 208.3 / 211.6
# with its attn_out too (alone 16.0 vs 25.2 us), while the MLP on cuBLAS
# lost 4.5 % (205.3 vs 214.8); config 5 (384 / 256 rows): cuBLAS attn_out
# 246.7 / 246.2 vs 240.0 / 241.5, the MLP even.  The QKV projection has no
# cuBLAS counterpart (RoPE and the cache scatter are in its epilogue).
_OWN_UP_TO = {"attn_out": 0, "mlp": 256, "ff_out": 0, "lm_head": 0}


def _own_up_to_env() -> None:
    """``FDLLM_OWN_UP_TO`` (e.g. ``mlp:128,attn_out:0``) overrides row
    thresholds of the table above (tuning runs)."""
    v = os.environ.get("FDLLM_OWN_UP_TO")
    if not v:
        return
    for item in v.split(","):
        name, _, rows = item.partition(":")
        if name.strip() not in _OWN_UP_TO:
            raise ValueError(f"FDLLM_OWN_UP_TO: unknown projection {name!r}")
        _OWN_UP_TO[name.strip()] = int(rows)


_own_up_to_env()


def use_own(op: str, rows: int) -> bool:
    """This package's GEMM (True) or cuBLAS (False) for projection `op`."""
    if OWN_GEMMS is not None:
        return OWN_GEMMS[op]
    return rows <= _OWN_UP_TO[op]


def _norm_weight(module) -> torch.Tensor:
    w = getattr(module, "weight", None)
    if w is None or w.dtype != torch.bfloat16 or getattr(module, "bias", None) is not None:
        raise TypeError("flash_fused_elastic_cache needs bf16 RMSNorm modules with a weight and no bias")
    return w


def _eps(module) -> float:
    return float(getattr(module, "eps", 1e-5))


class _PlanCache:
    """The attention plan of one forward pass, one entry per device: every
    layer of a forward gets the same block-table tensor objects, so the plan
    is built at the first layer and reused by the others.  An entry matches
    only the same tensor objects (held, so their identity cannot be recycled
    while cached) at the same version counter (an in-place edit of a table
    bumps it and forces a new plan), and the same sizes."""

    def __init__(self):
        self.entries = {}

    @staticmethod
    def _key(masked, tracked, n_rows, batch, block_m, max_length):
        ver = tuple(None if t is None else t._version for t in (masked, tracked))
        return (masked, tracked, ver, n_rows, batch, block_m, max_length)

    def get(self, masked, tracked, n_rows, batch, block_m, max_length, device):
        dev = device.index if device.index is not None else torch.cuda.current_device()
        key = self._key(masked, tracked, n_rows, batch, block_m, max_length)
        hit = self.entries.get(dev)
        if hit is not None and all(a is b if isinstance(a, torch.Tensor) else a == b for a, b in zip(hit[0], key)):
            return hit[1]
        value = ops.plan_cache_attention(masked, tracked, n_rows, batch, block_m, max_length, device)
        self.entries[dev] = (key, value)
        return value


_PLANS = _PlanCache()


def flash_fused_elastic_cache(self, x: torch.Tensor, block_idx, positions, lengths, softmax_scale: float = None):
    query_pos_flat, key_pos_flat, rotary_emb_pos, _info, attn_scores, attn_mask = positions
    (_start_layer, query_verify_blocks, query_masked_blocks, query_tracked_blocks, _query_blocks, active_batch,
     _num_active, max_length, block_m, _block_n, _elastic, verify) = lengths
    d_model = self.config.d_model
    n_heads = self.config.n_heads
    head_dim = d_model // n_heads
    softmax_scale = softmax_scale or (1.0 / math.sqrt(head_dim))
    x = x.contiguous()
    n_rows = x.shape[0]
    x_normed = ops.rmsnorm(x, _norm_weight(self.attn_norm), _eps(self.attn_norm))
    att = torch.empty_like(x)
    q = torch.empty_like(x)
    sin, cos = rotary_emb_pos
    wq, wk, wv = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight

    if verify:
        k1 = torch.empty_like(x)
        v1 = torch.empty_like(x)
        ops.verify_qkv(x_normed, wq, wk, wv, query_pos_flat, sin, cos, q, k1, v1, n_heads)
        ops.verify_attn(q, k1, v1, att, self.k_cache, self.v_cache, key_pos_flat, attn_mask, query_verify_blocks,
                        2 * block_m, n_heads, softmax_scale, max_keys=max_length)
    else:
        if n_rows > 0:
            ops.qkv_rope_cache(x_normed, wq, wk, wv, query_pos_flat, sin, cos, q, self.k_cache, self.v_cache,
                               n_heads)
            plan, cap = _PLANS.get(query_masked_blocks, query_tracked_blocks, n_rows, len(active_batch), block_m,
                                   max_length, x.device)
            scores = attn_scores if block_idx > 1 else None
            ops.attn_cache(q, att, self.k_cache, self.v_cache, plan, cap, scores, 1.0 / (block_m * n_heads),
                           n_heads, max_length, softmax_scale, items_hint=-(-n_rows // 64))

    # Residual adds: into the GEMM epilogue (C = x + att W^T, one bf16 rounding
    # of the sum instead of two) when the projection is a plain bias-free
    # Linear and dropout is the identity; else the add is fused with ff_norm.
    plain = _plain_linear(self.attn_out) and _plain_linear(self.ff_out) and isinstance(
        self.dropout, torch.nn.Identity)
    if plain:
        if use_own("attn_out", n_rows):
            og_x = ops.linear(att, self.attn_out.weight, residual=x)
        else:
            og_x = torch.addmm(x, att, self.attn_out.weight.t())
        h = ops.rmsnorm(og_x, _norm_weight(self.ff_norm), _eps(self.ff_norm))
    else:
        og_x, h = ops.add_rmsnorm(x, self.dropout(self.attn_out(att)), _norm_weight(self.ff_norm),
                                  _eps(self.ff_norm))
    fused = getattr(self, "ffup_weight", None)
    silu = isinstance(self.act, torch.nn.SiLU)
    if fused is not None and silu and use_own("mlp", n_rows):
        h = ops.linear_swiglu(h, fused)  # [ff_proj; up_proj] stacked: one GEMM, SwiGLU in its epilogue
    else:
        if fused is not None:
            gu = torch.nn.functional.linear(h, fused)
            hid = gu.shape[1] // 2
            gate, up = gu[:, :hid], gu[:, hid:]
        else:
            gate, up = self.ff_proj(h), self.up_proj(h)
        h = ops.swiglu(gate, up) if silu else self.act(gate) * up
    if plain:
        if use_own("ff_out", n_rows):
            return ops.linear(h, self.ff_out.weight, residual=og_x).unsqueeze(0)
        return torch.addmm(og_x, h, self.ff_out.weight.t()).unsqueeze(0)
    h = self.dropout(self.ff_out(h))
    return (og_x + h).unsqueeze(0)


def _plain_linear(m) -> bool:
    return type(m) is torch.nn.Linear and m.bias is None and m.weight.dtype == torch.bfloat16


def install_into_reference(modeling_module) -> None:
    """Rebind the operator the reference model calls.

    The reference imports the operator into ``llada/model/modeling_llada.py``
    (line 55) and calls it from ``LLaDABlock.attention`` (line 760), so
    replacing that module attribute routes every layer through this package.
    """
    modeling_module.flash_fused_elastic_cache = flash_fused_elastic_cache
