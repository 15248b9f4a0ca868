"""Seeded LLaDA weights and a CPU forward over the oracle layer.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Parameter names follow the reference HF model
(``llada/model/modeling_llada.py``: ``LLaDAModel.transformer`` with ``wte``,
``blocks.{i}.{attn_norm,q_proj,k_proj,v_proj,attn_out,ff_norm,ff_proj,up_proj,
ff_out}``, ``ln_f``, ``ff_out``) so the same tensors load into the reference
model (for pinning) and into the product's model shell (for GPU tests).
"""
from __future__ import annotations

import dataclasses
from types import SimpleNamespace
from typing import Dict

import torch

from . import flash_cache_oracle as fco


@dataclasses.dataclass
class TinyConfig:
    d_model: int = 256
    n_heads: int = 2
    n_layers: int = 3
    mlp_hidden_size: int = 512
    vocab_size: int = 512
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-5
    init_std: float = 0.02
    head_std: float = 0.02  # std of the LM head; larger values make confident predictions


def make_weights(cfg: TinyConfig, seed: int) -> Dict[str, torch.Tensor]:
    """fp32 weights ``N(0, init_std)`` (norm weights 1, embedding N(0,1), LM
    head ``N(0, head_std)``), drawn from one seeded CPU generator in a fixed
    order."""
    g = torch.Generator().manual_seed(seed)
    d, h, v = cfg.d_model, cfg.mlp_hidden_size, cfg.vocab_size

    def n(*shape, std=cfg.init_std):
        return torch.randn(*shape, generator=g) * std

    w = {"model.transformer.wte.weight": n(v, d, std=1.0)}
    for i in range(cfg.n_layers):
        p = f"model.transformer.blocks.{i}."
        w[p + "attn_norm.weight"] = torch.ones(d)
        w[p + "q_proj.weight"] = n(d, d)
        w[p + "k_proj.weight"] = n(d, d)
        w[p + "v_proj.weight"] = n(d, d)
        w[p + "attn_out.weight"] = n(d, d)
        w[p + "ff_norm.weight"] = torch.ones(d)
        w[p + "ff_proj.weight"] = n(h, d)
        w[p + "up_proj.weight"] = n(h, d)
        w[p + "ff_out.weight"] = n(d, h)
    w["model.transformer.ln_f.weight"] = torch.ones(d)
    w["model.transformer.ff_out.weight"] = n(v, d, std=cfg.head_std)
    return w


def weights_checksum(w: Dict[str, torch.Tensor]) -> float:
    """Order-independent fp64 checksum used to detect RNG drift in fixtures."""
    return float(sum(t.double().abs().sum() for t in w.values()))


class _Lin:
    def __init__(self, weight):
        self.weight = weight


class TinyLLaDA:
    """CPU LLaDA forward: embedding -> oracle layers -> ln_f -> LM head
    (modeling_llada.py:1386-1488 on the ``use_cache`` path)."""

    def __init__(self, cfg: TinyConfig, weights: Dict[str, torch.Tensor], dtype=torch.float32):
        self.cfg = cfg
        self.dtype = dtype
        W = {k: t.to(dtype) for k, t in weights.items()}
        self.wte = W["model.transformer.wte.weight"]
        self.ln_f = W["model.transformer.ln_f.weight"]
        self.head = W["model.transformer.ff_out.weight"]
        conf = SimpleNamespace(d_model=cfg.d_model, n_heads=cfg.n_heads)
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"model.transformer.blocks.{i}."
            blk = SimpleNamespace(config=conf)
            an, fn = W[p + "attn_norm.weight"], W[p + "ff_norm.weight"]
            blk.attn_norm = (lambda x, w=an: fco.rms_norm(x, w, cfg.rms_norm_eps))
            blk.ff_norm = (lambda x, w=fn: fco.rms_norm(x, w, cfg.rms_norm_eps))
            for name in ("q_proj", "k_proj", "v_proj", "attn_out", "ff_proj", "up_proj", "ff_out"):
                setattr(blk, name, _Lin(W[p + name + ".weight"]))
            self.layers.append(blk)

    def forward(self, x_query: torch.Tensor, lengths, positions) -> torch.Tensor:
        x = self.wte[x_query.view(-1)]
        for i, blk in enumerate(self.layers):
            x = fco.flash_fused_elastic_cache(blk, x, i, positions, lengths).squeeze(0)
        x = fco.rms_norm(x, self.ln_f, self.cfg.rms_norm_eps)
        return fco.linear(x, self.head)
