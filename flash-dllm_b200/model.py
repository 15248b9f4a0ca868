"""LLaDA model shell around the fused layer operator.

Mirrors the module tree of the reference HF model
(``llada/model/modeling_llada.py``: ``LLaDAModelLM.model.transformer`` with
``wte``, ``blocks[i]`` = LLaMA-style ``LLaDALlamaBlock``, ``ln_f``,
``ff_out``), so state dicts of the reference load unchanged and
``generate_with_Flash_dLLM`` reaches the same attributes
(``model.model.transformer.blocks``, ``model.config.{d_model,n_heads,
n_layers,rope_theta}``, ``model.device``, ``model.dtype``).  Only the
inference path the decode driver uses is kept: embedding -> blocks (each one
``flash_fused_elastic_cache`` call) -> ``ln_f`` -> LM head.  ``logit_rows``
optionally limits the LM head to the rows the driver reads.
"""
from __future__ import annotations

import dataclasses
from types import SimpleNamespace
from typing import Optional

import torch
from torch import nn

from . import ops
from .flash_cache import flash_fused_elastic_cache, use_own


@dataclasses.dataclass
class LLaDAConfigB200:
    """LLaDA-8B shape by default (configuration_llada.py fields of the same names)."""
    d_model: int = 4096
    n_heads: int = 32
    n_layers: int = 32
    mlp_hidden_size: int = 12288
    vocab_size: int = 126464
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-5
    mask_token_id: int = 126336
    eos_token_id: int = 126081


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, device=device, dtype=dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        return ops.rmsnorm(x.reshape(-1, shape[-1]).contiguous(), self.weight, self.eps).view(shape)


class LLaDABlockB200(nn.Module):
    def __init__(self, cfg: LLaDAConfigB200, layer_id: int, device=None, dtype=None):
        super().__init__()
        kw = dict(bias=False, device=device, dtype=dtype)
        d, h = cfg.d_model, cfg.mlp_hidden_size
        self.layer_id = layer_id
        self.config = cfg
        self.attn_norm = RMSNorm(d, cfg.rms_norm_eps, device, dtype)
        self.ff_norm = RMSNorm(d, cfg.rms_norm_eps, device, dtype)
        self.q_proj = nn.Linear(d, d, **kw)
        self.k_proj = nn.Linear(d, d, **kw)
        self.v_proj = nn.Linear(d, d, **kw)
        self.attn_out = nn.Linear(d, d, **kw)
        self.ff_proj = nn.Linear(d, h, **kw)
        self.up_proj = nn.Linear(d, h, **kw)
        self.ff_out = nn.Linear(h, d, **kw)
        self.act = nn.SiLU()
        self.dropout = nn.Identity()
        self.k_cache = None
        self.v_cache = None

    def forward(self, x, positions=None, lengths=None, block_idx=0):
        return flash_fused_elastic_cache(self, x.squeeze(0), block_idx, positions, lengths)

    @torch.no_grad()
    def fuse_mlp_weights(self) -> None:
        """Stack ``ff_proj`` and ``up_proj`` weights into one (2*hidden,
        d_model) tensor ``ffup_weight`` so the operator runs one GEMM for
        both; the two Linear weights become views of it (no extra memory, and
        a later ``load_state_dict`` copies into the views)."""
        w1, w2 = self.ff_proj.weight, self.up_proj.weight
        fused = torch.cat([w1.detach(), w2.detach()], 0)
        h = w1.shape[0]
        self.ff_proj.weight = nn.Parameter(fused[:h], requires_grad=False)
        self.up_proj.weight = nn.Parameter(fused[h:], requires_grad=False)
        self.ffup_weight = fused


class _Transformer(nn.Module):
    def __init__(self, cfg, device, dtype):
        super().__init__()
        self.wte = nn.Embedding(cfg.vocab_size, cfg.d_model, device=device, dtype=dtype)
        self.blocks = nn.ModuleList(LLaDABlockB200(cfg, i, device, dtype) for i in range(cfg.n_layers))
        self.ln_f = RMSNorm(cfg.d_model, cfg.rms_norm_eps, device, dtype)
        self.ff_out = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False, device=device, dtype=dtype)


class _Inner(nn.Module):
    def __init__(self, cfg, device, dtype):
        super().__init__()
        self.transformer = _Transformer(cfg, device, dtype)


class LLaDAModelB200(nn.Module):
    def __init__(self, cfg: Optional[LLaDAConfigB200] = None, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.config = cfg or LLaDAConfigB200()
        self.model = _Inner(self.config, device, dtype)

    @property
    def device(self) -> torch.device:
        return self.model.transformer.wte.weight.device

    @property
    def dtype(self) -> torch.dtype:
        return self.model.transformer.wte.weight.dtype

    @classmethod
    def random_init(cls, cfg: Optional[LLaDAConfigB200] = None, device="cuda", seed: int = 0, std: float = 0.02):
        """Weights N(0, std), norm weights 1, drawn on ``device`` in bf16."""
        with torch.device("meta"):
            m = cls(cfg, device="meta")
        m = m.to_empty(device=device)
        g = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for name, p in m.named_parameters():
                if name.endswith("norm.weight") or name.endswith("ln_f.weight"):
                    p.fill_(1.0)
                else:
                    p.normal_(0.0, std, generator=g)
        m.fuse_mlp_weights()
        return m.eval()

    def fuse_mlp_weights(self) -> None:
        """``LLaDABlockB200.fuse_mlp_weights`` on every block."""
        for blk in self.model.transformer.blocks:
            blk.fuse_mlp_weights()

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, use_cache: bool = True, lengths=None, positions=None,
                logit_rows: Optional[torch.Tensor] = None, layer_hook=None, **_unused):
        """``input_ids`` (1, Nq) -> ``.logits`` (1, Nq, vocab), or (1, R, vocab)
        for the R rows listed in ``logit_rows`` (an int64 index tensor or an
        int prefix length).  ``layer_hook(block_idx)`` runs after each block
        (the decode loop uses it to split a CUDA-graph capture)."""
        t = self.model.transformer
        x = t.wte(input_ids.reshape(-1))
        for block_idx, block in enumerate(t.blocks):
            x = flash_fused_elastic_cache(block, x, block_idx, positions, lengths).squeeze(0)
            if layer_hook is not None:
                layer_hook(block_idx)
        if logit_rows is not None:
            x = x[:logit_rows] if isinstance(logit_rows, int) else x.index_select(0, logit_rows)
        x = t.ln_f(x.contiguous())
        w = t.ff_out.weight
        if use_own("lm_head", x.shape[0]) and t.ff_out.bias is None and w.dtype == torch.bfloat16 and w.shape[0] % 32 == 0 \
                and w.shape[1] % 64 == 0:
            return SimpleNamespace(logits=ops.linear(x, w).unsqueeze(0))
        return SimpleNamespace(logits=t.ff_out(x).unsqueeze(0))
