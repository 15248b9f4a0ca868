"""Loading a LLaDA checkpoint and its tokenizer from a local directory.

The reference loads the model with ``LLaDAModelLM.from_pretrained(model_path,
torch_dtype=torch.bfloat16)`` and the tokenizer with
``AutoTokenizer.from_pretrained(model_path, trust_remote_code=True)``
(``llada/eval_llada.py:104-119``).  A LLaDA checkpoint directory holds
``config.json`` (``configuration_llada.py`` field names), the weights as
safetensors (``model.safetensors``, or shards listed by
``model.safetensors.index.json``) under the reference's parameter names
(``model.transformer.blocks.<i>.q_proj.weight`` ...), and the tokenizer
files.  This module reads them into :class:`LLaDAModelB200`, whose module
tree carries the same names, so the state dict loads with ``strict=True``.

The safetensors reader is this package's own: an 8-byte little-endian header
length, a JSON header (name -> dtype, shape, byte range; optional
``__metadata__``), then the raw little-endian tensor bytes; tensors are read
one at a time and copied to the target device (a full LLaDA-8B never sits in
host memory whole).
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, Iterator, Optional, Tuple

import numpy as np
import torch

from .model import LLaDAConfigB200, LLaDAModelB200

_DTYPES = {
    "BF16": (torch.bfloat16, 2), "F16": (torch.float16, 2), "F32": (torch.float32, 4), "F64": (torch.float64, 8),
    "I64": (torch.int64, 8), "I32": (torch.int32, 4), "I16": (torch.int16, 2), "I8": (torch.int8, 1),
    "U8": (torch.uint8, 1), "BOOL": (torch.bool, 1),
}


def safetensors_header(path: str) -> Tuple[dict, int]:
    """(header without ``__metadata__``, byte offset of the data section)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        (n,) = struct.unpack("<Q", raw)
        if n > 100 << 20:
            raise ValueError(f"{path}: safetensors header of {n} bytes")
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header, 8 + n


def iter_safetensors(path: str, device="cpu") -> Iterator[Tuple[str, torch.Tensor]]:
    """Yield (name, tensor) for every tensor of one safetensors file: each is
    read straight into a host tensor of its own and copied onto `device`."""
    header, base = safetensors_header(path)
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        for name, meta in sorted(header.items(), key=lambda kv: kv[1]["data_offsets"][0]):
            dtype, item = _DTYPES[meta["dtype"]]
            shape = tuple(int(s) for s in meta["shape"])
            b0, b1 = (int(v) for v in meta["data_offsets"])
            n = int(np.prod(shape)) if shape else 1
            if b1 - b0 != n * item or base + b1 > size:
                raise ValueError(f"{path}: tensor {name} has {b1 - b0} bytes for shape {shape} {meta['dtype']}")
            raw = torch.empty(b1 - b0, dtype=torch.uint8)
            f.seek(base + b0)
            if f.readinto(raw.numpy()) != b1 - b0:
                raise ValueError(f"{path}: tensor {name} is truncated")
            yield name, raw.view(dtype).reshape(shape).to(device)


def weight_files(path: str) -> list:
    """The safetensors files of a checkpoint directory (sharded or not)."""
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, s) for s in shards]
    single = os.path.join(path, "model.safetensors")
    if os.path.exists(single):
        return [single]
    raise FileNotFoundError(f"no model.safetensors or model.safetensors.index.json in {path}")


def config_from_json(path: str) -> LLaDAConfigB200:
    """LLaDAConfigB200 from a checkpoint's ``config.json`` (the reference's
    ``configuration_llada.py`` names; ``embedding_size`` sizes the embedding
    and LM head when it differs from ``vocab_size``)."""
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    if c.get("block_type", "llama") != "llama" or c.get("include_bias", False):
        raise ValueError("only LLaMA-style LLaDA blocks without biases are supported")
    if c.get("weight_tying", False):
        raise ValueError("weight-tied checkpoints are not supported (LLaDA-8B has an untied LM head)")
    vocab = int(c.get("embedding_size") or c["vocab_size"])
    return LLaDAConfigB200(d_model=int(c["d_model"]), n_heads=int(c["n_heads"]), n_layers=int(c["n_layers"]),
                           mlp_hidden_size=int(c["mlp_hidden_size"]), vocab_size=vocab,
                           rope_theta=float(c.get("rope_theta", 500000.0)),
                           rms_norm_eps=float(c.get("rms_norm_eps", 1e-5)),
                           mask_token_id=int(c.get("mask_token_id", 126336)),
                           eos_token_id=int(c.get("eos_token_id", 126081)))


@torch.no_grad()
def load_model(path: str, device="cuda", dtype=torch.bfloat16, fuse_mlp: bool = True) -> LLaDAModelB200:
    """LLaDAModelB200 with the weights of the checkpoint directory `path`
    (every parameter must be present, none may be left over), cast to
    `dtype` on `device`; the MLP weights are stacked for the fused GEMM."""
    cfg = config_from_json(path)
    with torch.device("meta"):
        model = LLaDAModelB200(cfg, device="meta", dtype=dtype)
    model = model.to_empty(device=device)
    params = dict(model.named_parameters())
    seen = set()
    for f in weight_files(path):
        for name, t in iter_safetensors(f, device):
            p = params.get(name)
            if p is None:
                raise KeyError(f"unexpected tensor {name} in {f}")
            if tuple(p.shape) != tuple(t.shape):
                raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} vs model {tuple(p.shape)}")
            p.copy_(t.to(dtype))
            seen.add(name)
    missing = sorted(set(params) - seen)
    if missing:
        raise KeyError(f"checkpoint lacks {len(missing)} tensors, e.g. {missing[:3]}")
    if fuse_mlp:
        model.fuse_mlp_weights()
    return model.eval()


def load_tokenizer(path: str, trust_remote_code: bool = True):
    """The checkpoint's tokenizer, as the reference loads it
    (``AutoTokenizer.from_pretrained(path, trust_remote_code=True)``)."""
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained(path, trust_remote_code=trust_remote_code)


def from_pretrained(path: str, device="cuda", dtype=torch.bfloat16, tokenizer: bool = True
                    ) -> Tuple[LLaDAModelB200, Optional[object]]:
    """(model, tokenizer or None) from a local LLaDA checkpoint directory."""
    model = load_model(path, device=device, dtype=dtype)
    return model, (load_tokenizer(path) if tokenizer else None)


def state_dict_from_files(path: str, device="cpu") -> Dict[str, torch.Tensor]:
    """Every tensor of the checkpoint directory as one dict (tests, tools)."""
    out = {}
    for f in weight_files(path):
        out.update(dict(iter_safetensors(f, device)))
    return out
