"""Checkpoint loading (CPU): a LLaDA checkpoint directory written with the
official safetensors writer -- config.json with the reference's field names,
the reference's parameter names, one file or shards with an index -- loads
into LLaDAModelB200 tensor for tensor through this package's own reader;
missing, unexpected and mis-shaped tensors are refused."""
import json
import os

import pytest
import torch

import cases

safetensors_torch = pytest.importorskip("safetensors.torch")


def _write(tmp, w, cfg, shards=1):
    names = sorted(w)
    conf = dict(d_model=cfg.d_model, n_heads=cfg.n_heads, n_layers=cfg.n_layers,
                mlp_hidden_size=cfg.mlp_hidden_size, vocab_size=cfg.vocab_size, embedding_size=cfg.vocab_size,
                rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps, block_type="llama", include_bias=False,
                weight_tying=False, mask_token_id=511, eos_token_id=510)
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump(conf, f)
    if shards == 1:
        safetensors_torch.save_file({n: w[n].contiguous() for n in names}, os.path.join(tmp, "model.safetensors"),
                                    metadata={"format": "pt"})
        return
    wmap = {}
    for k in range(shards):
        part = names[k::shards]
        fn = f"model-{k + 1:05d}-of-{shards:05d}.safetensors"
        safetensors_torch.save_file({n: w[n].contiguous() for n in part}, os.path.join(tmp, fn))
        wmap.update({n: fn for n in part})
    with open(os.path.join(tmp, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wmap}, f)


@pytest.mark.parametrize("shards,dtype", [(1, torch.float32), (3, torch.bfloat16)])
def test_checkpoint_round_trip(tmp_path, shards, dtype):
    from flash_dllm_b200.checkpoint import load_model, state_dict_from_files
    cfg, w = cases.gen_weights()
    w = {k: v.to(dtype) for k, v in w.items()}
    _write(str(tmp_path), w, cfg, shards)
    assert all(torch.equal(state_dict_from_files(str(tmp_path))[k], w[k]) for k in w)
    m = load_model(str(tmp_path), device="cpu", dtype=dtype)
    assert m.config.mask_token_id == 511 and m.config.n_layers == cfg.n_layers
    sd = m.state_dict()
    for k, v in w.items():
        assert torch.equal(sd[k], v), k
    blk = m.model.transformer.blocks[1]
    h = cfg.mlp_hidden_size
    assert torch.equal(blk.ffup_weight[:h], w["model.transformer.blocks.1.ff_proj.weight"])  # stacked MLP weight
    assert torch.equal(blk.ffup_weight[h:], w["model.transformer.blocks.1.up_proj.weight"])


def test_checkpoint_refuses_incomplete_or_foreign(tmp_path):
    from flash_dllm_b200.checkpoint import load_model
    cfg, w = cases.gen_weights()
    w = dict(w)
    w.pop("model.transformer.ln_f.weight")
    _write(str(tmp_path), w, cfg)
    with pytest.raises(KeyError, match="lacks"):
        load_model(str(tmp_path), device="cpu", dtype=torch.float32)
    cfg, w = cases.gen_weights()
    w = dict(w, extra=torch.zeros(3))
    _write(str(tmp_path), w, cfg)
    with pytest.raises(KeyError, match="unexpected"):
        load_model(str(tmp_path), device="cpu", dtype=torch.float32)
    cfg, w = cases.gen_weights()
    w = dict(w)
    w["model.transformer.ln_f.weight"] = torch.ones(7)
    _write(str(tmp_path), w, cfg)
    with pytest.raises(ValueError, match="shape"):
        load_model(str(tmp_path), device="cpu", dtype=torch.float32)
