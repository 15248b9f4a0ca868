"""Generate the golden fixtures in this folder from the reference itself.

Run once in a container that has the reference checkout (VILA-Lab/Flash-dLLM)
and triton; the GPU box never runs this:

    python tests/golden/make_golden.py --reference <checkout>/llada

It imports the reference read-only and runs, on the CPU in fp32:

* the five Triton kernels of ``llada/flash_cache_triton.py`` under Triton's
  interpreter (``TRITON_INTERPRET=1``) on the seeded inputs of
  ``cases.py`` -> ``kernels_fp32.npz``;
* the reference layer driver ``flash_fused_elastic_cache`` on a reference
  ``LLaDALlamaBlock`` in both modes -> ``layer_fp32.npz``;
* the reference ``generate_with_Flash_dLLM`` on a tiny random-init LLaDA in
  both modes, recording every forward's query tokens and slots ->
  ``generate_fp32.npz``.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

os.environ["TRITON_INTERPRET"] = "1"

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root (for oracle/, tests/)
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import cases  # noqa: E402


def _ref_modules(ref_dir):
    sys.path.insert(0, ref_dir)
    import flash_cache_triton as fct  # noqa: F401
    import generate as rgen
    from model.configuration_llada import LLaDAConfig
    from model.modeling_llada import LLaDAModelLM
    return fct, rgen, LLaDAConfig, LLaDAModelLM


def kernels(fct):
    c = cases.cache_case()
    D, H, hd, bm = cases.D_MODEL, cases.N_HEADS, cases.HEAD_DIM, cases.BLOCK_M
    q = torch.zeros_like(c["xn"])
    kc, vc = c["k_cache"].clone(), c["v_cache"].clone()
    qb = torch.cat([c["masked_blocks"], c["tracked_blocks"]])
    fct._flash_qkv_proj_cache_fwd[(qb.shape[0], H)](
        c["xn"], q, kc, vc, c["pos"], qb, c["wq"], c["wk"], c["wv"], c["sin"], c["cos"],
        D_MODEL=D, HALF=hd // 2, HEAD_DIM=hd, BLOCK_M=bm, BLOCK_D=64, NUM_BLOCKS=qb.shape[0],
        num_stages=2)
    att = torch.zeros_like(c["xn"])
    S = torch.zeros((bm, H, 2, cases.LMAX), dtype=torch.float32)
    scale = 1.0 / hd ** 0.5
    fct._flash_masked_attention_fwd[(c["masked_blocks"].shape[0], H)](
        q, att, kc, vc, S, S.stride(0), S.stride(1), S.stride(2), c["masked_blocks"], scale,
        SEQLEN_MAX=cases.LMAX, D_MODEL=D, HEAD_DIM=hd, BLOCK_M=bm, BLOCK_N=128)
    fct._flash_tracked_attention_fwd[(c["tracked_blocks"].shape[0], H)](
        q, att, kc, vc, c["tracked_blocks"], scale, NUM_BLOCKS=c["tracked_blocks"].shape[0],
        SEQLEN_MAX=cases.LMAX, D_MODEL=D, HEAD_DIM=hd, BLOCK_M=bm, BLOCK_N=128, num_stages=2)

    v = cases.verify_case()
    q1, k1, v1, o = (torch.zeros_like(v["xn"]) for _ in range(4))
    nb = v["blocks"].shape[0]
    fct._flash_verify_qkv_proj_fwd[(nb, H)](
        v["xn"], q1, k1, v1, v["pos"], v["wq"], v["wk"], v["wv"], v["sin"], v["cos"], v["blocks"],
        HALF=hd // 2, D_MODEL=D, HEAD_DIM=hd, BLOCK_M=2 * bm, BLOCK_D=32)
    fct._flash_verify_attention_fwd[(nb, H)](
        q1, k1, v1, o, v["k_cache"], v["v_cache"], v["pos_k"], v["attn_mask"], v["blocks"], scale,
        D_MODEL=D, HEAD_DIM=hd, BLOCK_M=2 * bm, BLOCK_N=64)
    p = c["pos"]
    np.savez_compressed(os.path.join(HERE, "kernels_fp32.npz"),
                        q=q.numpy(), k_rows=kc[p].numpy(), v_rows=vc[p].numpy(), att=att.numpy(),
                        S=S.numpy(), vq1=q1.numpy(), vk1=k1.numpy(), vv1=v1.numpy(), vo=o.numpy())


def _ref_model(LLaDAConfig, LLaDAModelLM, cfg, weights):
    rc = LLaDAConfig(d_model=cfg.d_model, n_heads=cfg.n_heads, n_layers=cfg.n_layers,
                     mlp_hidden_size=cfg.mlp_hidden_size, vocab_size=cfg.vocab_size,
                     embedding_size=cfg.vocab_size, weight_tying=False, block_type="llama",
                     layer_norm_type="rms", activation_type="silu", rope=True, rope_theta=cfg.rope_theta,
                     rms_norm_eps=cfg.rms_norm_eps, include_bias=False, residual_dropout=0.0,
                     embedding_dropout=0.0, attention_dropout=0.0, flash_attention=False,
                     init_device="cpu", max_sequence_length=4096)
    m = LLaDAModelLM(rc, init_params=False)
    m.load_state_dict(weights, strict=True)
    return m.eval()


def layer(fct, LLaDAConfig, LLaDAModelLM):
    cfg, w = cases.gen_weights()
    m = _ref_model(LLaDAConfig, LLaDAModelLM, cfg, w)
    blk = m.model.transformer.blocks[2]
    out = {}
    c = cases.cache_case()
    blk.k_cache, blk.v_cache = c["k_cache"].clone(), c["v_cache"].clone()
    scores = torch.zeros(2 * cases.LMAX)
    qb = torch.cat([c["masked_blocks"], c["tracked_blocks"]])
    positions = [c["pos"], torch.tensor([], dtype=torch.int32), [c["sin"], c["cos"]], [], scores, []]
    lengths = [[-1, -1], None, c["masked_blocks"], c["tracked_blocks"], qb, [0, 1], 2, cases.LMAX,
               cases.BLOCK_M, 128, None, False]
    with torch.no_grad():
        y = fct.flash_fused_elastic_cache(blk, c["xn"], 2, positions, lengths)
    out.update(cache_out=y.squeeze(0).numpy(), cache_scores=scores.numpy(),
               cache_k_rows=blk.k_cache[c["pos"]].numpy(), cache_v_rows=blk.v_cache[c["pos"]].numpy())
    v = cases.verify_case()
    blk.k_cache, blk.v_cache = v["k_cache"].clone(), v["v_cache"].clone()
    positions = [v["pos"], v["pos_k"], [v["sin"], v["cos"]], [], torch.zeros(2 * cases.LMAX), v["attn_mask"]]
    lengths = [[-1, -1], v["blocks"], None, torch.tensor([], dtype=torch.int32), None, [0, 1], 2,
               cases.LMAX, cases.BLOCK_M, 128, None, True]
    with torch.no_grad():
        y = fct.flash_fused_elastic_cache(blk, v["xn"], 2, positions, lengths)
    out.update(verify_out=y.squeeze(0).numpy())
    np.savez_compressed(os.path.join(HERE, "layer_fp32.npz"), **out)


class _Recorder:
    def __init__(self):
        self.rows = []

    def __call__(self, module, args, kwargs):
        pos = kwargs["positions"]
        ln = kwargs["lengths"]
        x_query = args[0] if args else kwargs["input_ids"]
        verify = bool(ln[11])
        self.rows.append(dict(
            verify=verify,
            x=x_query.reshape(-1).numpy().copy(),
            qpos=pos[0].reshape(-1).numpy().astype(np.int64).copy(),
            kpos=(pos[1].reshape(-1).numpy().astype(np.int64).copy() if verify else np.zeros(0, np.int64)),
        ))


def _pack(prefix, rows):
    out = {}
    for key in ("x", "qpos", "kpos"):
        arrs = [r[key] for r in rows]
        out[f"{prefix}_{key}"] = np.concatenate(arrs) if arrs else np.zeros(0, np.int64)
        out[f"{prefix}_{key}_len"] = np.array([len(a) for a in arrs], np.int64)
    out[f"{prefix}_verify"] = np.array([r["verify"] for r in rows], np.bool_)
    return out


def generate(rgen, LLaDAConfig, LLaDAModelLM):
    from oracle.decode_oracle import StubTokenizer
    from oracle.tiny_model import weights_checksum
    cfg, w = cases.gen_weights()
    out = {}
    for verify in (False, True):
        m = _ref_model(LLaDAConfig, LLaDAModelLM, cfg, w)
        rec = _Recorder()
        m.register_forward_pre_hook(rec, with_kwargs=True)
        prompts = cases.gen_prompts()
        n = len(prompts)
        responses, n_steps = [""] * n, [0] * n
        t = time.time()
        responses, num_tokens, max_num_tokens = rgen.generate_with_Flash_dLLM(
            m, prompts, list(cases.GEN_PROMPT_LENS), cases.GEN_BATCH, responses, n_steps,
            verify=verify, tokenizer=StubTokenizer(), stop_tokens=[], gen_length=cases.GEN_LEN[verify],
            **cases.GEN_KW)
        tag = "verify" if verify else "cache"
        print(f"reference generate verify={verify}: {time.time() - t:.1f}s, {len(rec.rows)} forwards",
              flush=True)
        out.update(_pack(tag, rec.rows))
        out[f"{tag}_n_steps"] = np.array(n_steps, np.int64)
        out[f"{tag}_num_tokens"] = np.array([num_tokens, max_num_tokens], np.int64)
        toks = [np.array([int(t) for t in r.split()], np.int64) for r in responses]
        out[f"{tag}_resp"] = np.concatenate(toks)
        out[f"{tag}_resp_len"] = np.array([len(t) for t in toks], np.int64)
        out["weights_checksum"] = np.array(weights_checksum(w))
        # save after each mode so a later failure keeps the earlier results
        np.savez_compressed(os.path.join(HERE, "generate_fp32.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference's llada/ directory")
    ap.add_argument("--only", default="kernels,layer,generate")
    a = ap.parse_args()
    fct, rgen, LLaDAConfig, LLaDAModelLM = _ref_modules(os.path.abspath(a.reference))
    torch.manual_seed(0)
    only = a.only.split(",")
    if "kernels" in only:
        kernels(fct)
    if "layer" in only:
        layer(fct, LLaDAConfig, LLaDAModelLM)
    if "generate" in only:
        generate(rgen, LLaDAConfig, LLaDAModelLM)


if __name__ == "__main__":
    main()
