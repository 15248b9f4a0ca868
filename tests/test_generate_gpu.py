"""End-to-end decode parity on the GPU by replay.

The product's ``generate_with_Flash_dLLM`` runs on the GPU (bf16, this
package's kernels) on the tiny LLaDA of the golden fixtures and records every
forward: its query tokens and slots, verify key slots, the logit rows it read
and the attention scores.  The CPU oracle of the reference decode loop is then
driven with those recorded logits and scores; every forward it issues must ask
for exactly the recorded queries, and the step counts, token counts and
decoded tokens must match.  This checks the whole decode driver (acceptance,
verify build and scan, refresh order, continuous-batch refill, EOS handling)
against the reference's semantics given identical model outputs."""
import numpy as np
import pytest
import torch

import cases
from oracle import decode_oracle as do

pytestmark = pytest.mark.gpu


def _model():
    from flash_dllm_b200.model import LLaDAConfigB200, LLaDAModelB200
    cfg, w = cases.gen_weights()
    c = LLaDAConfigB200(d_model=cfg.d_model, n_heads=cfg.n_heads, n_layers=cfg.n_layers,
                        mlp_hidden_size=cfg.mlp_hidden_size, vocab_size=cfg.vocab_size, rope_theta=cfg.rope_theta,
                        rms_norm_eps=cfg.rms_norm_eps, mask_token_id=cases.GEN_KW["mask_id"],
                        eos_token_id=cases.GEN_KW["eos_id"])
    m = LLaDAModelB200(c, device="cuda")
    m.load_state_dict({k: v.to(torch.bfloat16) for k, v in w.items()}, strict=True)
    m.fuse_mlp_weights()
    return m.eval()


@pytest.mark.parametrize("verify,min_keep", [(False, 1), (True, 1), (False, 2)])
def test_generate_replays_through_oracle(verify, min_keep):
    from flash_dllm_b200.generate import generate_with_Flash_dLLM
    from flash_dllm_b200._lib import check_device_status
    model = _model()
    recs = []

    def record(v, xq, qpos, kpos, logits, rows, scores):
        recs.append(dict(v=v, x=xq.reshape(-1).cpu(), q=qpos.cpu(), k=None if kpos is None else kpos.cpu(),
                         logits=None if logits is None else logits.float().cpu(), rows=rows.cpu(),
                         scores=scores.cpu().clone()))

    prompts = cases.gen_prompts()
    n = len(prompts)
    resp, steps = [None] * n, [0] * n
    trace = []
    resp, ntok, nmax = generate_with_Flash_dLLM(
        model, [p.cuda() for p in prompts], list(cases.GEN_PROMPT_LENS), cases.GEN_BATCH, resp, steps,
        gen_length=cases.GEN_LEN[verify], verify=verify, min_keep=min_keep, record=record, trace=trace,
        **cases.GEN_KW)
    check_device_status()

    it = iter(recs)
    vocab = cases.GEN_CFG["vocab_size"]

    def replay(x_query, lengths, positions):
        r = next(it)
        v = bool(lengths[11])
        assert v == r["v"]
        assert torch.equal(x_query.reshape(-1), r["x"])
        assert torch.equal(positions[0].reshape(-1).to(torch.long), r["q"])
        if v:
            assert torch.equal(positions[1].reshape(-1).to(torch.long), r["k"])
        positions[4].copy_(r["scores"])
        out = torch.zeros(x_query.numel(), vocab)
        if r["logits"] is not None:
            out[r["rows"]] = r["logits"]
        return out

    class _L:  # layer stand-ins: the oracle loop only allocates caches on them
        pass

    o_resp, o_steps = [""] * n, [0] * n
    o_resp, o_ntok, o_nmax = do.generate(
        replay, [_L() for _ in range(3)], 3, cases.GEN_CFG["d_model"], cases.HEAD_DIM, cases.THETA, torch.float32,
        prompts, list(cases.GEN_PROMPT_LENS), cases.GEN_BATCH, o_resp, o_steps, gen_length=cases.GEN_LEN[verify],
        verify=verify, min_keep=min_keep, **cases.GEN_KW)
    assert next(it, None) is None, "product issued more forwards than the oracle"
    assert steps == o_steps
    assert (ntok, nmax) == (o_ntok, o_nmax)
    assert [list(r) for r in resp] == [[int(t) for t in s.split()] for s in o_resp]
    keeps = [k for t in trace for k in t["keep"].values()]
    assert max(keeps) >= 1 and len(trace) > 3
