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


def _run(model, verify, min_keep, kw, record=None):
    from flash_dllm_b200.generate import generate_with_Flash_dLLM
    from flash_dllm_b200._lib import check_device_status
    prompts = cases.gen_prompts()
    n = len(prompts)
    resp, steps = [None] * n, [0] * n
    trace = []
    resp, ntok, nmax = generate_with_Flash_dLLM(
        model, [p.cuda() for p in prompts], list(cases.GEN_PROMPT_LENS), cases.GEN_BATCH, resp, steps,
        gen_length=cases.GEN_LEN[verify], verify=verify, min_keep=min_keep, record=record, trace=trace, **kw)
    check_device_status()
    return resp, steps, ntok, nmax, trace


@pytest.mark.parametrize("verify,min_keep,track_num", [(False, 1, 1), (True, 1, 1), (False, 2, 1), (False, 1, 2),
                                                       (True, 1, 2)])
def test_generate_replays_through_oracle(verify, min_keep, track_num):
    """track_num 2 is BASELINE config 5's refresh budget (2 blocks of decoded
    slots refreshed per step)."""
    model = _model()
    kw = dict(cases.GEN_KW, track_num=track_num)
    recs = []

    def record(v, xq, qpos, kpos, logits, rows, scores):
        recs.append(dict(v=v, x=xq.reshape(-1).cpu(), q=qpos.cpu(), k=None if kpos is None else kpos.cpu(),
                         logits=None if logits is None else logits.float().cpu(), rows=rows.cpu(),
                         scores=scores.cpu().clone()))

    prompts = cases.gen_prompts()
    n = len(prompts)
    resp, steps, ntok, nmax, trace = _run(model, verify, min_keep, kw, record)

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
        verify=verify, min_keep=min_keep, **kw)
    assert next(it, None) is None, "product issued more forwards than the oracle"
    assert steps == o_steps
    assert (ntok, nmax) == (o_ntok, o_nmax)
    assert [list(r) for r in resp] == [[int(t) for t in s.split()] for s in o_resp]
    keeps = [k for t in trace for k in t["keep"].values()]
    assert max(keeps) >= 1 and len(trace) > 3


@pytest.mark.parametrize("verify", [False, True])
def test_generate_is_reproducible(verify):
    """Two runs of the same prompts give the same trajectory: the attention
    scores that order the refresh are reduced in a fixed order, so every
    decision (and every forward's query set) repeats exactly."""
    model = _model()
    runs = []
    for _ in range(2):
        recs = []

        def record(v, xq, qpos, kpos, logits, rows, scores, recs=recs):
            recs.append((qpos.cpu(), scores.cpu().clone()))

        runs.append((_run(model, verify, 1, dict(cases.GEN_KW, track_num=2), record), recs))
    (r0, rec0), (r1, rec1) = runs
    assert [list(map(int, r)) for r in r0[0]] == [list(map(int, r)) for r in r1[0]]
    assert r0[1] == r1[1] and r0[2:4] == r1[2:4]
    assert len(rec0) == len(rec1)
    for (q0, s0), (q1, s1) in zip(rec0, rec1):
        assert torch.equal(q0, q1)
        assert torch.equal(s0, s1)
