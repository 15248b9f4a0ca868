"""CPU restatement of the reference decode driver ``generate_with_Flash_dLLM``.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Reference file: ``llada/generate.py`` (VILA-Lab/Flash-dLLM).  The reference
sorts with ``torch.sort`` (unstable on ties).  This restatement fixes the tie
order: every sort here is stable (ties keep their current order), which is
the order the CUDA kernels implement, so integer decisions can be compared
bit-exactly given identical scores.

The per-step decisions are split into small functions (each citing its
lines) so tests can drive them directly; :func:`generate` strings them
together exactly like the reference loop.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F


# ----------------------------------------------------------------- tables --

def get_rotary_embedding(seq_len: int, dim: int, rope_theta: float):
    """RoPE tables (generate.py:44-50): ``inv_freq = theta^(-2i/dim)``,
    ``freqs = [f, f]``; returns fp32 ``(sin, cos)`` of shape (seq_len, dim)."""
    inv_freq = 1.0 / (rope_theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    seq = torch.arange(seq_len, dtype=torch.float32)
    freqs = torch.einsum("i , j -> i j", seq, inv_freq)
    pos = torch.cat((freqs, freqs), dim=-1)
    return pos.sin(), pos.cos()


def make_blocks(j: int, seqlen_k: Sequence[int], start_m: int, end_m: int, block_m: int) -> torch.Tensor:
    """Block-table rows ``(seq, k_end, q_start, q_end)`` covering query rows
    ``[start_m, end_m)`` in ``block_m`` tiles (generate.py:52-58)."""
    q_starts = torch.arange(start_m, end_m, block_m)
    q_ends = q_starts + block_m
    q_ends[-1] = end_m
    return torch.stack((torch.full_like(q_starts, j), torch.full_like(q_starts, seqlen_k[j]),
                        q_starts, q_ends), dim=1)


def build_block_tables(masked_counts: Sequence[int], tracked_counts: Sequence[int],
                       seqlen_k: Sequence[int], block_m: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """All masked tiles (sequence order) then all tracked tiles, in one flat
    query-row space (generate.py:146-163, 439-465).  Empty tables are int32
    ``tensor([])`` like the reference's ``empty_int32``."""
    acc = 0
    masked, tracked = [], []
    for j, n in enumerate(masked_counts):
        if n > 0:
            masked.append(make_blocks(j, seqlen_k, acc, acc + n, block_m))
            acc += n
    for j, n in enumerate(tracked_counts):
        if n > 0:
            tracked.append(make_blocks(j, seqlen_k, acc, acc + n, block_m))
            acc += n
    empty = torch.tensor([], dtype=torch.int32)
    return (torch.cat(masked) if masked else empty), (torch.cat(tracked) if tracked else empty)


# -------------------------------------------------------------- decisions --

def confidence(logits: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp64 softmax over the vocabulary, then (max prob, argmax)
    (generate.py:218-219, 337-338).  Ties in the maximum resolve to the
    lowest token id."""
    p = F.softmax(logits.to(torch.float64), dim=-1)
    pmax = p.max(dim=-1).values
    first = (p == pmax[:, None]).to(torch.int8).argmax(dim=-1)
    return pmax, first


def token_prob(logits: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    """fp64 softmax probability of ``tokens[i]`` in row ``i``
    (generate.py:320-321)."""
    p = F.softmax(logits.to(torch.float64), dim=-1)
    return p.gather(1, tokens.view(-1, 1).to(torch.long)).view(-1)


def sort_desc_stable(x: torch.Tensor) -> torch.Tensor:
    """Descending order, ties keep index order (the reference's
    ``x.sort(descending=True)`` at generate.py:230, 343 with ties fixed)."""
    return torch.sort(x, descending=True, stable=True).indices


def accept_count(p: torch.Tensor, threshold: float, min_keep: int = 1) -> int:
    """``keep = max(#(p >= threshold), 1)`` (generate.py:231-233, 344-346).
    ``min_keep`` > 1 is the forced-accept harness knob (not a reference
    feature); a forced count never exceeds the window (with ``min_keep`` = 1
    and a non-empty window the clamp never applies)."""
    return min(max(int((p >= threshold).sum()), min_keep), p.numel())


def verify_keep(p_draft: torch.Tensor, gamma: float) -> int:
    """Prefix acceptance ``#(cumprod(p) >= gamma)`` (generate.py:326-328)."""
    if p_draft.numel() == 0:
        return 0
    return int((p_draft.cumprod(dim=0) >= gamma).sum())


def verify_split(length_num: int, keep_num: int, block_m: int) -> Tuple[int, int]:
    """``S = min(max(length_num - keep, 0), bm//2)`` drafts and
    ``T = 2*bm - 2*S`` tracked rows (generate.py:254-258)."""
    s = min(max(length_num - keep_num, 0), block_m // 2)
    return s, 2 * block_m - 2 * s


def verify_mask(block_m: int, s: int) -> torch.Tensor:
    """The (2bm, 2bm) boolean verify mask (generate.py:262-269): tracked rows
    see no drafts; draft x draft ``i>=j``; draft -> mask-view ``i<j``;
    mask-view -> draft ``i>j``; mask-view x mask-view ``i<=j``."""
    t = 2 * block_m - 2 * s
    m = torch.ones((2 * block_m, 2 * block_m), dtype=torch.bool)
    i = torch.arange(s)
    m11 = i.view(-1, 1) >= i.view(1, -1)
    m12 = i.view(-1, 1) < i.view(1, -1)
    m21 = i.view(-1, 1) > i.view(1, -1)
    m22 = i.view(-1, 1) <= i.view(1, -1)
    m[:t, t:t + s] = False
    m[t:t + 2 * s, t:t + 2 * s] = torch.cat([torch.cat([m11, m12], 1), torch.cat([m21, m22], 1)], 0)
    return m


def refresh_order(scores: torch.Tensor) -> torch.Tensor:
    """Ascending stable order of decoded slots by attention score
    (generate.py:365)."""
    return torch.sort(scores, descending=False, stable=True).indices


def tracked_slots(full_pos_j: torch.Tensor, nd: int, block_m: int, seqlen_k: int,
                  track_num: int, mask_num: int) -> torch.Tensor:
    """Refresh rows for the next step (generate.py:368-381)."""
    if track_num < 0:
        return torch.cat([full_pos_j[:nd], full_pos_j[nd + block_m: seqlen_k]])
    t0 = max(0, nd - track_num * block_m)
    t1 = min(seqlen_k, nd + block_m * mask_num)
    return torch.cat([full_pos_j[t0:nd], full_pos_j[nd + block_m: t1]])


# ------------------------------------------------------------------ loop --

class StubTokenizer:
    """Identity tokenizer for the finish path (generate.py:387-394)."""

    def decode(self, ids, skip_special_tokens=False):
        return " ".join(str(int(i)) for i in ids)

    def __call__(self, text):
        return {"input_ids": [int(t) for t in text.split()]}


ForwardFn = Callable[[torch.Tensor, List, List], torch.Tensor]


@torch.no_grad()
def generate(forward: ForwardFn, layers: Sequence, n_layers: int, d_model: int, head_dim: int,
             rope_theta: float, cache_dtype, prompts, prompt_lengths, batch_size, responses, n_steps,
             gen_length=128, block_length=128, mask_id=126336, threshold=0.9, gamma=0.9,
             track_num=4, mask_num=4, eos_id=126081, verify=False, tokenizer=None, stop_tokens=None,
             min_keep: int = 1, trace: Optional[list] = None):
    """Restatement of ``generate_with_Flash_dLLM`` (generate.py:61-472).

    ``forward(x_query (1,Nq) long, lengths, positions) -> logits (Nq, V)``
    runs the model; ``layers`` are the per-layer objects whose ``k_cache`` /
    ``v_cache`` attributes this function allocates (generate.py:178-180).
    Returns ``(responses, num_tokens, max_num_tokens)``; ``n_steps`` is
    updated in place.  ``trace`` (a list) receives one dict per step with the
    integer decisions, for golden comparisons.
    """
    tokenizer = tokenizer or StubTokenizer()
    stop_tokens = stop_tokens or []
    block_m = block_length
    block_n = 128
    max_length = max(prompt_lengths) + gen_length + block_m
    max_length = (max_length // block_n + 1) * block_n
    num_tokens = 0
    max_num_tokens = 0
    info: list = []
    empty_int32 = torch.tensor([], dtype=torch.int32)
    count = 0
    x = torch.full((batch_size * max_length,), mask_id, dtype=torch.long)
    x_draft = torch.full((batch_size * max_length,), mask_id, dtype=torch.long)
    full_pos = torch.arange(batch_size * max_length).reshape(batch_size, max_length)
    attn_scores = torch.zeros((batch_size * max_length,), dtype=torch.float32)
    num_decoded, query_masked_pos, query_tracked_pos, query_verify_pos = [], [], [], []
    predicted_length, decoded_eos_pos, start_layer, active_batch = [], [], [], []
    seqlen_keep, seqlen_k = [], []

    for j in range(batch_size):
        x[j * max_length: j * max_length + prompt_lengths[count]] = prompts[count]
        x_draft[j * max_length: j * max_length + prompt_lengths[count]] = prompts[count]
        x[j * max_length + prompt_lengths[count] + gen_length: (j + 1) * max_length] = eos_id
        seqlen_k.append((prompt_lengths[count] + gen_length) // block_n * block_n + block_n)
        num_decoded.append(prompt_lengths[count])
        query_masked_pos.append(full_pos[j, num_decoded[j]: num_decoded[j] + block_m])
        query_tracked_pos.append(torch.cat([full_pos[j, :num_decoded[j]],
                                            full_pos[j, num_decoded[j] + block_m: seqlen_k[j]]]))
        predicted_length.append(num_decoded[j] + gen_length + j * max_length)
        decoded_eos_pos.append(-1)
        start_layer.append(-1)
        active_batch.append(count)
        query_verify_pos.append(empty_int32)
        seqlen_keep.append(0)
        count += 1

    def tables():
        return build_block_tables([p.shape[0] for p in query_masked_pos],
                                  [p.shape[0] for p in query_tracked_pos], seqlen_k, block_m)

    query_masked_blocks, query_tracked_blocks = tables()
    num_active = query_masked_blocks.shape[0]
    query_pos_flat = torch.cat(query_masked_pos + query_tracked_pos)
    x_query = x[query_pos_flat].unsqueeze(0)
    key_pos_flat = empty_int32
    attn_mask: list = []
    pos_sin, pos_cos = get_rotary_embedding(max_length, head_dim, rope_theta)
    rotary_emb_pos = [pos_sin.repeat(batch_size, 1), pos_cos.repeat(batch_size, 1)]
    for layer in layers:
        layer.k_cache = torch.zeros((max_length * batch_size, d_model), dtype=cache_dtype)
        layer.v_cache = torch.zeros((max_length * batch_size, d_model), dtype=cache_dtype)

    num_verify = 0
    while True:
        step = {"keep": [], "verify_s": [], "full_pos": None}
        query_blocks = torch.cat([query_masked_blocks, query_tracked_blocks], dim=0)
        positions = [query_pos_flat, key_pos_flat, rotary_emb_pos, info, attn_scores, attn_mask]
        lengths = [start_layer, None, query_masked_blocks, query_tracked_blocks, query_blocks,
                   active_batch, num_active, max_length, block_m, block_n, None, False]
        logits = forward(x_query, lengths, positions)
        x_query = x_query.squeeze(0)
        acc_seqlen_masked = 0
        x_verify, key_pos_flat, attn_mask, query_verify_blocks = [], [], [], []
        acc_q = acc_k = 0

        if verify:
            for j, i in enumerate(active_batch):
                if i == -1:
                    continue
                # The reference slices ``block_m`` rows here (generate.py:215) and then
                # fails on a shape mismatch when the window is cut short by the end of
                # the slot buffer; the actual window length is used instead.
                query_masked_pos[j] = query_masked_pos[j][:block_m]
                logits_j = logits[acc_seqlen_masked: acc_seqlen_masked + query_masked_pos[j].shape[0]]
                acc_seqlen_masked += query_masked_pos[j].shape[0]
                x0_p, x0 = confidence(logits_j)
                if decoded_eos_pos[j] != -1:
                    length_mask = query_masked_pos[j] >= predicted_length[j]
                    x0_p[length_mask] = 0
                    length_num = query_masked_pos[j].shape[0] - int(length_mask.sum())
                else:
                    length_num = query_masked_pos[j].shape[0]
                sorted_idx = sort_desc_stable(x0_p)
                keep_num = accept_count(x0_p, threshold, min_keep)
                x_draft[query_masked_pos[j]] = x0
                nd = num_decoded[j]
                full_pos[j, nd: nd + query_masked_pos[j].shape[0]] = query_masked_pos[j][sorted_idx]
                pos_new = full_pos[j, nd: nd + keep_num]
                tok_new = x0[sorted_idx][:keep_num]
                x[pos_new] = tok_new
                num_decoded[j] += keep_num
                if decoded_eos_pos[j] == -1:
                    pos_eos = pos_new[tok_new.eq(eos_id)]
                    if pos_eos.shape[0] > 0:
                        decoded_eos_pos[j] = int(pos_eos.max())
                        predicted_length[j] = decoded_eos_pos[j] + 1
                s, t = verify_split(length_num, keep_num, block_m)
                num_verify = s
                seqlen_keep[j] = t
                step["verify_s"].append((j, keep_num, s))
                attn_mask.append(verify_mask(block_m, s))
                nd = num_decoded[j]
                drafts = full_pos[j, nd: nd + s]
                tracked = full_pos[j, nd - t: nd]
                x_verify.append(torch.cat([x[tracked], x_draft[drafts], x[drafts]]))
                query_verify_pos[j] = torch.cat([tracked, drafts, drafts])
                key_pos_flat.append(torch.cat([full_pos[j, :nd - t], full_pos[j, nd + s: seqlen_k[j]]]))
                query_verify_blocks.append((acc_k, acc_k + key_pos_flat[-1].shape[0],
                                            acc_q, acc_q + query_verify_pos[j].shape[0]))
                acc_q += query_verify_pos[j].shape[0]
                acc_k += key_pos_flat[-1].shape[0]
            query_verify_blocks = torch.tensor(query_verify_blocks, dtype=torch.int32)
            attn_mask = torch.cat(attn_mask, dim=0)
            query_pos_flat = torch.cat(query_verify_pos)
            key_pos_flat = torch.cat(key_pos_flat)
            x_query = torch.cat(x_verify).unsqueeze(0)
            positions = [query_pos_flat, key_pos_flat, rotary_emb_pos, info, attn_scores, attn_mask]
            lengths = [start_layer, query_verify_blocks, None, query_tracked_blocks, None, active_batch,
                       num_active, max_length, block_m, block_n, None, True]
            logits = forward(x_query, lengths, positions)
            x_query = x_query.squeeze(0)

        acc_verify = 0
        for j, i in enumerate(active_batch):
            if i == -1:
                continue
            n_steps[i] += 1
            if verify:
                t = seqlen_keep[j]
                s = (block_m * 2 - t) // 2
                if s == 0:
                    keep_num = 0
                else:
                    logits_v = logits[acc_verify + t + s: acc_verify + t + 2 * s]
                    x_v = x_query[acc_verify + t: acc_verify + t + s]
                    p_v = token_prob(logits_v, x_v)
                    if decoded_eos_pos[j] != -1:
                        p_v[query_pos_flat[acc_verify + t: acc_verify + t + s] >= predicted_length[j]] = 0
                    keep_num = verify_keep(p_v, gamma)
                    pos_new = full_pos[j, num_decoded[j]: num_decoded[j] + keep_num]
                    tok_new = x_v[:keep_num]
                acc_verify += query_verify_pos[j].shape[0]
            else:
                logits_j = logits[acc_seqlen_masked + num_verify:
                                  acc_seqlen_masked + num_verify + query_masked_pos[j].shape[0]]
                acc_seqlen_masked += query_masked_pos[j].shape[0]
                x0_p, x0 = confidence(logits_j)
                if decoded_eos_pos[j] != -1:
                    x0_p[query_masked_pos[j] >= predicted_length[j]] = 0
                sorted_idx = sort_desc_stable(x0_p)
                keep_num = accept_count(x0_p, threshold, min_keep)
                nd = num_decoded[j]
                full_pos[j, nd: nd + query_masked_pos[j].shape[0]] = query_masked_pos[j][sorted_idx]
                pos_new = full_pos[j, nd: nd + keep_num]
                tok_new = x0[sorted_idx][:keep_num]
            step["keep"].append((j, keep_num))
            if keep_num > 0:
                x[pos_new] = tok_new
                num_decoded[j] += keep_num
                if decoded_eos_pos[j] == -1:
                    pos_eos = pos_new[tok_new.eq(eos_id)]
                    if pos_eos.shape[0] > 0:
                        decoded_eos_pos[j] = int(pos_eos.max())
                        predicted_length[j] = decoded_eos_pos[j] + 1

            nd = num_decoded[j]
            if bool((full_pos[j, nd:] < predicted_length[j]).any()):
                head = full_pos[j, :nd - keep_num]
                order = refresh_order(attn_scores[head])
                full_pos[j, :nd - keep_num] = head[order]
                query_masked_pos[j] = full_pos[j, nd: nd + block_m]
                query_tracked_pos[j] = tracked_slots(full_pos[j], nd, block_m, seqlen_k[j],
                                                     track_num, mask_num)
                start_layer[j] = n_layers
            else:
                ids = x[j * max_length + prompt_lengths[i]: j * max_length + nd]
                text = tokenizer.decode(ids, skip_special_tokens=False)
                for stop_seq in stop_tokens:
                    if stop_seq in text:
                        text = text.split(stop_seq)[0]
                ids = torch.tensor(tokenizer(text)["input_ids"])
                text = tokenizer.decode(ids, skip_special_tokens=True)
                num_tokens += nd - prompt_lengths[i]
                max_num_tokens += gen_length
                responses[i] = text
                if count < len(prompts):
                    active_batch[j] = count
                    x[j * max_length:(j + 1) * max_length] = mask_id
                    x[j * max_length: j * max_length + prompt_lengths[count]] = prompts[count]
                    x[j * max_length + prompt_lengths[count] + gen_length:(j + 1) * max_length] = eos_id
                    seqlen_k[j] = (prompt_lengths[count] + gen_length) // block_n * block_n + block_n
                    x_draft[j * max_length:(j + 1) * max_length] = mask_id
                    x_draft[j * max_length: j * max_length + prompt_lengths[count]] = prompts[count]
                    num_decoded[j] = prompt_lengths[count]
                    full_pos[j] = torch.arange(j * max_length, (j + 1) * max_length)
                    query_verify_pos[j] = empty_int32
                    query_masked_pos[j] = full_pos[j, num_decoded[j]: num_decoded[j] + block_m]
                    query_tracked_pos[j] = torch.cat([full_pos[j, :num_decoded[j]],
                                                      full_pos[j, num_decoded[j] + block_m: seqlen_k[j]]])
                    predicted_length[j] = num_decoded[j] + gen_length + j * max_length
                    start_layer[j] = -1
                    decoded_eos_pos[j] = -1
                    count += 1
                else:
                    active_batch[j] = -1
                    query_masked_pos[j] = empty_int32
                    query_tracked_pos[j] = empty_int32
                    query_verify_pos[j] = empty_int32

        if trace is not None:
            step["full_pos"] = full_pos.clone()
            step["num_decoded"] = list(num_decoded)
            trace.append(step)
        if sum(active_batch) == -batch_size:
            break
        query_masked_blocks, query_tracked_blocks = tables()
        num_active = query_masked_blocks.shape[0]
        query_pos_flat = torch.cat(query_masked_pos + query_tracked_pos)
        x_query = x[query_pos_flat].unsqueeze(0)
        attn_scores.fill_(0)

    return responses, num_tokens, max_num_tokens
