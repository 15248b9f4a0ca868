"""Flash-Cache / Flash-Verify decode driver (``generate_with_Flash_dLLM``).

Same entry point, arguments and results as ``llada/generate.py:61-472``:
continuous batching over ``batch_size`` sequence slots, a masked window of
``block_length`` slots decoded by confidence (``threshold``), top-k selective
refresh of the ``track_num * block_length`` highest-attention decoded slots
plus ``mask_num - 1`` future windows, and with ``verify=True`` a second
forward that checks up to ``block_length // 2`` drafts against their
mask-view (acceptance prefix ``cumprod >= gamma``).

What differs is how a step is executed.  Per-sequence host loops with
``.item()`` syncs become batched device kernels (fp64 confidence
statistics, window acceptance, verify acceptance scan, refresh sort) with
one small device->host read per forward; the host keeps each sequence's
query and key slots as index ranges into the device's slot order and sends
one packed index array per forward; the LM head runs only on the
rows the step reads (masked rows; verify mask-view rows); KV caches are
zero-initialised.  Sorting ties resolve in index order (the reference's
``torch.sort`` is unstable).  Where the reference cannot continue -- a
verify step whose masked window is cut short by the end of the slot buffer
(generate.py:215 slices a full window and the assignment at :235 raises) --
the actual window length is used.

Forwards whose input shapes repeat are replayed as CUDA graphs.  The KV
caches, score buffer, RoPE tables and graphs live in a per-model session
(one per batch size / slot length), so a later call of the same shape zeroes
the caches and replays the graphs an earlier call captured.

``min_keep`` (default 1, the reference) forces a minimum number of accepted
tokens per step; ``trace`` (a list) receives the per-step decisions.
"""
from __future__ import annotations

from typing import Optional

import weakref

import numpy as np
import torch

from . import ops


def get_rotary_embedding(seq_len: int, dim: int, rope_theta: float, device=None):
    """RoPE tables (generate.py:44-50): fp32 (sin, cos) of shape (seq_len, dim)."""
    inv_freq = 1.0 / (rope_theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    seq = torch.arange(seq_len, device=device, dtype=torch.float32)
    freqs = torch.einsum("i , j -> i j", seq, inv_freq)
    pos = torch.cat((freqs, freqs), dim=-1)
    return pos.sin(), pos.cos()


def make_blocks(j: int, seqlen_k, max_length, start_m: int, end_m: int, block_m: int, device=None):
    """Block-table rows (seq, k_end, q_start, q_end) in ``block_m`` tiles (generate.py:52-58)."""
    q_starts = torch.arange(start_m, end_m, block_m, device=device)
    q_ends = q_starts + block_m
    q_ends[-1] = end_m
    return torch.stack((torch.full_like(q_starts, j), torch.full_like(q_starts, seqlen_k[j]), q_starts, q_ends), 1)


class _Forwarder:
    """Runs the model's forward passes.  A forward whose input shapes were
    seen before is captured into CUDA graphs (on its second occurrence, after
    an eager run of that same step sized the workspaces) and replayed from
    then on, with the step's inputs copied into the graph's static tensors.
    Forwards are pure functions of their inputs apart from the in-place cache
    and score updates, which the graph performs exactly like the eager call.

    A forward is captured as two graphs, split after layer ``split_after``:
    launching a graph of a few hundred kernels takes the host ~0.3 ms, during
    which the GPU would wait; the small first graph starts the GPU at once and
    the large second one is launched while it runs."""

    def __init__(self, enabled: bool, split_after: int = 2):
        self.enabled = enabled
        self.split_after = split_after
        self.seen = {}
        self.graphs = {}
        self.pool = None
        self.stream = None

    def __call__(self, key, inputs: dict, build):
        if not self.enabled:
            return build(inputs, None)
        hit = self.graphs.get(key)
        if hit is not None:
            static, graphs, out = hit
            for name, t in inputs.items():
                if t is not static[name]:  # (built in place by the caller: see static_inputs)
                    static[name].copy_(t)
            for graph in graphs:
                graph.replay()
            return out
        self.seen[key] = self.seen.get(key, 0) + 1
        if self.seen[key] < 2:
            return build(inputs, None)
        static = {name: t.clone() for name, t in inputs.items()}
        result = build(static, None)  # this step's real forward; also sizes workspaces
        # Capture on a side stream into one memory pool shared by all of this
        # generation's graphs.  (torch.cuda.graph would also run gc and empty
        # the allocator cache before every capture: ~0.5 s each.)
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
            self.stream = torch.cuda.Stream()
        graphs = [torch.cuda.CUDAGraph()]

        def split(block_idx: int) -> None:
            if block_idx == self.split_after:
                graphs[-1].capture_end()
                graphs.append(torch.cuda.CUDAGraph())
                graphs[-1].capture_begin(pool=self.pool)

        cur = torch.cuda.current_stream()
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            graphs[0].capture_begin(pool=self.pool)
            try:
                out = build(static, split)
            finally:
                graphs[-1].capture_end()
        cur.wait_stream(self.stream)
        self.graphs[key] = (static, graphs, out)
        return result


    def static_inputs(self, key):
        """The captured graph's input tensors for ``key`` (None before its
        capture): a caller may build a step's inputs straight into them."""
        hit = self.graphs.get(key) if self.enabled else None
        return None if hit is None else hit[0]


class _Staging:
    """Pinned host buffers for the host->device copies of a step's tables,
    reused across steps (pinning a fresh host tensor per copy costs a few
    hundred microseconds of host time while the GPU waits).  A ring of
    buffers; one is refilled only after the copy that last read it is done."""

    def __init__(self, n: int = 4):
        self.bufs = [None] * n
        self.events = [None] * n
        self.i = 0

    def send(self, t: torch.Tensor, dev) -> torch.Tensor:
        k = self.i
        self.i = (self.i + 1) % len(self.bufs)
        nbytes = t.numel() * t.element_size()
        if self.events[k] is not None:
            self.events[k].synchronize()
        buf = self.bufs[k]
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8).pin_memory()
            self.bufs[k] = buf
        staged = buf[:nbytes].view(t.dtype).view(t.shape)
        staged.copy_(t)
        out = staged.to(dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.events[k] = ev
        return out


class _Session:
    """Device state one model keeps between generate calls of the same shape
    (batch size, slot length, dtype, device): the per-layer KV caches, the
    attention-score buffer, the RoPE tables and the CUDA graphs of the
    forwards, which all reference these buffers.  A call zeroes the caches
    and scores instead of allocating them, so forwards captured by an earlier
    call replay unchanged."""

    def __init__(self, model, B: int, L: int, head_dim: int, use_graphs: bool):
        dev, cfg = model.device, model.config
        self.caches = [(torch.zeros((L * B, cfg.d_model), dtype=model.dtype, device=dev),
                        torch.zeros((L * B, cfg.d_model), dtype=model.dtype, device=dev))
                       for _ in model.model.transformer.blocks]
        self.attn_scores = torch.zeros(B * L, dtype=torch.float32, device=dev)
        sin, cos = get_rotary_embedding(L, head_dim, cfg.rope_theta, dev)
        self.rotary = [sin.repeat(B, 1).contiguous(), cos.repeat(B, 1).contiguous()]
        self.empty_i32 = torch.zeros(0, device=dev, dtype=torch.int32)
        self.empty_i64 = torch.zeros(0, device=dev, dtype=torch.int64)
        self.forward = _Forwarder(use_graphs and dev.type == "cuda")
        self.staging = _Staging() if dev.type == "cuda" else None

    def reset(self, model) -> None:
        for block, (kc, vc) in zip(model.model.transformer.blocks, self.caches):
            kc.zero_()
            vc.zero_()
            block.k_cache, block.v_cache = kc, vc
        self.attn_scores.zero_()


_SESSIONS = weakref.WeakKeyDictionary()


def _session(model, B: int, L: int, head_dim: int, use_graphs: bool) -> _Session:
    key = (B, L, model.dtype, str(model.device), use_graphs)
    held = _SESSIONS.get(model)
    if held is None or held[0] != key:
        held = (key, None)
        _SESSIONS[model] = held  # drop the previous shape's buffers first
        held = (key, _Session(model, B, L, head_dim, use_graphs))
        _SESSIONS[model] = held
    sess = held[1]
    sess.reset(model)
    return sess


class _Slots:
    """Host-side state of the sequence slots (the reference's per-slot lists).
    The masked and tracked query sets are position ranges of the slot's row
    of ``full_pos`` (the device-side slot order), gathered when a forward
    runs."""

    def __init__(self, b: int):
        self.active = [-1] * b
        self.nd = [0] * b
        self.pred = [0] * b
        self.eos = [-1] * b
        self.seqlen_k = [0] * b
        self.masked = [()] * b   # ((start, end),) positions of row j
        self.tracked = [()] * b  # ((start, end), ...)


class _Pack:
    """Host arrays sent to the device in one pinned copy; ``views`` returns
    the device tensors in the order they were added."""

    def __init__(self):
        self.parts = []

    def add(self, a) -> None:
        self.parts.append(np.ascontiguousarray(a, dtype=np.int64).reshape(-1))

    def send(self, h2d):
        sizes = [a.size for a in self.parts]
        flat = h2d(torch.from_numpy(np.concatenate(self.parts) if self.parts else np.zeros(0, np.int64)))
        out, o = [], 0
        for n in sizes:
            out.append(flat[o:o + n])
            o += n
        return out


@torch.no_grad()
def generate_with_Flash_dLLM(model, prompts, prompt_lengths, batch_size, responses, n_steps, steps=128,
                             gen_length=128, block_length=128, temperature=0., remasking='low_confidence',
                             mask_id=126336, threshold=0.9, gamma=0.9, track_num=4, mask_num=4, eos_id=126081,
                             verify=False, sliding_window=True, is_instruct=True, tokenizer=None, stop_tokens=None,
                             min_keep: int = 1, trace: Optional[list] = None, max_steps: Optional[int] = None,
                             step_hook=None, record=None, stats: Optional[dict] = None, use_graphs: bool = True):
    """Returns ``(responses, num_tokens, max_num_tokens)`` like the reference;
    ``responses[i]`` is the decoded text (token ids when ``tokenizer`` is
    None) and ``n_steps[i]`` counts the steps of prompt ``i``.  ``max_steps``
    stops early (benchmarking); ``step_hook(step)`` runs after each step;
    ``record(verify, x_query, query_pos, key_pos, logits, logit_rows,
    attn_scores)`` sees every forward (tests replay it through the oracle);
    ``stats`` (a dict) accumulates ``h2d_bytes`` / ``d2h_bytes`` / ``steps``;
    ``use_graphs`` replays repeated forward shapes as CUDA graphs."""
    dev = model.device
    cfg = model.config
    io = stats if stats is not None else {}
    io.setdefault("h2d_bytes", 0)
    io.setdefault("d2h_bytes", 0)
    io.setdefault("steps", 0)

    def h2d(t: torch.Tensor) -> torch.Tensor:
        io["h2d_bytes"] += t.numel() * t.element_size()
        if t.device.type != "cpu":
            return t
        staging = sess.staging
        return staging.send(t.contiguous(), dev) if staging is not None else t.to(dev)

    def d2h(t: torch.Tensor) -> list:
        io["d2h_bytes"] += t.numel() * t.element_size()
        return t.cpu().tolist()

    d_model, n_heads, n_layers = cfg.d_model, cfg.n_heads, cfg.n_layers
    head_dim = d_model // n_heads
    bm, bn = block_length, 128
    L = ((max(prompt_lengths) + gen_length + bm) // bn + 1) * bn
    B = batch_size
    stop_tokens = stop_tokens or []
    num_tokens = max_num_tokens = 0
    x = torch.full((B * L,), mask_id, dtype=torch.long, device=dev)
    x_draft = torch.full((B * L,), mask_id, dtype=torch.long, device=dev)
    full_pos = torch.arange(B * L, device=dev).reshape(B, L)
    sess = _session(model, B, L, head_dim, use_graphs)
    attn_scores = sess.attn_scores
    rotary_emb_pos = sess.rotary
    empty_i32, empty_i64 = sess.empty_i32, sess.empty_i64
    ar_L = torch.arange(L, device=dev)
    st = _Slots(B)
    forward = sess.forward
    count = 0
    start_layer = [-1] * B

    def load(j: int, i: int) -> None:
        p = prompt_lengths[i]
        x[j * L:(j + 1) * L] = mask_id
        prompt = h2d(prompts[i]) if prompts[i].device.type == "cpu" else prompts[i]
        x[j * L: j * L + p] = prompt
        x[j * L + p + gen_length:(j + 1) * L] = eos_id
        x_draft[j * L:(j + 1) * L] = mask_id
        x_draft[j * L: j * L + p] = prompt
        full_pos[j] = torch.arange(j * L, (j + 1) * L, device=dev)
        st.active[j] = i
        st.nd[j] = p
        st.pred[j] = p + gen_length + j * L
        st.eos[j] = -1
        st.seqlen_k[j] = (p + gen_length) // bn * bn + bn
        st.masked[j] = ((p, p + bm),)
        st.tracked[j] = ((0, p), (p + bm, max(st.seqlen_k[j], p + bm)))
        start_layer[j] = -1

    for j in range(B):
        if count < len(prompts):
            load(j, count)
            count += 1

    def refresh(cont_d, nd_cur_d) -> None:
        """Reorder each continuing sequence's decoded slots (those decoded
        before the step's last forward: ``nd_cur_d``) by ascending attention
        score, then clear the scores -- issued on the device before the
        step's decisions are read, so the host waits for it in the same read
        (generate.py:364-381)."""
        counts = torch.zeros(B, dtype=torch.int64, device=dev).index_copy_(0, act_d, nd_cur_d * cont_d)
        ops.refresh_sort(full_pos, counts, attn_scores)
        attn_scores.zero_()

    step = 0
    while True:
        act = [j for j in range(B) if st.active[j] != -1]
        if not act:
            break
        # ---------------------------------------------------- Flash-Cache --
        # per sequence: its slot row, k_end, nd, predicted length, the masked
        # range and the (up to two) tracked ranges as positions of its row of
        # full_pos, and its row / block-table tile offsets (masked rows of all
        # sequences first, then the tracked rows); the block tables, query
        # slots and tokens are built from these on the device
        # (fdllm_cache_build)
        na = len(act)
        seqtab = np.zeros((na, 16), np.int64)
        for k, j in enumerate(act):
            mr, tr = st.masked[j], st.tracked[j]
            seqtab[k, 0:4] = (j, st.seqlen_k[j], st.nd[j], st.pred[j])
            for c, (a, b) in zip((4, 6, 8), list(mr[:1]) + [(0, 0)] * (1 - len(mr[:1])) + list(tr[:2])
                                 + [(0, 0)] * (2 - len(tr[:2]))):
                seqtab[k, c:c + 2] = (a, max(0, b - a))
        m_n, t_n = seqtab[:, 5], seqtab[:, 7] + seqtab[:, 9]
        m_tl, t_tl = -(-m_n // bm), -(-t_n // bm)
        r_m, n_m = int(m_n.sum()), int(m_tl.sum())
        seqtab[:, 10] = np.cumsum(m_n) - m_n
        seqtab[:, 11] = r_m + np.cumsum(t_n) - t_n
        seqtab[:, 12] = np.cumsum(m_tl) - m_tl
        seqtab[:, 13] = n_m + np.cumsum(t_tl) - t_tl
        n_t = int(t_tl.sum())
        pk = _Pack()
        pk.add(seqtab)
        pk.add([1 if st.eos[j] != -1 else 0 for j in act])
        pk.add(act)
        pk.add(seqtab[:, 2])
        pk.add(seqtab[:, 3])
        seq_d, eos_known, act_d, nd_d, pred_d = pk.send(h2d)
        ckey = ("cache", r_m + int(t_n.sum()), n_m, n_t, r_m)
        st_in = forward.static_inputs(ckey)
        tables, query_pos_flat, x_query, seq_info = ops.cache_build(
            seq_d.view(-1, 16), r_m + int(t_n.sum()), n_m + n_t, bm, full_pos, x,
            out=None if st_in is None else (st_in["tables"], st_in["qpos"], st_in["x"]))
        eos_known = eos_known.to(torch.int32)

        def cache_forward(t, hook, n_m=n_m, r_m=r_m, has_t=n_t > 0):
            masked_blocks = t["tables"][:n_m] if n_m else empty_i32
            tracked_blocks = t["tables"][n_m:] if has_t else empty_i32
            positions = [t["qpos"], empty_i64, rotary_emb_pos, [], attn_scores, []]
            lengths = [start_layer, None, masked_blocks, tracked_blocks, t["tables"], st.active, n_m, L, bm, bn,
                       None, False]
            return _call_model(model, t["x"].unsqueeze(0), lengths, positions, r_m, hook)

        logits = forward(ckey,
                         {"x": x_query, "qpos": query_pos_flat, "tables": tables}, cache_forward)
        if record is not None:
            record(False, x_query, query_pos_flat, None, logits, torch.arange(r_m, device=dev), attn_scores)
        p_max, x0, _ = ops.row_stats(logits)
        keep_d, len_d, eos_d = ops.window_accept(p_max, x0, query_pos_flat[:r_m], seq_info, eos_known, L, threshold,
                                                 min_keep, eos_id, full_pos, x, x_draft if verify else None)
        parts = [keep_d.long(), len_d.long(), eos_d]
        if not verify:
            cont_d = _continues(full_pos, ar_L, act_d, nd_d, keep_d, pred_d, eos_known, eos_d)
            parts.append(cont_d)
            refresh(cont_d, nd_d)  # the step's last forward: refresh before the read
        host = d2h(torch.cat(parts))  # one device->host read
        keep1, lnum, eos1 = host[:na], host[na:2 * na], host[2 * na:3 * na]
        cont = host[3 * na:]
        for k, j in enumerate(act):
            st.nd[j] += keep1[k]
            if st.eos[j] == -1 and eos1[k] >= 0:
                st.eos[j] = eos1[k]
                st.pred[j] = eos1[k] + 1
        rec = {"keep": dict(zip(act, keep1))}

        # --------------------------------------------------- Flash-Verify --
        if verify:
            s_list = [min(max(lnum[k] - keep1[k], 0), bm // 2) for k in range(len(act))]
            # every sequence has 2*bm verify rows: t trailing decoded slots, its
            # s drafts, the same s slots again (mask view); keys are the rest
            # of its cache range
            # per sequence: its slot row, s drafts, decoded count, key range end,
            # predicted length and running key / draft offsets; the verify rows,
            # keys, mask and the acceptance rows are built from these on the
            # device (fdllm_verify_build)
            s_a = np.array(s_list, np.int64)
            t_a = 2 * bm - 2 * s_a
            nd_a = np.array([st.nd[j] for j in act], np.int64)
            sk_a = np.array([st.seqlen_k[j] for j in act], np.int64)
            nk = np.maximum(nd_a - t_a, 0) + np.maximum(sk_a - nd_a - s_a, 0)
            pred_a = np.array([st.pred[j] for j in act], np.int64)
            seqtab = np.stack([np.array(act, np.int64), s_a, nd_a, sk_a, pred_a, np.cumsum(nk) - nk,
                               np.cumsum(s_a) - s_a, np.zeros_like(s_a)], 1)
            pk = _Pack()
            pk.add(seqtab)
            pk.add([1 if st.eos[j] != -1 else 0 for j in act])
            pk.add(nd_a)
            pk.add(pred_a)
            seq_d, eos_known, nd_d, pred_d = pk.send(h2d)
            vkey = ("verify", na * 2 * bm, int(nk.sum()), na, int(s_a.sum()))
            st_in = forward.static_inputs(vkey) if sum(s_list) > 0 else None
            qpos, x_verify, attn_mask, key_pos_flat, draft_slots, lidx, vblocks, info2_d = ops.verify_build(
                seq_d.view(-1, 8), int(nk.sum()), int(s_a.sum()), bm, full_pos, x, x_draft,
                out=None if st_in is None else (st_in["qpos"], st_in["x"], st_in["mask"], st_in["kpos"],
                                                st_in["lidx"], st_in["vblocks"]))
            eos_known = eos_known.to(torch.int32)

            def verify_forward(t, hook, n_m=n_m):
                positions = [t["qpos"], t["kpos"], rotary_emb_pos, [], attn_scores, t["mask"]]
                lengths = [start_layer, t["vblocks"], None, empty_i32, None, st.active, n_m, L, bm, bn, None, True]
                return _call_model(model, t["x"].unsqueeze(0), lengths, positions, t["lidx"], hook)

            if sum(s_list) > 0:
                logits_v = forward(vkey,
                                   {"x": x_verify, "qpos": qpos, "kpos": key_pos_flat, "mask": attn_mask,
                                    "vblocks": vblocks, "lidx": lidx}, verify_forward)
                if record is not None:
                    record(True, x_verify, qpos, key_pos_flat, logits_v, lidx, attn_scores)
                draft_tok = x_draft[draft_slots]
                _, _, p_tok = ops.row_stats(logits_v, draft_tok)
            else:
                # No sequence has a draft to check: the verify forward would write
                # nothing (no cache, no scores) and none of its logits are read.
                if record is not None:
                    record(True, x_verify, qpos, key_pos_flat, None, lidx, attn_scores)
                draft_tok = draft_slots
                p_tok = torch.zeros(0, dtype=torch.float64, device=dev)
            keep2_d, eos2_d = ops.verify_accept(p_tok, draft_tok, draft_slots, info2_d, eos_known, gamma, eos_id, x)
            cont_d = _continues(full_pos, ar_L, act_d, nd_d, keep2_d, pred_d, eos_known, eos2_d)
            refresh(cont_d, nd_d)
            host = d2h(torch.cat([keep2_d.long(), eos2_d, cont_d]))
            keep2, eos2, cont = host[:na], host[na:2 * na], host[2 * na:]
            for k, j in enumerate(act):
                st.nd[j] += keep2[k]
                if st.eos[j] == -1 and eos2[k] >= 0:
                    st.eos[j] = eos2[k]
                    st.pred[j] = eos2[k] + 1
            rec.update(verify_s=dict(zip(act, s_list)), verify_keep=dict(zip(act, keep2)))

        for j in act:
            n_steps[st.active[j]] += 1

        # -------------------------------------------- refresh / finish --
        for k, j in enumerate(act):
            nd = st.nd[j]
            if cont[k]:
                # full_pos only changes again in the next step's acceptance,
                # after these ranges were gathered
                st.masked[j] = ((nd, min(nd + bm, L)),)
                if track_num < 0:
                    st.tracked[j] = ((0, nd), (min(nd + bm, L), max(st.seqlen_k[j], min(nd + bm, L))))
                else:
                    t0 = max(0, nd - track_num * bm)
                    t1 = min(st.seqlen_k[j], nd + bm * mask_num)
                    st.tracked[j] = ((t0, nd), (min(nd + bm, L), max(t1, min(nd + bm, L))))
                start_layer[j] = n_layers
            else:
                i = st.active[j]
                ids = d2h(x[j * L + prompt_lengths[i]: j * L + nd])
                if tokenizer is not None:
                    text = tokenizer.decode(ids, skip_special_tokens=False)
                    for stop_seq in stop_tokens:
                        if stop_seq in text:
                            text = text.split(stop_seq)[0]
                    ids2 = torch.tensor(tokenizer(text)["input_ids"])
                    responses[i] = tokenizer.decode(ids2, skip_special_tokens=True)
                else:
                    responses[i] = ids
                num_tokens += nd - prompt_lengths[i]
                max_num_tokens += gen_length
                if count < len(prompts):
                    load(j, count)
                    count += 1
                else:
                    st.active[j] = -1
                    st.masked[j] = ()
                    st.tracked[j] = ()
        if trace is not None:
            rec["nd"] = list(st.nd)
            trace.append(rec)
        step += 1
        io["steps"] += 1
        if step_hook is not None:
            step_hook(step)
        if max_steps is not None and step >= max_steps:
            break
    return responses, num_tokens, max_num_tokens


def _call_model(model, x, lengths, positions, logit_rows, hook):
    """The model's forward; ``hook`` (a graph-capture split) only reaches
    models whose forward takes ``layer_hook`` (this package's)."""
    kw = {"layer_hook": hook} if hook is not None else {}
    return model(x, use_cache=True, lengths=lengths, positions=positions, logit_rows=logit_rows, **kw).logits[0]


def _continues(full_pos, ar_L, act_d, nd_d, keep_d, pred_d, eos_known, eos_d) -> torch.Tensor:
    """Per active sequence (int64 0/1): does a slot before its predicted end
    remain undecoded after this forward's acceptance?  ``nd_d``/``pred_d``
    are the decoded count and predicted end before it; a newly found EOS
    moves the end to just after it."""
    nd = nd_d + keep_d.long()
    pred = torch.where((eos_known == 0) & (eos_d >= 0), eos_d + 1, pred_d)
    rows = full_pos.index_select(0, act_d)
    return ((ar_L[None, :] >= nd[:, None]) & (rows < pred[:, None])).any(1).long()


def _verify_mask(bm: int, s: int) -> np.ndarray:
    """(2bm, 2bm) bool verify mask for S drafts (generate.py:262-269)."""
    t = 2 * bm - 2 * s
    m = np.ones((2 * bm, 2 * bm), dtype=np.bool_)
    i = np.arange(s)
    m[:t, t:t + s] = False
    blk = np.block([[i[:, None] >= i[None, :], i[:, None] < i[None, :]],
                    [i[:, None] > i[None, :], i[:, None] <= i[None, :]]])
    m[t:t + 2 * s, t:t + 2 * s] = blk
    return m
