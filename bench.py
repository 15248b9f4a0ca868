"""Benchmark: generated tokens/s of Flash-Cache + Flash-Verify decoding of a
random-init LLaDA-8B (batch 8 synthetic 256-token prompts,
gen 512, block 32, threshold 0.9, gamma 0.8, refresh budget 32 = track_num 1 /
mask_num 1), sequence-sharded over N GPUs of one node (one process per GPU,
no collective on the hot path; NCCL only gathers the counters).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

A step is one decode iteration on every rank: the Flash-Cache forward, the
Flash-Verify forward and the bookkeeping kernels for that rank's sequences.
``value`` = tokens committed by all ranks during the K timed steps / max
over ranks of their CUDA-event time (weights, caches and prompts already in
HBM; W warm-up steps first, the first being the prefill).  ``e2e`` = one full
``generate_with_Flash_dLLM`` call per rank from pinned host prompts to host
responses (every step's table uploads and decision reads included), tokens
counted like the reference (generate.py:396).  ``roofline`` covers the fused
QKV + RoPE + cache-scatter kernel at the per-GPU step shape, timed live with
CUDA events; ``kernels`` lists the other hot kernels' times the same way.
``--impl reference`` times the reference algorithm's CPU restatement
(``oracle/``) on the host cores on a bounded sample of the same step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "generated tokens/s (LLaDA-8B, gen 512) at 1/2/4/8 B200; fused-layer us & HBM GB/s"
WORKLOAD = dict(workload="llada8b_flash_cache_verify_decode", model="LLaDA-8B (random init N(0,0.02))",
                global_batch=8, prompt_len=256, gen_length=512, block_length=32, threshold=0.9, gamma=0.8,
                track_num=1, mask_num=1, seq_len=896)
GEN_KW = dict(gen_length=512, block_length=32, threshold=0.9, gamma=0.8, track_num=1, mask_num=1,
              mask_id=126336, eos_id=126081, verify=True)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def _prompts(n, vocab, mask_id, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        p = torch.randint(0, vocab - 1, (WORKLOAD["prompt_len"],), generator=g)
        p[p >= mask_id] += 1  # uniform over the vocabulary without the mask id
        out.append(p)
    return out


class _Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        def run():
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            while not self._stop.is_set():
                try:
                    r = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                        "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                    if r.returncode == 0 and r.stdout.strip():
                        self.samples.append([v.strip() for v in r.stdout.strip().split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 3 + i and
                          s[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def _time_kernels(model, n_rows, batch, lmax, dev):
    """CUDA-event times of the hot kernels at the per-GPU step shape (layer 0
    weights, synthetic activations, inputs >> L2 via the weights)."""
    from flash_dllm_b200 import ops
    blk = model.model.transformer.blocks[0]
    d = model.config.d_model
    H = model.config.n_heads
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(n_rows, d, device=dev, generator=g).to(torch.bfloat16)
    pos = torch.stack([torch.randperm(lmax, device=dev, generator=g)[:n_rows // batch] + j * lmax
                       for j in range(batch)]).reshape(-1)
    kc = torch.randn(batch * lmax, d, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    from flash_dllm_b200.generate import get_rotary_embedding
    sin, cos = get_rotary_embedding(lmax, 128, model.config.rope_theta, dev)
    sin, cos = sin.repeat(batch, 1).contiguous(), cos.repeat(batch, 1).contiguous()
    q = torch.empty_like(x)
    att = torch.empty_like(x)
    bm = 32
    per = n_rows // batch
    mrows = [(j, lmax, j * bm, (j + 1) * bm) for j in range(batch)]
    trows = []
    for j in range(batch):
        s0 = batch * bm + j * (per - bm)
        for s in range(s0, s0 + per - bm, bm):
            trows.append((j, lmax, s, min(s + bm, s0 + per - bm)))
    mb = torch.tensor(mrows, dtype=torch.int64, device=dev)
    tb = torch.tensor(trows, dtype=torch.int64, device=dev).reshape(-1, 4)
    plan, cap = ops.plan_cache_attention(mb, tb, n_rows, batch, bm, lmax, dev)
    scores = torch.zeros(batch * lmax, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > L2, rewritten between launches

    def timed(fn, reps=int(os.environ.get("BENCH_KERNEL_REPS", "10"))):
        ts = []
        for _ in range(reps + 2):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b) * 1e-3)
        return float(np.mean(ts[2:]))

    t_qkv = timed(lambda: ops.qkv_rope_cache(x, blk.q_proj.weight, blk.k_proj.weight, blk.v_proj.weight, pos, sin,
                                             cos, q, kc, vc, H))
    t_attn = timed(lambda: ops.attn_cache(q, att, kc, vc, plan, cap, scores, 1.0 / (bm * H), H, lmax,
                                          128 ** -0.5))
    t_norm = timed(lambda: ops.rmsnorm(x, blk.attn_norm.weight, 1e-5))
    # Flash-Verify attention at the steady-state verify shape: per sequence 16
    # drafts (2*bm rows: 32 trailing + 16 drafts twice), keys = the cache minus
    # the block's own rows, the reference's verify mask
    from flash_dllm_b200.generate import _verify_mask
    s_d, t_d = 16, 2 * bm - 2 * 16
    nd = lmax // 2
    kparts, vrows, acc_k = [], [], 0
    for j in range(batch):
        kp = torch.cat([torch.arange(j * lmax, j * lmax + nd - t_d), torch.arange(j * lmax + nd + s_d, (j + 1) * lmax)])
        kparts.append(kp)
        vrows.append((acc_k, acc_k + kp.numel(), j * 2 * bm, (j + 1) * 2 * bm))
        acc_k += kp.numel()
    kpos = torch.cat(kparts).to(dev)
    vblocks = torch.tensor(vrows, dtype=torch.int32, device=dev)
    vmask = torch.from_numpy(np.concatenate([_verify_mask(bm, s_d)] * batch)).to(dev)
    k1 = torch.randn(batch * 2 * bm, d, device=dev, generator=g).to(torch.bfloat16)
    v1 = torch.randn_like(k1)
    qv = torch.randn_like(k1)
    ov = torch.empty_like(k1)
    t_vattn = timed(lambda: ops.verify_attn(qv, k1, v1, ov, kc, vc, kpos, vmask, vblocks, 2 * bm, H, 128 ** -0.5,
                                            max_keys=lmax))
    qkv_bytes = 3 * d * d * 2 + n_rows * d * 2 * 4 + n_rows * 8 + n_rows * 128 * 4 * 2
    qkv_flops = 2.0 * n_rows * d * 3 * d
    attn_bytes = batch * lmax * d * 2 * 2 + n_rows * d * 2 * 2 + batch * lmax * 4 * 2
    attn_flops = 4.0 * n_rows * lmax * d
    # algorithmic bytes: every sequence's gathered cache K/V rows and its 2*bm own K/V rows read once, Q read
    # and O written once
    vattn_bytes = (acc_k + batch * 2 * bm) * d * 2 * 2 + batch * 2 * bm * d * 2 * 2
    return dict(qkv_s=t_qkv, attn_s=t_attn, norm_s=t_norm, vattn_s=t_vattn, qkv_bytes=qkv_bytes, qkv_flops=qkv_flops,
                attn_bytes=attn_bytes, attn_flops=attn_flops, vattn_bytes=vattn_bytes, rows=n_rows)


def _cpu_reference(sample_layers: int = 1, vocab_slice: int = 8192):
    """Reference algorithm (CPU restatement in oracle/) on the host cores: one
    steady-state decode step of config 4 on one sequence-batch of 8, timed on
    `sample_layers` of 32 layers and a `vocab_slice` of the LM head, scaled to
    the full model; tokens per step from the oracle's own acceptance."""
    from oracle import decode_oracle as do
    from oracle import flash_cache_oracle as fco
    from oracle import tiny_model as tm
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    d, H, hid, V, B, bm, L = 4096, 32, 12288, 126464, 8, 32, 896
    g = torch.Generator().manual_seed(0)
    tc = tm.TinyConfig(d_model=d, n_heads=H, n_layers=1, mlp_hidden_size=hid, vocab_size=8, init_std=0.02)
    blk = tm.TinyLLaDA(tc, tm.make_weights(tc, 0)).layers[0]
    blk.k_cache = torch.randn(B * L, d, generator=g)
    blk.v_cache = torch.randn(B * L, d, generator=g)
    sin, cos = do.get_rotary_embedding(L, 128, 500000.0)
    rot = [sin.repeat(B, 1), cos.repeat(B, 1)]
    masked = [torch.arange(j * L + 400, j * L + 432) for j in range(B)]
    tracked = [torch.arange(j * L + 368, j * L + 400) for j in range(B)]
    mb, tb = do.build_block_tables([bm] * B, [bm] * B, [L] * B, bm)
    qpos = torch.cat(masked + tracked)
    x = torch.randn(qpos.numel(), d, generator=g)
    scores = torch.zeros(B * L)
    head = torch.randn(vocab_slice, d, generator=g) * 0.02
    t0 = time.perf_counter()
    lengths = [[-1] * B, None, mb, tb, torch.cat([mb, tb]), list(range(B)), B, L, bm, 128, None, False]
    positions = [qpos, torch.tensor([], dtype=torch.int64), rot, [], scores, []]
    for _ in range(sample_layers):
        y = fco.flash_fused_elastic_cache(blk, x, 2, positions, lengths).squeeze(0)
    t_cache = (time.perf_counter() - t0) / sample_layers
    s_list = [16] * B
    vq = torch.cat([torch.arange(j * L + 336, j * L + 400) for j in range(B)])
    kp = torch.cat([torch.cat([torch.arange(j * L, j * L + 336), torch.arange(j * L + 416, j * L + L)])
                    for j in range(B)])
    nk = kp.numel() // B
    vb = torch.tensor([(j * nk, (j + 1) * nk, j * 64, (j + 1) * 64) for j in range(B)], dtype=torch.int32)
    mask = torch.cat([do.verify_mask(bm, s) for s in s_list])
    t0 = time.perf_counter()
    lengths_v = [[-1] * B, vb, None, tb, None, list(range(B)), B, L, bm, 128, None, True]
    positions_v = [vq, kp, rot, [], scores, mask]
    for _ in range(sample_layers):
        yv = fco.flash_fused_elastic_cache(blk, torch.randn(vq.numel(), d, generator=g), 2, positions_v,
                                           lengths_v).squeeze(0)
    t_verify = (time.perf_counter() - t0) / sample_layers
    t0 = time.perf_counter()
    lc = y[:B * bm] @ head.T
    lv = yv[:B * 16] @ head.T
    t_head = (time.perf_counter() - t0) * (V / vocab_slice)
    # decisions on full-width logits (slice tiled to the vocabulary width)
    t0 = time.perf_counter()
    full_c = lc.repeat(1, math.ceil(V / vocab_slice))[:, :V]
    full_v = lv.repeat(1, math.ceil(V / vocab_slice))[:, :V]
    keeps = 0
    for j in range(B):
        p, _ = do.confidence(full_c[j * bm:(j + 1) * bm])
        keeps += do.accept_count(p, 0.9)
        pv = do.token_prob(full_v[j * 16:(j + 1) * 16], torch.zeros(16, dtype=torch.long))
        keeps += do.verify_keep(pv, 0.8)
        do.refresh_order(scores[torch.arange(j * L, j * L + 400)])
    t_dec = time.perf_counter() - t0
    step_s = 32 * (t_cache + t_verify) + t_head + t_dec
    sample = (f"one steady-state step of config 4 (8 seqs x 64 query rows, 896-slot caches, both forwards): "
              f"{sample_layers} of 32 layers timed and scaled x32, LM head on a {vocab_slice}-row vocabulary slice "
              f"scaled to 126464, fp64 decisions on full-width rows; {keeps} tokens committed")
    return keeps / step_s, threads, sample, step_s


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args):
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return
    vals = []
    sample = threads = None
    for i in range(args.warmup + args.steps):
        v, threads, sample, _ = _cpu_reference()
        if i >= args.warmup:
            vals.append(v)
    value = float(np.mean(vals))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * 8 / value if value else None,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": dict(WORKLOAD, parallelism="cpu"),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--kernels-only", type=int, default=0, metavar="SEQS",
                    help="time only the hot kernels of one random LLaDA-8B layer at the step shape of SEQS "
                         "sequences per GPU (small case for ncu captures)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.kernels_only:
        return run_kernels_only(args.kernels_only)
    assert args.warmup >= 3, "at least 3 warm-up steps"
    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from flash_dllm_b200 import LLaDAConfigB200, LLaDAModelB200, generate_with_Flash_dLLM
    import flash_dllm_b200._lib as L
    cfg = LLaDAConfigB200()
    model = LLaDAModelB200.random_init(cfg, device=dev, seed=0)
    prompts = _prompts(WORKLOAD["global_batch"], cfg.vocab_size, cfg.mask_token_id)
    from flash_dllm_b200.shard import reduce_counters, shard_range
    s0, s1 = shard_range(WORKLOAD["global_batch"], rank, world)
    mine = prompts[s0:s1]
    per = len(mine)
    dist = None
    if world > 1:
        import torch.distributed as dist

    # ------------------------------------------------ device-resident steps --
    trace = []
    ev = {}
    clocks = _Clocks(local)

    def hook(step):
        if step == args.warmup:
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            clocks.start()
            ev["a"] = torch.cuda.Event(enable_timing=True)
            ev["a"].record()
            ev["t0"] = len(trace)
        elif step == args.warmup + args.steps:
            ev["b"] = torch.cuda.Event(enable_timing=True)
            ev["b"].record()
            torch.cuda.synchronize()
            ev["t1"] = len(trace)
            ev["clocks"] = clocks.stop()
            if dist:
                dist.barrier()

    prompts_dev = [p.to(dev) for p in mine]
    torch.cuda.synchronize()
    n_steps = [0] * per
    generate_with_Flash_dLLM(model, prompts_dev, [p.numel() for p in mine], per, [None] * per, n_steps,
                             max_steps=args.warmup + args.steps, trace=trace, step_hook=hook, **GEN_KW)
    L.check_device_status()
    elapsed = ev["a"].elapsed_time(ev["b"]) * 1e-3
    tok = 0
    for rec in trace[ev["t0"]:ev["t1"]]:
        tok += sum(rec["keep"].values()) + sum(rec.get("verify_keep", {}).values())
    launches = _count_launches(model, per, args)

    # ------------------------------------------------------------ kernels --
    kt = _time_kernels(model, 64 * per, per, WORKLOAD["seq_len"], dev)

    # ---------------------------------------------------------------- e2e --
    e2e = None
    if not args.no_e2e:
        host_prompts = [p.pin_memory() for p in mine]
        # warm-up: one untimed full generation of the same prompts, so the
        # timed one replays the CUDA graphs of every forward shape it meets
        # (a serving process captures them once at start-up)
        generate_with_Flash_dLLM(model, host_prompts, [p.numel() for p in mine], per, [None] * per, [0] * per,
                                 **GEN_KW)
        stats = {}
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        resp, ntok, _ = generate_with_Flash_dLLM(model, host_prompts, [p.numel() for p in mine], per,
                                                 [None] * per, [0] * per, stats=stats, **GEN_KW)
        b.record()
        b.synchronize()
        e2e = dict(t=a.elapsed_time(b) * 1e-3, tok=ntok, steps=stats["steps"], h2d=stats["h2d_bytes"],
                   d2h=stats["d2h_bytes"])

    # ------------------------------------------------------------- gather --
    (elapsed_all, e2e_t), (tok_all, e2e_tok) = reduce_counters(
        [elapsed, e2e["t"] if e2e else 0.0], [tok, e2e["tok"] if e2e else 0.0], device=dev)
    if rank == 0:
        hbm, tf, tf_sus, src = _peaks()
        rows = kt["rows"]
        # DRAM bytes (read + write) of one QKV launch at the 8-sequence step
        # shape, from the ncu capture summarised in
        # profiles/qkv_rope_cache_512rows.md; other shapes: not captured
        traffic = (105.458944e6 + 4.807680e6) if rows == 512 else None
        compute_bound = kt["qkv_flops"] / kt["qkv_bytes"] > (tf * 1e12) / (hbm * 1e9)
        if compute_bound:
            ach = kt["qkv_flops"] / kt["qkv_s"] / 1e12
            roof = {"kernel": "qkv_rope_cache (tcgen05)", "bound": "tensor", "achieved": ach, "peak": tf,
                    "unit": "TFLOP/s", "frac": ach / tf, "peak_source": src, "traffic": traffic,
                    "traffic_unit": "bytes per launch (ncu)", "rows": rows}
        else:
            ach = kt["qkv_bytes"] / kt["qkv_s"] / 1e9
            roof = {"kernel": "qkv_rope_cache (tcgen05)", "bound": "hbm", "achieved": ach, "peak": hbm,
                    "unit": "GB/s", "frac": ach / hbm, "peak_source": src, "traffic": traffic,
                    "traffic_unit": "bytes per launch (ncu)", "rows": rows}
        attn_gbs = kt["attn_bytes"] / kt["attn_s"] / 1e9
        line = {
            "metric": METRIC, "value": tok_all / elapsed_all, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed_all / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform random prompts)",
            "config": dict(WORKLOAD, parallelism=f"seq-shard x{world}", sequences_per_gpu=per,
                           l2="inputs larger than L2 (16 GB of weights streamed per forward)"),
            "tokens_timed": tok_all, "gpu_launches": launches * args.steps * world,
            "layer": {"qkv_us": kt["qkv_s"] * 1e6, "attn_us": kt["attn_s"] * 1e6, "rmsnorm_us": kt["norm_s"] * 1e6,
                      "attn_hbm_gbs": attn_gbs, "attn_frac_hbm": attn_gbs / hbm,
                      "verify_attn_us": kt["vattn_s"] * 1e6,
                      "verify_attn_frac_hbm": kt["vattn_bytes"] / kt["vattn_s"] / 1e9 / hbm,
                      "qkv_hbm_gbs": kt["qkv_bytes"] / kt["qkv_s"] / 1e9,
                      "qkv_tflops": kt["qkv_flops"] / kt["qkv_s"] / 1e12, "rows_per_gpu": rows},
            "roofline": roof,
            "clocks": ev.get("clocks"),
        }
        if e2e:
            line["e2e"] = {"value": e2e_tok / e2e_t, "unit": "tokens/s",
                           "h2d_bytes_per_step": e2e["h2d"] / max(1, e2e["steps"]),
                           "d2h_bytes_per_step": e2e["d2h"] / max(1, e2e["steps"]), "seconds": e2e_t,
                           "tokens": e2e_tok, "steps": e2e["steps"],
                           "warmup": "one untimed full generation of the same prompts (graph capture)"}
        if world == 1 and not args.no_cpu:
            v, threads, sample, _ = _cpu_reference()
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_kernels_only(seqs: int) -> None:
    from types import SimpleNamespace
    from flash_dllm_b200.model import LLaDABlockB200, LLaDAConfigB200
    dev = torch.device("cuda", 0)
    cfg = LLaDAConfigB200()
    blk = LLaDABlockB200(cfg, 0, device=dev, dtype=torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(0)
    with torch.no_grad():
        for name, p in blk.named_parameters():
            p.fill_(1.0) if "norm" in name else p.normal_(0.0, 0.02, generator=g)
    fake = SimpleNamespace(model=SimpleNamespace(transformer=SimpleNamespace(blocks=[blk])), config=cfg)
    kt = _time_kernels(fake, 64 * seqs, seqs, WORKLOAD["seq_len"], dev)
    print(json.dumps({k: v for k, v in kt.items()}), flush=True)


def _count_launches(model, per, args):
    """Kernels of this library launched per decode step.  Each forward (the
    cache forward and the verify forward) launches per layer RMSNorm, the QKV
    GEMM, attention, the fused residual-add + RMSNorm and SwiGLU, plus ln_f's
    RMSNorm; the cache forward adds the attention plan.  The step's decisions
    add row_stats x2, window_accept, verify_accept and refresh_sort.  Split-KV
    combine launches (only when the grid underfills) are not counted."""
    n_layers = model.config.n_layers
    per_forward = n_layers * 5 + 1
    return 2 * per_forward + 1 + 5


if __name__ == "__main__":
    main()
