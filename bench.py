"""Benchmark of the B200 speculative-verification path (driver contract).

Workload ("c2"): one released-shape MoE layer,
expert-major verification of 64 verify tokens (8 sequences x 8 drafts):
hidden 7168, 384 routed experts + 1 shared (SwiGLU, intermediate 2048),
Top-16 sigmoid router with per-expert bias, experts MXFP4 from N(0, 0.02),
hidden states bf16 N(0, 1), seed 1. Synthetic data generated on the GPU.

A step = route -> expert-major plan -> grouped expert FFN -> slot-ordered
combine + shared expert, for all 64 tokens (one KDA+MoE layer's MoE half;
the metric is tokens verified per step / step time x layers).

`value` times the device entry point with inputs resident in HBM; `e2e`
times k3xb_moe_layer_forward_host (pinned host hidden in, output + routes
out, copies inside the timed region). Every step streams ~8.4 GB of expert
weights, far above the 126 MB L2, so no flush is needed.

--impl reference times the reference's own CPU code (oracle/_ref, compiled
from the reference sources) on a bounded sample of the same tokens using all
host threads.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "project-k3x_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "verified draft tokens/s per KDA+MoE layer"
C2 = dict(hidden=7168, inter=2048, experts=384, top_k=16, shared_inter=2048, tokens=64, seed=1,
          sequences=8, drafts=8)
EXPERT_BYTES = 3 * 7168 * 2048 * (0.5 + 1 / 32)   # S_e = 23,396,352 B per expert
# DRAM bytes (read + write) of the routed gate/up + down kernels per
# algorithmic byte, from one ncu capture of a reduced c2 case (128 experts,
# 24 tokens): 2963.3 MB against 2872 MB algorithmic (expected 122.8 unique
# experts). Traffic grows with the unique experts, so a full-size launch is
# this ratio times its algorithmic bytes (profiles/expert_ffn_traffic_128x24.md).
EXPERT_TRAFFIC_RATIO = (1969.4 + 7.3 + 976.3 + 10.3) / (122.8 * 3 * 7168 * 2048 * 0.53125 / 1e6)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """Samples nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def dist_setup(n_gpus):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def graphed(torch, ctx, step, stream, enabled):
    """Counts the library's kernel launches of one eager step, then (when
    enabled) captures the step into a CUDA graph on `stream` so the timed
    loop replays it without host launch overhead. Returns (run, launches per
    step, graph used). Only for steps without NCCL calls: a graph holding
    collectives would have to be released before the communicator is."""
    l0 = ctx.stats()["kernel_launches"]
    step()
    torch.cuda.synchronize()
    per = ctx.stats()["kernel_launches"] - l0
    if not enabled:
        return step, per, False
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    return g.replay, per, True


def phase_profile(ctx, torch, step, steps):
    """Device ms per step of each phase of the path (the library's phase
    timing, k3xb_set_profiling), over `steps` eager steps run after the timed
    region: the events it records never touch the reported numbers."""
    ctx.set_profiling(True)
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    prof = ctx.profile()
    ctx.set_profiling(False)
    dropped = prof.pop("dropped")
    return {"steps": steps, "dropped": dropped, "source": "CUDA events per phase (k3xb_get_profile), eager",
            "ms_per_step": {k: round(v[0] / steps, 4) for k, v in prof.items()}}


def make_c2_layer(ctx, torch, cfg, engine, act_terms):
    import k3xb
    H, I, E, Is = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["shared_inter"]
    seed = cfg["seed"]
    u8 = lambda *s: torch.empty(s, dtype=torch.uint8, device="cuda")
    w = dict(hidden=H, inter=I, experts=E, top_k=cfg["top_k"], shared_inter=Is,
             activation=k3xb.ACT_SWIGLU)
    w["gate_packed"], w["gate_scales"] = u8(E, I, H // 2), u8(E, I, H // 32)
    w["up_packed"], w["up_scales"] = u8(E, I, H // 2), u8(E, I, H // 32)
    w["down_packed"], w["down_scales"] = u8(E, H, I // 2), u8(E, H, I // 32)
    ctx.fill_normal_mxfp4(w["gate_packed"], w["gate_scales"], E * I, H, seed, 10, 0.02)
    ctx.fill_normal_mxfp4(w["up_packed"], w["up_scales"], E * I, H, seed, 11, 0.02)
    ctx.fill_normal_mxfp4(w["down_packed"], w["down_scales"], E * H, I, seed, 12, 0.02)
    w["router"] = torch.empty((E, H), dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(w["router"], seed, 20, 0.02)
    w["correction"] = torch.empty(E, dtype=torch.float32, device="cuda")
    ctx.fill_normal_f32(w["correction"], seed, 21, 0.0, 0.02)
    for i, name in enumerate(("shared_gate", "shared_up")):
        w[name] = torch.empty((Is, H), dtype=torch.int16, device="cuda")
        ctx.fill_normal_bf16(w[name], seed, 22 + i, 0.02)
    w["shared_down"] = torch.empty((H, Is), dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(w["shared_down"], seed, 24, 0.02)
    words = torch.empty((cfg["tokens"], H), dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(words, seed, 30, 1.0)
    hidden = (words.to(torch.int32) << 16).view(torch.float32).contiguous()
    if engine == k3xb.ENGINE_MXF4:
        ctx.prepare_layer_scales(w)   # one-time tcgen05 scale layout of the resident weights
    desc = k3xb.moe_layer_desc(w, engine=engine, act_terms=act_terms)
    return w, desc, hidden


C4 = dict(hidden=7168, inter=2048, experts=384, top_k=16, shared_inter=2048, heads=32, head_dim=128,
          conv_width=4, layers=2, sequences=16, drafts=8, vocab=129280, seed=3)
C3 = dict(heads=32, head_dim=128, nodes=32, depth=4, prefix=1024, seed=2)


def bf16_ones(torch, n):
    return torch.full((n,), 0x3F80, dtype=torch.int16, device="cuda")


def make_kda_gpu(ctx, torch, H, h, d, w, seed):
    """Synthetic official KDA block weights generated on the GPU."""
    P = h * d
    bf = lambda stream, sigma, *shape: _fill_bf16(ctx, torch, shape, seed, stream, sigma)
    f32 = lambda stream, sigma, *shape: _fill_f32(ctx, torch, shape, seed, stream, sigma)
    return dict(heads=h, head_dim=d, conv_width=w, eps=1e-5, gate_lower_bound=-5.0,
                q_proj=bf(40, 0.02, P, H), k_proj=bf(41, 0.02, P, H), v_proj=bf(42, 0.02, P, H),
                q_conv=f32(43, 0.5, P, w), k_conv=f32(44, 0.5, P, w), v_conv=f32(45, 0.5, P, w),
                f_a_proj=bf(46, 0.02, d, H), f_b_proj=bf(47, 0.1, P, d), a_log=f32(48, 0.3, d),
                dt_bias=f32(49, 0.3, P), b_proj=bf(50, 0.02, h, H), g_proj=bf(51, 0.02, P, H),
                o_norm=torch.ones(d, dtype=torch.float32, device="cuda"), o_proj=bf(52, 0.02, H, P))


def _fill_bf16(ctx, torch, shape, seed, stream, sigma):
    t = torch.empty(shape, dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(t, seed, stream, sigma)
    return t


def _fill_f32(ctx, torch, shape, seed, stream, sigma, mean=0.0):
    t = torch.empty(shape, dtype=torch.float32, device="cuda")
    ctx.fill_normal_f32(t, seed, stream, mean, sigma)
    return t


def make_c4_stack(ctx, torch, cfg):
    """Two KDA + MoE layers at c2/c3 dims, embedding, final norm, LM head."""
    import k3xb
    H = cfg["hidden"]
    layers, keep = [], []
    for l in range(cfg["layers"]):
        lcfg = dict(cfg, tokens=1, seed=cfg["seed"] * 100 + l)
        moe, _, _ = make_c2_layer(ctx, torch, lcfg, k3xb.ENGINE_MXF4, 6)
        kda = make_kda_gpu(ctx, torch, H, cfg["heads"], cfg["head_dim"], cfg["conv_width"], lcfg["seed"])
        w = dict(hidden=H, rms_eps=1e-6, kda=kda, moe=moe, self_residual_norm=bf16_ones(torch, H),
                 self_residual_proj=_fill_bf16(ctx, torch, (H,), lcfg["seed"], 60, 0.02),
                 input_norm=bf16_ones(torch, H), moe_residual_norm=bf16_ones(torch, H),
                 moe_residual_proj=_fill_bf16(ctx, torch, (H,), lcfg["seed"], 61, 0.02),
                 post_norm=bf16_ones(torch, H))
        keep.append(w)
        layers.append(k3xb.layer_desc(w))
    V = cfg["vocab"]
    emb = _fill_bf16(ctx, torch, (V, H), cfg["seed"], 70, 1.0)
    lm = _fill_bf16(ctx, torch, (V, H), cfg["seed"], 71, 0.02)
    fnorm = bf16_ones(torch, H)
    model = k3xb.verify_model_desc(layers, V, lm, embedding=emb, final_norm=fnorm)
    return model, (keep, emb, lm, fnorm)


def run_c4(args, rank, world, local, ctx, stream):
    import torch

    import k3xb
    cfg = dict(C4)
    model, keep = make_c4_stack(ctx, torch, cfg)
    S, p, V, L, H = cfg["sequences"], cfg["drafts"], cfg["vocab"], cfg["layers"], cfg["hidden"]
    h, d, w = cfg["heads"], cfg["head_dim"], cfg["conv_width"]
    N, P = p + 1, cfg["heads"] * cfg["head_dim"]
    g = torch.Generator(device="cpu").manual_seed(cfg["seed"])
    tokens = torch.randint(0, V, (S, N), generator=g, dtype=torch.int32)
    tok_d = tokens.cuda()
    drafts_d = tokens[:, 1:].contiguous().cuda()
    conv = torch.empty((L, S, 3, w - 1, P), dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(conv, cfg["seed"], 80, 0.5)
    rec = _fill_f32(ctx, torch, (L, S, h, d, d), cfg["seed"], 81, 0.05)
    draft_logits = _fill_f32(ctx, torch, (S, p, V), cfg["seed"], 82, 1.0)
    logits = torch.empty((S, N, V), dtype=torch.float32, device="cuda")
    acc = torch.zeros(S, dtype=torch.int32, device="cuda")
    com = torch.zeros((S, N), dtype=torch.int32, device="cuda")
    cnt = torch.zeros(S, dtype=torch.int32, device="cuda")
    mode = k3xb.ACCEPT_REJECTION if args.accept == "rejection" else k3xb.ACCEPT_GREEDY
    io = k3xb.verify_io_desc(S, p, conv, rec, acc, com, cnt, drafts_d, tokens=tok_d, logits=logits, mode=mode,
                             draft_logits=draft_logits, temperature=1.0, seed=cfg["seed"])

    def step():
        ctx.verify_step(model, io)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    # unique experts (layer 0 on this step's input; the layers are statistically alike)
    ids = torch.empty((S * N, cfg["top_k"]), dtype=torch.int32, device="cuda")
    x0 = torch.empty((S, N, H), dtype=torch.float32, device="cuda")
    emb = keep[1]
    x0.copy_(((emb[tokens.cuda().long()].to(torch.int32) << 16)).view(torch.float32))
    trace = torch.empty(ctx.kda_trace_bytes(model.layer[0].kda, N, S), dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x0)
    ctx.layer_forward(model.layer[0], x0, x0, list(range(-1, N - 1)), conv[0], rec[0], y, ids, trace)
    ctx.sync()
    unique = int(torch.unique(ids).numel())
    del trace, y, x0
    barrier(world)
    torch.cuda.synchronize()
    launches0 = ctx.stats()["kernel_launches"]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = ctx.stats()["kernel_launches"] - launches0
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    # e2e: host token/draft buffers in, acceptance results out (pinned)
    tok_h, dr_h = tokens.pin_memory(), tokens[:, 1:].contiguous().pin_memory()
    out_h = [torch.empty_like(t, device="cpu").pin_memory() for t in (acc, com, cnt)]
    dl_h = draft_logits.cpu().pin_memory() if mode == k3xb.ACCEPT_REJECTION else None

    def e2e_step():
        tok_d.copy_(tok_h, non_blocking=True)
        drafts_d.copy_(dr_h, non_blocking=True)
        if dl_h is not None:
            draft_logits.copy_(dl_h, non_blocking=True)
        step()
        for hbuf, dbuf in zip(out_h, (acc, com, cnt)):
            hbuf.copy_(dbuf, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s0.elapsed_time(s1) / args.steps, world)
    h2d = tokens.numel() * 4 + S * p * 4 + (S * p * V * 4 if dl_h is not None else 0)
    d2h = (S + S * N + S) * 4
    # whole-step HBM roofline: weights streamed once per step
    kda_bytes = (4 * P * H + d * H + P * d + h * H + H * P) * 2
    moe_bytes = unique * EXPERT_BYTES + cfg["experts"] * H * 2 + 3 * cfg["shared_inter"] * H * 2
    step_bytes = L * (kda_bytes + moe_bytes) + V * H * 2 + S * N * V * 4
    hbm, peak_kind = peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    units = sum_over_ranks(S * p * L, world)
    result = {
        "metric": METRIC, "value": units / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 experts x e2m1-term activations; bf16 KDA/LM-head weights; fp32 accumulate",
        "data": "synthetic (seeded, generated on the GPU)",
        "config": {"workload": f"c4: {L} stacked KDA+MoE layers, LM head V={V}, {args.accept} acceptance",
                   "hidden": H, "experts": cfg["experts"], "top_k": cfg["top_k"], "inter": cfg["inter"],
                   "heads": h, "head_dim": d, "sequences_x_drafts": f"{S}x{p}", "verify_positions": S * N,
                   "layers": L, "vocab": V, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "no flush: each step streams ~19 GB of weights (>> 126 MB L2)"},
        "e2e": {"value": units / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "whole verify step (weights streamed once)", "achieved": achieved,
                     "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "alg_bytes_per_launch": step_bytes, "unique_experts_layer0": unique, "traffic": None},
        "gpu_launches": launches, "clocks": clk.summary(),
        "accepted_mean": float(acc.float().mean().item()),
        # the same inputs every step, so the last step's decisions are every step's
        "accepted_tokens_per_s": sum_over_ranks(int(acc.sum().item()), world) / (ms * 1e-3),
        "committed_tokens_per_s": sum_over_ranks(int(cnt.sum().item()), world) / (ms * 1e-3),
    }
    if args.profile:
        result["phases"] = phase_profile(ctx, torch, step, max(3, args.steps))
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_c3(args, rank, world, local, ctx, stream):
    """KDA recurrence over the c3 draft tree (32 nodes, depth 4) from a
    1024-token prefix state, for `--sequences` sequences sharing the tree."""
    import numpy as np
    import torch
    cfg = dict(C3)
    h, d, Nn, S = cfg["heads"], cfg["head_dim"], cfg["nodes"], args.sequences
    rng = np.random.default_rng(cfg["seed"])
    parent, frontier = [-1], [(0, 1)]
    while len(parent) < Nn:   # BFS, branching 2-3, depth <= 4
        node, depth = frontier.pop(0)
        for _ in range(int(rng.integers(2, 4))):
            if len(parent) >= Nn or depth >= cfg["depth"]:
                break
            parent.append(node)
            frontier.append((len(parent) - 1, depth + 1))
        if not frontier:
            break
    Nn = len(parent)
    P = h * d
    bf = lambda stream, *shape: (_fill_bf16(ctx, torch, shape, cfg["seed"], stream, 1.0).to(torch.int32) << 16
                                 ).view(torch.float32).contiguous()
    q, k, v = bf(1, S, Nn, P), bf(2, S, Nn, P), bf(3, S, Nn, P)
    # q, k L2-normalised per head (official_kda.cpp:259-290: q also x 1/sqrt(d))
    k = (k.view(S, Nn, h, d) / k.view(S, Nn, h, d).norm(dim=-1, keepdim=True)).view(S, Nn, P).contiguous()
    q = (q.view(S, Nn, h, d) / q.view(S, Nn, h, d).norm(dim=-1, keepdim=True) / d ** 0.5).view(S, Nn, P).contiguous()
    ld = torch.nn.functional.logsigmoid(_fill_f32(ctx, torch, (S, Nn, P), cfg["seed"], 4, 1.0)).contiguous()
    beta = torch.sigmoid(_fill_f32(ctx, torch, (S, Nn, h), cfg["seed"], 5, 1.0)).contiguous()
    # prefix state: the recurrence over a 1024-token linear prefix from zero
    T0 = cfg["prefix"]
    pq, pk, pv = bf(6, S, T0, P), bf(7, S, T0, P), bf(8, S, T0, P)
    pk = (pk.view(S, T0, h, d) / pk.view(S, T0, h, d).norm(dim=-1, keepdim=True)).view(S, T0, P).contiguous()
    pld = torch.nn.functional.logsigmoid(_fill_f32(ctx, torch, (S, T0, P), cfg["seed"], 9, 1.0)).contiguous()
    pbe = torch.sigmoid(_fill_f32(ctx, torch, (S, T0, h), cfg["seed"], 10, 1.0)).contiguous()
    zero = torch.zeros((S, h, d, d), dtype=torch.float32, device="cuda")
    state = torch.empty_like(zero)
    ctx.kda_commit(zero, list(range(-1, T0 - 1)), pq, pk, pv, pld, pbe, [T0 - 1] * S, state)
    out = torch.empty((S, Nn, P), dtype=torch.float32, device="cuda")

    def step():
        ctx.kda_tree(state, parent, q, k, v, ld, beta, out)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")   # > L2: each step starts cold
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    with Clocks(local) as clk:
        for i in range(args.steps):
            flush.add_(1)
            ev[2 * i].record(stream)
            step()
            ev[2 * i + 1].record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(statistics.mean(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)), world)
    alg = 2 * S * h * d * d * 4 + S * Nn * h * (3 * d * 2 + d * 4 + 4 + d * 4)
    hbm, peak_kind = peaks()
    result = {
        "metric": METRIC, "value": sum_over_ranks(S * Nn, world) / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 state",
        "data": "synthetic (seeded, generated on the GPU)",
        "config": {"workload": "c3: KDA recurrence over a draft tree", "heads": h, "head_dim": d,
                   "nodes": Nn, "depth": cfg["depth"], "prefix_tokens": T0, "sequences": S,
                   "l2": "flushed (256 MB write) before every timed step"},
        "roofline": {"bound": "hbm", "kernel": "kda_tree_kernel", "achieved": alg / (ms * 1e-3) / 1e9,
                     "peak": hbm, "unit": "GB/s", "frac": alg / (ms * 1e-3) / 1e9 / hbm,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})", "alg_bytes_per_launch": alg,
                     "traffic": None},
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_c2_ep(args, rank, world, local, ctx, stream, cfg):
    """c2 at N > 1: expert parallelism. Rank r holds experts [r*E/N, ...) and
    the hidden rows of its 8/N sequences; tokens reach the experts' ranks and
    come back by NCCL all-to-all (k3xb_ep_moe_layer_forward). Total work is
    fixed (64 verify tokens): strong scaling."""
    import torch
    import torch.distributed as dist

    import k3xb
    E, T, H, K = cfg["experts"], cfg["tokens"], cfg["hidden"], cfg["top_k"]
    if T % world or E % world:
        raise SystemExit(f"c2 expert parallelism needs tokens ({T}) and experts ({E}) divisible by {world}")
    w, _, hidden = make_c2_layer(ctx, torch, cfg, k3xb.ENGINE_MXF4, args.act_terms)
    lw = k3xb.ep_local_layer(w, rank, world)
    desc = k3xb.moe_layer_desc(lw, engine=k3xb.ENGINE_MXF4, act_terms=args.act_terms)
    Tr = T // world
    x = hidden[rank * Tr:(rank + 1) * Tr].contiguous()
    uid = [k3xb.ep_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ctx.ep_init(uid[0], rank, world)
    out = torch.empty((Tr, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((Tr, K), dtype=torch.int32, device="cuda")
    con = torch.empty((Tr, K), dtype=torch.float32, device="cuda")

    def step():
        ctx.ep_moe_layer_forward(desc, E, x, out, ids, con)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    all_ids = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(all_ids, ids)
    unique = int(torch.unique(torch.cat(all_ids)).numel())
    # eager launches: a CUDA graph that holds NCCL calls must be released
    # before the communicator and the process group are destroyed; this
    # path keeps the collectives out of graphs altogether
    run, per_step, used_graph = graphed(torch, ctx, step, stream, False)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            run()
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = per_step * args.steps
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    # e2e: pinned host rows in, layer output out, copies inside the timed region
    x_h = x.cpu().pin_memory()
    o_h = torch.empty((Tr, H), dtype=torch.float32).pin_memory()

    def e2e_step():
        x.copy_(x_h, non_blocking=True)
        step()
        o_h.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s0.elapsed_time(s1) / args.steps, world)
    hbm, peak_kind = peaks()
    alg = unique * EXPERT_BYTES + T * H * 6
    achieved = alg / (ms * 1e-3) / 1e9
    result = {
        "metric": METRIC, "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "mxfp4 weights (e2m1+e8m0) x e2m1-term activations, fp32 accumulate",
        "data": "synthetic (seeded, generated on the GPU)",
        "config": {"workload": "c2: single released-shape MoE layer, expert-major verify",
                   "hidden": H, "experts": E, "top_k": K, "inter": cfg["inter"],
                   "shared_inter": cfg["shared_inter"], "verify_tokens": T, "sequences_x_drafts": "8x8",
                   "layers": 1, "engine": "mxf4", "act_terms": args.act_terms,
                   "parallelism": f"expert parallel x{world} (NCCL all-to-all), {Tr} tokens per rank",
                   "cuda_graph": used_graph,
                   "l2": "no flush: each step streams ~8.4 GB of expert weights (>> 126 MB L2)"},
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4},
        "roofline": {"bound": "hbm", "kernel": "whole EP layer (weights of the used experts, all ranks)",
                     "achieved": achieved, "peak": hbm * world, "unit": "GB/s", "frac": achieved / (hbm * world),
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs x {world} ({peak_kind})",
                     "alg_bytes_per_launch": alg, "unique_experts": unique, "traffic": None},
        "gpu_launches": launches, "clocks": clk.summary(),
    }
    if args.profile:   # every rank takes the same profiled steps (same collectives)
        result["phases"] = phase_profile(ctx, torch, step, max(3, args.steps))
    if rank == 0:
        print(json.dumps(result), flush=True)
    ctx.ep_finalize()


def run_tc_sweep(args, rank, world, local, ctx, stream):
    """Tensor-core sweep of the expert GEMM: 8 experts x M
    tokens each (Top-8 of 8, so every token uses every expert) for
    M in {256, 1024, 4096}, c2 expert shapes. Reports useful TFLOP/s
    (2 * T * k * 3 * H * I per call) and the MMA work, which is `terms`
    times larger because each activation row enters as E2M1 terms."""
    import ctypes as C

    import torch

    import k3xb
    lines = []
    for M in (256, 1024, 4096):
        cfg = dict(C2, experts=8, top_k=8, tokens=M)
        w, desc, hidden = make_c2_layer(ctx, torch, cfg, k3xb.ENGINE_MXF4, args.act_terms)
        T, E, K, H, I = M, 8, 8, cfg["hidden"], cfg["inter"]
        ids = torch.arange(K, dtype=torch.int32, device="cuda").repeat(T, 1).contiguous()
        con = torch.full((T, K), 1.0 / K, dtype=torch.float32, device="cuda")
        plan = dict(group_expert=torch.empty(E, dtype=torch.int32, device="cuda"),
                    group_offset=torch.empty(E + 1, dtype=torch.int32, device="cuda"),
                    assign_token=torch.empty(T * K, dtype=torch.int32, device="cuda"),
                    assign_slot=torch.empty(T * K, dtype=torch.int32, device="cuda"),
                    assign_contrib=torch.empty(T * K, dtype=torch.float32, device="cuda"),
                    group_count=torch.empty(1, dtype=torch.int32, device="cuda"),
                    status=torch.zeros(1, dtype=torch.int32, device="cuda"))
        ctx.expert_major_plan(ids, con, E, plan)
        slot_out = torch.empty((T * K, H), dtype=torch.float32, device="cuda")
        pl = k3xb.Plan(*(k3xb._p(plan[k]) for k in ("group_expert", "group_offset", "assign_token",
                                                      "assign_slot", "assign_contrib", "group_count", "status")))

        def experts():
            ctx._check(ctx.lib.k3xb_moe_experts(ctx.h, C.byref(desc), k3xb._p(hidden), T, C.byref(pl),
                                                k3xb._p(slot_out)), "moe_experts")

        for _ in range(args.warmup):
            experts()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            experts()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        useful = 2.0 * T * K * 3 * H * I
        lines.append({"tokens_per_expert": M, "ms": ms, "useful_tflops": useful / (ms * 1e-3) / 1e12,
                      "mma_tflops": useful * args.act_terms / (ms * 1e-3) / 1e12})
        del w, desc, hidden, slot_out
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"metric": "expert GEMM tensor-core sweep (useful TFLOP/s)", "config":
                          {"workload": "8 experts x M tokens, Top-8 of 8, H 7168, I 2048, MXFP4",
                           "act_terms": args.act_terms}, "sweep": lines,
                          "peak_note": "mxf4 dense peak 9 PFLOP/s nominal; MMA work = terms x useful"}), flush=True)


def run_ours(args):
    import torch

    import k3xb
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    cfg = dict(C2)
    if args.experts:   # reduced c2 case for profiler captures (a few GB on the device)
        cfg["experts"] = args.experts
    if args.tokens:
        cfg["tokens"] = args.tokens
    ctx = k3xb.Context(local)
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx.use_stream(stream)
    if args.config == "c4":
        run_c4(args, rank, world, local, ctx, stream)
        return finish(ctx, world)
    if args.config == "c3":
        run_c3(args, rank, world, local, ctx, stream)
        return finish(ctx, world)
    if args.config == "tc":
        run_tc_sweep(args, rank, world, local, ctx, stream)
        return finish(ctx, world)
    if world > 1:
        run_c2_ep(args, rank, world, local, ctx, stream, cfg)
        return finish(ctx, world)
    engine = k3xb.ENGINE_SIMT if args.engine == "simt" else k3xb.ENGINE_MXF4
    w, desc, hidden = make_c2_layer(ctx, torch, cfg, engine, args.act_terms)
    T, H, K, E = cfg["tokens"], cfg["hidden"], cfg["top_k"], cfg["experts"]
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    con = torch.empty((T, K), dtype=torch.float32, device="cuda")

    def step():
        ctx.moe_layer_forward(desc, hidden, out, ids, con)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    # unique experts of this workload (for the algorithmic byte count)
    unique = int(torch.unique(ids).numel())
    run, per_step, used_graph = graphed(torch, ctx, step, stream, not args.no_graph)

    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            run()
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = per_step * args.steps
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = max_over_ranks(ms, world)
    barrier(world)

    # dominant kernel(s): the grouped expert FFN, timed alone on the same stream
    plan = dict(group_expert=torch.empty(E, dtype=torch.int32, device="cuda"),
                group_offset=torch.empty(E + 1, dtype=torch.int32, device="cuda"),
                assign_token=torch.empty(T * K, dtype=torch.int32, device="cuda"),
                assign_slot=torch.empty(T * K, dtype=torch.int32, device="cuda"),
                assign_contrib=torch.empty(T * K, dtype=torch.float32, device="cuda"),
                group_count=torch.empty(1, dtype=torch.int32, device="cuda"),
                status=torch.zeros(1, dtype=torch.int32, device="cuda"))
    ctx.expert_major_plan(ids, con, E, plan)
    slot_out = torch.empty((T * K, H), dtype=torch.float32, device="cuda")
    pl = k3xb.Plan(*(k3xb._p(plan[k]) for k in ("group_expert", "group_offset", "assign_token",
                                                  "assign_slot", "assign_contrib", "group_count", "status")))
    import ctypes as C

    def experts():
        ctx._check(ctx.lib.k3xb_moe_experts(ctx.h, C.byref(desc), k3xb._p(hidden), T, C.byref(pl),
                                            k3xb._p(slot_out)), "moe_experts")

    for _ in range(2):
        experts()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, args.steps)
    e0.record(stream)
    for _ in range(reps):
        experts()
    e1.record(stream)
    torch.cuda.synchronize()
    exp_ms = e0.elapsed_time(e1) / reps
    alg_bytes = unique * EXPERT_BYTES + T * H * 2 + T * H * 4
    hbm, peak_kind = peaks()
    achieved = alg_bytes / (exp_ms * 1e-3) / 1e9

    # e2e through the host-buffer C-ABI entry point (pinned host memory)
    h_host = hidden.cpu().pin_memory()
    o_host = torch.empty((T, H), dtype=torch.float32).pin_memory()
    i_host = torch.empty((T, K), dtype=torch.int32).pin_memory()
    c_host = torch.empty((T, K), dtype=torch.float32).pin_memory()
    for _ in range(2):
        ctx.moe_layer_forward_host(desc, h_host, o_host, i_host, c_host)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        ctx.moe_layer_forward_host(desc, h_host, o_host, i_host, c_host)
    s1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s0.elapsed_time(s1) / args.steps, world)
    wall_e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps

    total_tokens = sum_over_ranks(T, world)
    result = {
        "metric": METRIC,
        "value": total_tokens / (ms_max * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "mxfp4 weights (e2m1+e8m0) x e2m1-term activations, fp32 accumulate",
        "data": "synthetic (seeded, generated on the GPU)",
        "config": {"workload": "c2: single released-shape MoE layer, expert-major verify"
                   + ("" if (E, T) == (C2["experts"], C2["tokens"]) else f" (reduced: {E} experts, {T} tokens)"),
                   "hidden": H, "experts": E, "top_k": K, "inter": cfg["inter"],
                   "shared_inter": cfg["shared_inter"], "verify_tokens": T,
                   "sequences_x_drafts": "8x8", "layers": 1, "engine": args.engine,
                   "act_terms": args.act_terms if args.engine == "mxf4" else None,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "cuda_graph": used_graph,
                   "l2": "no flush: each step streams ~8.4 GB of expert weights (>> 126 MB L2)"},
        "e2e": {"value": total_tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4 + 2 * T * K * 4,
                "wall_ms_per_step": wall_e2e_ms},
        "roofline": {"bound": "hbm", "kernel": f"expert FFN ({args.engine})", "achieved": achieved,
                     "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "alg_bytes_per_launch": alg_bytes, "unique_experts": unique,
                     "launch_ms": exp_ms, "traffic": unique * EXPERT_BYTES * EXPERT_TRAFFIC_RATIO,
                     "traffic_source": "ncu dram__bytes_read+write of gate/up + down on a reduced c2 case, "
                                       "scaled by unique experts (profiles/expert_ffn_traffic_128x24.md)"},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    if args.profile:
        result["phases"] = phase_profile(ctx, torch, step, max(3, args.steps))
    if rank == 0 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(w, hidden, cfg, args)
    if rank == 0:
        print(json.dumps(result), flush=True)
    finish(ctx, world)


def finish(ctx, world):
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def host_layer(w, cfg):
    """Copies the device-generated layer to host numpy for the CPU reference."""
    import numpy as np
    L = dict(hidden=cfg["hidden"], inter=cfg["inter"], experts=cfg["experts"], top_k=cfg["top_k"],
             shared_inter=cfg["shared_inter"], activation=0, situ_beta=4.0, situ_linear_beta=0.0)
    for k in ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales"):
        L[k] = w[k].cpu().numpy()
    for k in ("router", "shared_gate", "shared_up", "shared_down"):
        L[k] = w[k].cpu().numpy().view(np.uint16)
    L["correction"] = w["correction"].cpu().numpy()
    return L


def cpu_sample_tokens(cores):
    # ~7.7 s of single-core work per token at c2 (48 matvecs of 2048x7168)
    return max(1, min(64, cores))


def cpu_baseline(w, hidden, cfg, args):
    import numpy as np

    from oracle import Reference, have_reference
    if not have_reference():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    ref = Reference()
    L = host_layer(w, cfg)
    x = hidden.cpu().numpy()
    cores = max(1, os.cpu_count() or 1)
    n = cpu_sample_tokens(cores)
    t0 = time.perf_counter()
    ref.moe_layer(L, x, 0, n, threads=cores)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tokens/s", "cores": cores, "kind": "reference",
            "sample": f"{n} of the 64 c2 tokens through the reference CPU functions "
                      f"(route_official_moe, mxfp4_matmul, situ_glu) on {cores} threads, {dt:.1f} s"}


def run_reference(args):
    """--impl reference: the reference's CPU implementation of the path."""
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import Reference, have_reference, make_moe_layer  # noqa: F401
    if not have_reference():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libk3x_ref.so was not built"}))
        return
    import torch

    import k3xb
    cfg = dict(C2)
    # same synthetic workload as our arm (generated with the same seeds)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    w, desc, hidden = make_c2_layer(ctx, torch, cfg, k3xb.ENGINE_SIMT, 6)
    torch.cuda.synchronize()
    L = host_layer(w, cfg)
    x = hidden.cpu().numpy()
    del w
    ref = Reference()
    cores = max(1, os.cpu_count() or 1)
    n = cpu_sample_tokens(cores)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        ref.moe_layer(L, x, 0, n, threads=cores)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    dt = statistics.mean(times)
    value = n / dt
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 64 / value * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32/fp64 (reference CPU)", "data": "synthetic (same seeds as our arm)",
        "config": {"workload": "c2: single released-shape MoE layer, expert-major verify",
                   "hidden": cfg["hidden"], "experts": cfg["experts"], "top_k": cfg["top_k"],
                   "inter": cfg["inter"], "verify_tokens": cfg["tokens"], "layers": 1},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "reference",
                         "sample": f"{n} of 64 tokens per step on {cores} threads"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--engine", choices=["mxf4", "simt"], default=os.environ.get("K3XB_ENGINE", "mxf4"))
    ap.add_argument("--act-terms", type=int, default=6)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", choices=["c2", "c3", "c4", "tc"], default="c2",
                    help="c2 (default, the headline line), c3 KDA tree, c4 two-layer verify step, "
                         "tc tensor-core sweep of the expert GEMM")
    ap.add_argument("--accept", choices=["greedy", "rejection"], default="greedy", help="c4 acceptance rule")
    ap.add_argument("--sequences", type=int, default=1, help="c3: sequences sharing the draft tree")
    ap.add_argument("--experts", type=int, default=0, help="c2 with fewer experts (small profiler case)")
    ap.add_argument("--tokens", type=int, default=0, help="c2 with another verify-token count")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of a CUDA graph replay")
    ap.add_argument("--profile", action="store_true",
                    help="after the timed region, add per-phase device times (rank 0's) to the JSON line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
