"""Benchmark of the B200 speculative-verification path (driver contract).

Default workload (every N): BASELINE.json configs[4], "c5": an 8-layer
stack of KDA + MoE layers at the c2/c3 dims (hidden 7168; KDA 32 heads x
128; 384 routed experts + 1 shared, Top-16, intermediate 2048, SwiGLU,
MXFP4 experts), 64 sequences x (anchor + 8 drafts) = 576 verify positions,
embedding and V = 129,280 LM head, greedy acceptance, a Zipf(1.1) expert
bias, seed 4. At N = 1 it runs on one B200 (k3xb_verify_step); at N > 1
the experts are sharded over the GPUs and the sequences split between
them (k3xb_ep_verify_step): the same 512 drafts, so the scaling is strong.
One step = the whole verify step (layers, LM head, acceptance, state
commit). Other lines with --config: c4 (2 layers, 16 sequences), c2 (one
MoE layer, 64 tokens), c3 (KDA draft tree), tc (tensor-core sweep),
attnres (block attention residual over many sources).

Inputs are seeded synthetic data of the configs' shapes. Both arms build
them from one spec (seed, stream, sigma per tensor): the GPU arm with the
library's generator in HBM, the reference arm on the host with its exact
restatement (oracle/k3x_oracle.c:k3xo_fill_normal_*, pinned bit for bit in
tests/test_gpu_synth.py), so both see the same numbers.

`value` times the device entry point with every input in HBM; `e2e` adds
the host copies of the step's tokens (pinned) in and of its acceptance
results out, through the same public call. Each step streams tens of GB of
weights, far above the 126 MB L2, so no flush is needed.

--impl reference times the reference's own CPU code (oracle/_ref, compiled
from the reference sources) on a bounded sample of the same workload: one
KDA + MoE layer over the anchor positions of as many sequences as the host
has cores, one thread per sequence. It never loads this library.
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
C4 = dict(hidden=7168, inter=2048, experts=384, top_k=16, shared_inter=2048, heads=32, head_dim=128,
          conv_width=4, layers=2, sequences=16, drafts=8, vocab=129280, seed=3, zipf=0.0)
C5 = dict(C4, layers=8, sequences=64, seed=4, zipf=1.1)
C3 = dict(heads=32, head_dim=128, nodes=32, depth=4, prefix=1024, seed=2)
ZIPF_SCALE = 0.5   # c5: the rank-r expert's bias is ZIPF_SCALE * r^-1.1 (ranks a seeded permutation)
EXPERT_BYTES = 3 * 7168 * 2048 * (0.5 + 1 / 32)   # S_e = 23,396,352 B per expert
# DRAM bytes (read + write) of the routed expert kernels per algorithmic
# byte, from single-launch ncu captures: gate/up 1047.2 MB against 998.2 MB
# (64 experts x 96 tokens, profiles/expert_ffn_c5_density_64x96.md), down
# 985.2 MB against 957.9 MB (128 experts x 24 tokens,
# profiles/expert_ffn_traffic_128x24.md), weighted 2:1 as their bytes are.
# Traffic grows with the experts streamed, so a full-size launch is this
# ratio times its algorithmic bytes.
EXPERT_TRAFFIC_RATIO = (2 * (1032.679 + 14.555) / 998.244 + (976.479 + 8.689) / 957.9) / 3


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


def dist_setup():
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
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


def phase_profile(ctx, torch, step, steps):
    """Device ms per step of each phase of the path (the library's phase
    timing, k3xb_set_profiling: CUDA events on the launching streams), over
    `steps` eager steps run after the timed region: the events never touch
    the reported step times."""
    ctx.set_profiling(True)
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    prof = ctx.profile()
    ctx.set_profiling(False)
    dropped = prof.pop("dropped")
    return {"steps": steps, "dropped": dropped, "source": "CUDA events per phase (k3xb_get_profile), eager",
            "ms_per_step": {k: round(v[0] / steps, 4) for k, v in prof.items()}}


# ---- the workload spec ---------------------------------------------------------
# One entry per tensor: (kind, shape, seed, stream, sigma[, mean]); kind
# "mxfp4" [rows][cols] -> packed + scales, "bf16" words, "f32", "ones_bf16",
# "ones_f32". Both arms build every tensor from this table.

def moe_spec(cfg, seed):
    H, I, E, Is = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["shared_inter"]
    return {"gate": ("mxfp4", (E * I, H), seed, 10, 0.02), "up": ("mxfp4", (E * I, H), seed, 11, 0.02),
            "down": ("mxfp4", (E * H, I), seed, 12, 0.02), "router": ("bf16", (E, H), seed, 20, 0.02),
            "correction": ("f32", (E,), seed, 21, 0.02, 0.0),
            "shared_gate": ("bf16", (Is, H), seed, 22, 0.02), "shared_up": ("bf16", (Is, H), seed, 23, 0.02),
            "shared_down": ("bf16", (H, Is), seed, 24, 0.02)}


def kda_spec(cfg, seed):
    H, h, d, w = cfg["hidden"], cfg["heads"], cfg["head_dim"], cfg["conv_width"]
    P = h * d
    return {"q_proj": ("bf16", (P, H), seed, 40, 0.02), "k_proj": ("bf16", (P, H), seed, 41, 0.02),
            "v_proj": ("bf16", (P, H), seed, 42, 0.02), "q_conv": ("f32", (P, w), seed, 43, 0.5, 0.0),
            "k_conv": ("f32", (P, w), seed, 44, 0.5, 0.0), "v_conv": ("f32", (P, w), seed, 45, 0.5, 0.0),
            "f_a_proj": ("bf16", (d, H), seed, 46, 0.02), "f_b_proj": ("bf16", (P, d), seed, 47, 0.1),
            "a_log": ("f32", (d,), seed, 48, 0.3, 0.0), "dt_bias": ("f32", (P,), seed, 49, 0.3, 0.0),
            "b_proj": ("bf16", (h, H), seed, 50, 0.02), "g_proj": ("bf16", (P, H), seed, 51, 0.02),
            "o_norm": ("ones_f32", (d,)), "o_proj": ("bf16", (H, P), seed, 52, 0.02)}


def norm_spec(cfg, seed):
    H = cfg["hidden"]
    return {"self_residual_norm": ("ones_bf16", (H,)), "self_residual_proj": ("bf16", (H,), seed, 60, 0.02),
            "input_norm": ("ones_bf16", (H,)), "moe_residual_norm": ("ones_bf16", (H,)),
            "moe_residual_proj": ("bf16", (H,), seed, 61, 0.02), "post_norm": ("ones_bf16", (H,))}


def layer_seed(cfg, l):
    return cfg["seed"] * 100 + l


def zipf_correction(cfg):
    """c5's per-expert bias: ZIPF_SCALE * rank^-zipf, the ranks a permutation
    drawn from the config seed (None: the generator's N(0, 0.02) correction)."""
    import numpy as np
    if not cfg.get("zipf"):
        return None
    E = cfg["experts"]
    perm = np.random.default_rng(cfg["seed"]).permutation(E)
    return (ZIPF_SCALE * (perm + 1.0) ** -cfg["zipf"]).astype(np.float32)


def ep_owner(cfg, world):
    """The expert placement of an expert-parallel run: with a routing bias
    (c5's Zipf), the experts dealt over the ranks by bias (k3xb_ep_balance),
    so the hot experts of every layer (the bias is the same in each) land on
    different ranks; otherwise contiguous ranges (None). Placement changes
    no result."""
    import k3xb
    zc = zipf_correction(cfg)
    return None if zc is None else k3xb.ep_balance(zc, world)


def stack_tokens(cfg):
    import numpy as np
    return np.random.default_rng(cfg["seed"]).integers(0, cfg["vocab"], size=(cfg["sequences"], cfg["drafts"] + 1),
                                                       dtype=np.int64).astype(np.int32)


# ---- GPU arm: tensors in HBM from the spec ---------------------------------------

def gpu_tensor(ctx, torch, entry):
    kind, shape = entry[0], entry[1]
    if kind == "ones_bf16":
        return torch.full(shape, 0x3F80, dtype=torch.int16, device="cuda")
    if kind == "ones_f32":
        return torch.ones(shape, dtype=torch.float32, device="cuda")
    seed, stream, sigma = entry[2], entry[3], entry[4]
    if kind == "bf16":
        t = torch.empty(shape, dtype=torch.int16, device="cuda")
        ctx.fill_normal_bf16(t, seed, stream, sigma)
        return t
    if kind == "f32":
        t = torch.empty(shape, dtype=torch.float32, device="cuda")
        ctx.fill_normal_f32(t, seed, stream, entry[5], sigma)
        return t
    rows, cols = shape
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty((rows, cols // 32), dtype=torch.uint8, device="cuda")
    ctx.fill_normal_mxfp4(packed, scales, rows, cols, seed, stream, sigma)
    return packed, scales


def gpu_moe(ctx, torch, cfg, seed, rank=0, world=1):
    """One MoE layer dict in HBM; with world > 1 only this rank's experts
    (generated whole, sliced, the rest freed)."""
    import k3xb
    H, I, E = cfg["hidden"], cfg["inter"], cfg["experts"]
    spec = moe_spec(cfg, seed)
    w = dict(hidden=H, inter=I, experts=E, top_k=cfg["top_k"], shared_inter=cfg["shared_inter"],
             activation=k3xb.ACT_SWIGLU)
    for name in ("gate", "up", "down"):
        packed, scales = gpu_tensor(ctx, torch, spec[name])
        rows = I if name != "down" else H
        w[f"{name}_packed"] = packed.view(E, rows, -1)
        w[f"{name}_scales"] = scales.view(E, rows, -1)
    for name in ("router", "correction", "shared_gate", "shared_up", "shared_down"):
        w[name] = gpu_tensor(ctx, torch, spec[name])
    zc = zipf_correction(cfg)
    if zc is not None:
        w["correction"] = torch.from_numpy(zc).cuda()
    if world > 1:
        local = k3xb.ep_local_layer(w, rank, world, owner=ep_owner(cfg, world))
        for k in ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales"):
            local[k] = local[k].clone()
        w = local
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    ctx.prepare_layer_scales(w)   # one-time tcgen05 scale layout of the resident experts
    return w


def gpu_stack(ctx, torch, cfg, rank=0, world=1, act_terms=0):
    import k3xb
    layers, keep = [], []
    for l in range(cfg["layers"]):
        seed = layer_seed(cfg, l)
        w = {k: gpu_tensor(ctx, torch, v) for k, v in norm_spec(cfg, seed).items()}
        kda = {k: gpu_tensor(ctx, torch, v) for k, v in kda_spec(cfg, seed).items()}
        kda.update(heads=cfg["heads"], head_dim=cfg["head_dim"], conv_width=cfg["conv_width"], eps=1e-6,
                   gate_lower_bound=-5.0)
        w.update(hidden=cfg["hidden"], rms_eps=1e-6, kda=kda, moe=gpu_moe(ctx, torch, cfg, seed, rank, world))
        keep.append(w)
        layers.append(k3xb.layer_desc(w, act_terms=act_terms))
    H, V = cfg["hidden"], cfg["vocab"]
    emb = gpu_tensor(ctx, torch, ("bf16", (V, H), cfg["seed"], 70, 1.0))
    lm = gpu_tensor(ctx, torch, ("bf16", (V, H), cfg["seed"], 71, 0.02))
    fnorm = gpu_tensor(ctx, torch, ("ones_bf16", (H,)))
    model = k3xb.verify_model_desc(layers, V, lm, embedding=emb, final_norm=fnorm)
    return model, (keep, emb, lm, fnorm)


def gpu_states(ctx, torch, cfg):
    S, L, h, d, w = cfg["sequences"], cfg["layers"], cfg["heads"], cfg["head_dim"], cfg["conv_width"]
    P = h * d
    conv = gpu_tensor(ctx, torch, ("bf16", (L, S, 3, w - 1, P), cfg["seed"], 80, 0.5))
    rec = gpu_tensor(ctx, torch, ("f32", (L, S, h, d, d), cfg["seed"], 81, 0.05, 0.0))
    return conv, rec


# ---- reference arm: the same tensors on the host ----------------------------------

def host_threads():
    return max(1, os.cpu_count() or 1)


def parallel(fn, jobs, threads):
    """Runs fn(job) for every job on `threads` threads (the oracle's C calls
    release the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(fn, jobs))


def host_tensor(rs, entry, threads=1, rows=None):
    """The spec entry on the host (numpy), optionally only the given row
    range (start, stop) of its first dimension, generated in chunks on
    `threads` threads."""
    import numpy as np
    kind, shape = entry[0], entry[1]
    n_row = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    r0, r1 = rows if rows else (0, shape[0])
    out_shape = (r1 - r0,) + tuple(shape[1:])
    if kind == "ones_bf16":
        return np.full(out_shape, 0x3F80, np.uint16)
    if kind == "ones_f32":
        return np.ones(out_shape, np.float32)
    seed, stream, sigma = entry[2], entry[3], entry[4]
    n = (r1 - r0) * n_row
    first = r0 * n_row
    if kind in ("bf16", "f32"):
        out = np.empty(n, np.uint16 if kind == "bf16" else np.float32)
        chunk = max(1 << 16, (n + threads - 1) // threads)
        chunk += chunk % 2

        def job(a):
            b = min(n, a + chunk)
            if kind == "bf16":
                rs.lib.k3xo_fill_normal_bf16(out[a:b], b - a, first + a, seed, stream, sigma)
            else:
                rs.lib.k3xo_fill_normal_f32(out[a:b], b - a, first + a, seed, stream, entry[5], sigma)
        parallel(job, range(0, n, chunk), threads)
        return out.reshape(out_shape)
    cols = shape[1]
    blocks = n // 32
    packed = np.empty(blocks * 16, np.uint8)
    scales = np.empty(blocks, np.uint8)
    chunk = max(1024, (blocks + threads - 1) // threads)

    def mjob(a):
        b = min(blocks, a + chunk)
        rs.lib.k3xo_fill_normal_mxfp4(packed[a * 16:b * 16], scales[a:b], b - a, first // 32 + a, seed, stream,
                                      sigma)
    parallel(mjob, range(0, blocks, chunk), threads)
    return packed.reshape(r1 - r0, cols // 2), scales.reshape(r1 - r0, cols // 32)


def host_moe_shell(rs, cfg, seed, threads):
    """A MoE layer dict on the host with router, correction and shared
    expert built and the expert arrays allocated but not yet filled
    (host_fill_experts builds the experts a sample needs)."""
    import numpy as np
    H, I, E = cfg["hidden"], cfg["inter"], cfg["experts"]
    spec = moe_spec(cfg, seed)
    w = dict(hidden=H, inter=I, experts=E, top_k=cfg["top_k"], shared_inter=cfg["shared_inter"], activation=0,
             situ_beta=4.0, situ_linear_beta=0.0)
    for name in ("router", "correction", "shared_gate", "shared_up", "shared_down"):
        w[name] = host_tensor(rs, spec[name], threads)
    zc = zipf_correction(cfg)
    if zc is not None:
        w["correction"] = zc
    for name, rows in (("gate", I), ("up", I), ("down", H)):
        cols = H if name != "down" else I
        w[f"{name}_packed"] = np.zeros((E, rows, cols // 2), np.uint8)   # pages untouched until filled
        w[f"{name}_scales"] = np.zeros((E, rows, cols // 32), np.uint8)
    return w, spec


def host_fill_experts(rs, cfg, w, spec, experts, threads):
    """Builds experts `experts` of the shell (every matrix row range of
    each) on `threads` threads."""
    H, I = cfg["hidden"], cfg["inter"]
    jobs = [(name, int(e)) for e in sorted(set(int(x) for x in experts)) for name in ("gate", "up", "down")]

    def job(j):
        name, e = j
        rows = I if name != "down" else H
        p, s = host_tensor(rs, spec[name], 1, rows=(e * rows, (e + 1) * rows))
        w[f"{name}_packed"][e] = p
        w[f"{name}_scales"][e] = s
    parallel(job, jobs, threads)


def host_layer(rs, cfg, l, threads):
    seed = layer_seed(cfg, l)
    layer = {k: host_tensor(rs, v, threads) for k, v in norm_spec(cfg, seed).items()}
    kda = {k: host_tensor(rs, v, threads) for k, v in kda_spec(cfg, seed).items()}
    kda.update(hidden=cfg["hidden"], heads=cfg["heads"], head_dim=cfg["head_dim"], conv_width=cfg["conv_width"],
               eps=1e-6, gate_lower_bound=-5.0)
    moe, spec = host_moe_shell(rs, cfg, seed, threads)
    layer.update(hidden=cfg["hidden"], rms_eps=1e-6, kda=kda, moe=moe)
    return layer, spec


def decode_words(words):
    import numpy as np
    return (np.asarray(words, np.uint32) << 16).view(np.float32)


class ReferenceSample:
    """The reference CPU arm's bounded sample of a c4/c5 step: layer 0 over
    the anchor positions of n sequences (one thread each), through the
    reference's own functions (ref_shim.cpp:k3xr_plain_layer). Built from
    the spec on the host; the experts are built after a route-only pass
    finds the ones the sample uses."""

    def __init__(self, cfg):
        import numpy as np

        from oracle import Reference, Restatement
        self.ref, rs = Reference(), Restatement()
        self.cfg = cfg
        self.threads = host_threads()
        self.n = min(cfg["sequences"], self.threads)
        t0 = time.perf_counter()
        self.layer, spec = host_layer(rs, cfg, 0, self.threads)
        H, h, d, w = cfg["hidden"], cfg["heads"], cfg["head_dim"], cfg["conv_width"]
        P, S, n = h * d, cfg["sequences"], self.n
        tokens = stack_tokens(cfg)[:n, 0]
        rows = [host_tensor(rs, ("bf16", (cfg["vocab"], H), cfg["seed"], 70, 1.0), 1, rows=(int(t), int(t) + 1))[0]
                for t in tokens]
        self.hidden = decode_words(np.stack(rows)).reshape(n, 1, H)
        per_seq_conv = 3 * (w - 1) * P
        self.conv = host_tensor(rs, ("bf16", (cfg["layers"] * S, per_seq_conv), cfg["seed"], 80, 0.5), self.threads,
                                rows=(0, n)).reshape(n, 3, (w - 1) * P)
        self.rec = host_tensor(rs, ("f32", (cfg["layers"] * S, h * d * d), cfg["seed"], 81, 0.05, 0.0),
                               self.threads, rows=(0, n)).reshape(n, h, d, d)
        _, ids, _, _ = self.ref.plain_layer(self.layer, self.hidden, self.hidden, self.conv, self.rec,
                                            route_only=True, threads=self.threads)
        self.unique = len(set(ids.reshape(-1).tolist()))
        host_fill_experts(rs, cfg, self.layer["moe"], spec, ids.reshape(-1), self.threads)
        self.build_s = time.perf_counter() - t0

    def step(self):
        t0 = time.perf_counter()
        self.ref.plain_layer(self.layer, self.hidden, self.hidden, self.conv, self.rec, threads=self.n)
        return time.perf_counter() - t0

    def units(self):
        """Verified draft tokens of the sample: each position counts p/(p+1)
        of a draft (a sequence's step verifies p drafts over p+1 positions)."""
        p = self.cfg["drafts"]
        return self.n * p / (p + 1)

    def describe(self, dt):
        return (f"layer 0 of {self.cfg['layers']} over the anchor positions of {self.n} of the "
                f"{self.cfg['sequences']} sequences (one thread each; {self.unique} distinct experts), "
                f"through the reference's prepare_official_moe_input, official_kda_cpu, route_official_moe, "
                f"mxfp4_matmul and situ_glu; {dt:.2f} s per sample; counted as {self.units():.2f} verified "
                f"draft tokens (p/(p+1) of a draft per position)")


class ReferenceSampleC2:
    """The reference CPU arm's sample of c2: the first n of the 64 tokens
    through the plain MoE layer of the reference's functions
    (k3xr_moe_layer_forward), n = host threads."""

    def __init__(self, cfg):
        import numpy as np

        from oracle import Reference, Restatement
        self.ref, rs = Reference(), Restatement()
        self.cfg, self.threads = cfg, host_threads()
        self.n = min(cfg["tokens"], self.threads)
        t0 = time.perf_counter()
        self.layer, spec = host_moe_shell(rs, cfg, cfg["seed"], self.threads)
        H = cfg["hidden"]
        self.x = decode_words(host_tensor(rs, ("bf16", (cfg["tokens"], H), cfg["seed"], 30, 1.0), self.threads,
                                          rows=(0, self.n)))
        ids = np.stack([self.ref.route(self.x[t], self.layer["router"], self.layer["correction"], cfg["top_k"])[0]
                        for t in range(self.n)])
        self.unique = len(set(ids.reshape(-1).tolist()))
        host_fill_experts(rs, cfg, self.layer, spec, ids.reshape(-1), self.threads)
        self.build_s = time.perf_counter() - t0

    def step(self):
        t0 = time.perf_counter()
        self.ref.moe_layer(self.layer, self.x, 0, self.n, threads=self.n)
        return time.perf_counter() - t0

    def units(self):
        return float(self.n)

    def describe(self, dt):
        return (f"{self.n} of the 64 c2 tokens ({self.unique} distinct experts) through the reference's "
                f"route_official_moe, mxfp4_matmul and situ_glu on {self.n} threads, {dt:.2f} s per sample")


class AttnResSample:
    """The CPU arm of the attnres line: the block attention residual over
    all 576 positions (the whole workload; it takes well under a second of
    CPU), through the pinned restatement of model.cpp:645-666
    (oracle/k3x_oracle.c:k3xo_block_attention_residual). The reference's own
    function is private to its model engine, so this is the port. Inputs
    are the GPU arm's, built on the host with the generator's restatement;
    the positions are split into one contiguous chunk per host thread."""

    def __init__(self, sources):
        import numpy as np

        from oracle import Restatement
        self.rs = Restatement()
        self.threads = host_threads()
        T, H, S = C5["sequences"] * (C5["drafts"] + 1), C5["hidden"], sources
        self.T, self.S, self.n = T, S, T
        t0 = time.perf_counter()
        spec = ("f32", ((S + 1) * T, H), 11, 1, 1.0, 0.0)   # the GPU arm's [S + 1][T][H] values, flattened
        values = np.stack([host_tensor(self.rs, spec, self.threads, rows=(d * T, (d + 1) * T)) for d in range(S + 1)])
        self.norm = host_tensor(self.rs, ("f32", (H,), 11, 2, 0.1, 1.0))
        self.proj = host_tensor(self.rs, ("f32", (H,), 11, 3, 3.0 / H ** 0.5, 0.0))
        step = (T + self.threads - 1) // self.threads
        self.chunks = [(np.ascontiguousarray(values[S, a:a + step]), np.ascontiguousarray(values[:S, a:a + step]))
                       for a in range(0, T, step)]
        self.build_s = time.perf_counter() - t0

    def step(self):
        t0 = time.perf_counter()
        parallel(lambda c: self.rs.block_attention_residual(c[0], c[1], self.norm, self.proj, 1e-6), self.chunks,
                 len(self.chunks))
        return time.perf_counter() - t0

    def units(self):
        return float(self.T)

    def describe(self, dt):
        return (f"all {self.T} positions x {self.S + 1} depths at H {C5['hidden']} through the restatement of "
                f"model.cpp:645-666 (the reference's function is private to its engine), {len(self.chunks)} "
                f"threads, {dt * 1e3:.1f} ms per step")


def attnres_cpu_baseline(sources):
    """The attnres line's CPU port on this host: one untimed step, then the
    mean of three timed."""
    s = AttnResSample(sources)
    s.step()
    dt = statistics.mean(s.step() for _ in range(3))
    return {"value": s.units() / dt, "unit": "positions/s", "cores": len(s.chunks), "kind": "port",
            "sample": s.describe(dt) + f"; built on the host in {s.build_s:.1f} s"}


def reference_sample(cfg_name):
    from oracle import have_reference
    if not have_reference():
        return None
    return ReferenceSampleC2(dict(C2)) if cfg_name == "c2" else ReferenceSample(dict(C5 if cfg_name == "c5" else C4))


def cpu_baseline(cfg_name):
    """The reference's CPU code on a bounded sample, timed on this host
    (rank 0, N = 1): one untimed sample, then one timed."""
    s = reference_sample(cfg_name)
    if s is None:
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    s.step()
    dt = s.step()
    return {"value": s.units() / dt, "unit": "tokens/s", "cores": s.n, "kind": "reference",
            "sample": s.describe(dt) + f"; built on the host in {s.build_s:.1f} s"}


# ---- GPU arm: the verify-step stack (c4, c5) -------------------------------------------

def stack_config(cfg, world):
    S, L, H = cfg["sequences"], cfg["layers"], cfg["hidden"]
    return {"workload": (f"{cfg['name']}: {L} stacked KDA+MoE layers, {S} sequences x (anchor + {cfg['drafts']} "
                         f"drafts), LM head V={cfg['vocab']}, greedy acceptance"
                         + (f", Zipf({cfg['zipf']}) expert bias" if cfg.get("zipf") else "")),
            "hidden": H, "experts": cfg["experts"], "top_k": cfg["top_k"], "inter": cfg["inter"],
            "shared_inter": cfg["shared_inter"], "heads": cfg["heads"], "head_dim": cfg["head_dim"],
            "sequences_x_drafts": f"{S}x{cfg['drafts']}", "verify_positions": S * (cfg["drafts"] + 1),
            "layers": L, "vocab": cfg["vocab"], "seed": cfg["seed"],
            "parallelism": (f"expert parallel x{world} (experts {cfg['experts'] // world} per GPU"
                            + (", dealt by routing bias (k3xb_ep_balance)" if cfg.get("zipf") else "")
                            + f", {S // world} sequences per GPU, peer-memory exchange)") if world > 1 else "single GPU",
            "l2": "no flush: each step streams tens of GB of weights (>> 126 MB L2)"}


def run_stack(args, rank, world, local, ctx, stream, cfg):
    import numpy as np
    import torch

    import k3xb
    S, p, V, L, H = cfg["sequences"], cfg["drafts"], cfg["vocab"], cfg["layers"], cfg["hidden"]
    N = p + 1
    if S % world or cfg["experts"] % world:
        raise SystemExit(f"{cfg['name']}: sequences ({S}) and experts ({cfg['experts']}) must divide by {world}")
    if world > 1:
        import torch.distributed as dist
        uid = [k3xb.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.ep_init(uid[0], rank, world)
    model, keep = gpu_stack(ctx, torch, cfg, rank, world, args.act_terms)
    Sr = S // world
    mine = slice(rank * Sr, (rank + 1) * Sr)
    tokens = stack_tokens(cfg)[mine]
    conv_all, rec_all = gpu_states(ctx, torch, cfg)
    conv = conv_all[:, mine].contiguous()
    rec = rec_all[:, mine].contiguous()
    del conv_all, rec_all
    tok_d = torch.from_numpy(tokens).cuda()
    drafts_d = torch.from_numpy(np.ascontiguousarray(tokens[:, 1:])).cuda()
    logits = torch.empty((Sr, N, V), dtype=torch.float32, device="cuda")
    acc = torch.zeros(Sr, dtype=torch.int32, device="cuda")
    com = torch.zeros((Sr, N), dtype=torch.int32, device="cuda")
    cnt = torch.zeros(Sr, dtype=torch.int32, device="cuda")
    io = k3xb.verify_io_desc(Sr, p, conv, rec, acc, com, cnt, drafts_d, tokens=tok_d, logits=logits)

    def step():
        # each step verifies the same drafts from the state the previous one
        # committed: the same work every step
        if world > 1:
            ctx.ep_verify_step(model, io, cfg["experts"])
        else:
            ctx.verify_step(model, io)

    for _ in range(args.warmup):
        step()
    ctx.sync()
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
    ctx.sync()
    launches = (ctx.stats()["kernel_launches"] - launches0)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    accepted = int(acc.sum().item())
    committed = int(cnt.sum().item())
    # e2e: pinned host tokens and drafts in, acceptance results out, through the same call
    tok_h = torch.from_numpy(tokens).pin_memory()
    dr_h = torch.from_numpy(np.ascontiguousarray(tokens[:, 1:])).pin_memory()
    out_h = [torch.empty_like(t, device="cpu").pin_memory() for t in (acc, com, cnt)]

    def e2e_step():
        tok_d.copy_(tok_h, non_blocking=True)
        drafts_d.copy_(dr_h, non_blocking=True)
        step()
        for hbuf, dbuf in zip(out_h, (acc, com, cnt)):
            hbuf.copy_(dbuf, non_blocking=True)

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
    h2d = tokens.size * 4 + Sr * p * 4
    d2h = (Sr + Sr * N + Sr) * 4
    # the expert FFN (gate/up + down) of every layer, timed live with the
    # library's CUDA events on its own stream over extra eager steps
    prof = phase_profile(ctx, torch, step, max(3, min(args.steps, 5)))
    ph = prof["ms_per_step"]
    ffn_ms = ph.get("expert_gateup", 0.0) + ph.get("expert_down", 0.0)
    units = S * p * L
    hbm, peak_kind = peaks()
    E, E_r = cfg["experts"], cfg["experts"] // world
    # algorithmic bytes of the expert FFN per step on this rank: each expert
    # a layer's S*(p+1) positions x top_k slots reach, once per layer. With
    # uniform routing an expert goes unused with probability
    # (1 - k/E)^(S(p+1)): 0.2% at c4, ~1e-10 at c5 (whose bias only
    # concentrates routing further), so the expected count is used.
    used = E_r * (1.0 - (1.0 - cfg["top_k"] / E) ** (S * N))
    ffn_bytes = L * used * EXPERT_BYTES
    ffn_achieved = ffn_bytes / (ffn_ms * 1e-3) / 1e9 if ffn_ms > 0 else None
    P, h, d = cfg["heads"] * cfg["head_dim"], cfg["heads"], cfg["head_dim"]
    kda_bytes = (4 * P * H + d * H + P * d + h * H + H * P) * 2
    dense_bytes = cfg["experts"] * H * 2 + 3 * cfg["shared_inter"] * H * 2
    step_bytes = L * (kda_bytes + dense_bytes + used * EXPERT_BYTES) + V * H * 2 + Sr * N * V * 4
    step_achieved = step_bytes / (ms * 1e-3) / 1e9
    result = {
        "metric": METRIC, "value": units / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "mxfp4",
        "data": "synthetic (seeded; generated in HBM by the library's generator)",
        "config": stack_config(cfg, world),
        "e2e": {"value": units / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms},
        "roofline": {"bound": "hbm", "kernel": "expert FFN (gateup_kernel + down_kernel), every layer",
                     "achieved": ffn_achieved, "peak": hbm, "unit": "GB/s",
                     "frac": ffn_achieved / hbm if ffn_achieved else None,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "alg_bytes_per_step": ffn_bytes, "experts_per_layer_expected": used,
                     "ffn_ms_per_step": ffn_ms, "traffic": ffn_bytes * EXPERT_TRAFFIC_RATIO,
                     "traffic_source": "ncu dram__bytes_read+write per algorithmic byte of gate/up (64x96) and down (128x24), "
                                       "scaled by the experts streamed (profiles/expert_ffn_traffic_128x24.md)",
                     "whole_step": {"alg_bytes": step_bytes, "achieved": step_achieved,
                                    "frac": step_achieved / hbm}},
        "gpu_launches": launches, "clocks": clk.summary(), "mxf4_act_terms": cfg["terms"],
        "accepted_tokens_per_s": sum_over_ranks(accepted, world) / (ms * 1e-3),
        "committed_tokens_per_s": sum_over_ranks(committed, world) / (ms * 1e-3),
        "phases": prof,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg["name"])
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        ctx.ep_finalize()


# ---- c2: one MoE layer ---------------------------------------------------------------------

def c2_config(cfg, parallelism):
    return {"workload": "c2: single released-shape MoE layer, expert-major verify"
            + ("" if (cfg["experts"], cfg["tokens"]) == (C2["experts"], C2["tokens"])
               else f" (reduced: {cfg['experts']} experts, {cfg['tokens']} tokens)"),
            "hidden": cfg["hidden"], "experts": cfg["experts"], "top_k": cfg["top_k"], "inter": cfg["inter"],
            "shared_inter": cfg["shared_inter"], "verify_tokens": cfg["tokens"], "sequences_x_drafts": "8x8",
            "layers": 1, "seed": cfg["seed"], "parallelism": parallelism,
            "l2": "no flush: each step streams ~8 GB of expert weights (>> 126 MB L2)"}


def make_c2_layer(ctx, torch, cfg, engine, act_terms, rank=0, world=1):
    import k3xb
    w = gpu_moe(ctx, torch, cfg, cfg["seed"], rank, world)
    words = gpu_tensor(ctx, torch, ("bf16", (cfg["tokens"], cfg["hidden"]), cfg["seed"], 30, 1.0))
    hidden = (words.to(torch.int32) << 16).view(torch.float32).contiguous()
    return w, k3xb.moe_layer_desc(w, engine=engine, act_terms=act_terms), hidden


def run_c2(args, rank, world, local, ctx, stream, cfg):
    """One released-shape MoE layer over 64 verify tokens; at N > 1 expert
    parallel (each rank holds E/N experts and 64/N tokens)."""
    import ctypes as C

    import torch

    import k3xb
    T, H, K, E = cfg["tokens"], cfg["hidden"], cfg["top_k"], cfg["experts"]
    if T % world or E % world:
        raise SystemExit(f"c2 needs tokens ({T}) and experts ({E}) divisible by {world}")
    engine = k3xb.ENGINE_SIMT if args.engine == "simt" else k3xb.ENGINE_MXF4
    if world > 1:
        import torch.distributed as dist
        uid = [k3xb.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.ep_init(uid[0], rank, world)
    w, desc, hidden = make_c2_layer(ctx, torch, cfg, engine, args.act_terms, rank, world)
    Tr = T // world
    x = hidden[rank * Tr:(rank + 1) * Tr].contiguous()
    out = torch.empty((Tr, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((Tr, K), dtype=torch.int32, device="cuda")
    con = torch.empty((Tr, K), dtype=torch.float32, device="cuda")

    def step():
        if world > 1:
            ctx.ep_moe_layer_forward(desc, E, x, out, ids, con)
        else:
            ctx.moe_layer_forward(desc, x, out, ids, con)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    if world > 1:
        import torch.distributed as dist
        all_ids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(all_ids, ids)
        unique = int(torch.unique(torch.cat(all_ids)).numel())
    else:
        unique = int(torch.unique(ids).numel())
    l0 = ctx.stats()["kernel_launches"]
    step()
    torch.cuda.synchronize()
    per_step = ctx.stats()["kernel_launches"] - l0
    run = step
    used_graph = False
    if world == 1 and not args.no_graph:   # one GPU, no collectives: replay a CUDA graph
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        torch.cuda.synchronize()
        run, used_graph = g.replay, True
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            run()
        ev1.record(stream)
        torch.cuda.synchronize()
    ctx.sync()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    # the expert FFN timed alone on the same stream (one GPU)
    exp_ms = None
    if world == 1:
        plan = dict(group_expert=torch.empty(E, dtype=torch.int32, device="cuda"),
                    group_offset=torch.empty(E + 1, dtype=torch.int32, device="cuda"),
                    assign_token=torch.empty(T * K, dtype=torch.int32, device="cuda"),
                    assign_slot=torch.empty(T * K, dtype=torch.int32, device="cuda"),
                    assign_contrib=torch.empty(T * K, dtype=torch.float32, device="cuda"),
                    group_count=torch.empty(1, dtype=torch.int32, device="cuda"),
                    status=torch.zeros(1, dtype=torch.int32, device="cuda"))
        ctx.expert_major_plan(ids, con, E, plan)
        slot_out = torch.empty((T * K, H), dtype=torch.float32, device="cuda")
        pl = k3xb.Plan(*(k3xb._p(plan[k]) for k in ("group_expert", "group_offset", "assign_token", "assign_slot",
                                                      "assign_contrib", "group_count", "status")))

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
    # e2e through the host-buffer entry point (one GPU) or with host copies around the EP call
    h_host = x.cpu().pin_memory()
    o_host = torch.empty((Tr, H), dtype=torch.float32).pin_memory()
    i_host = torch.empty((Tr, K), dtype=torch.int32).pin_memory()
    c_host = torch.empty((Tr, K), dtype=torch.float32).pin_memory()

    def e2e_step():
        if world == 1:
            ctx.moe_layer_forward_host(desc, h_host, o_host, i_host, c_host)
        else:
            x.copy_(h_host, non_blocking=True)
            step()
            o_host.copy_(out, non_blocking=True)
            i_host.copy_(ids, non_blocking=True)
            c_host.copy_(con, non_blocking=True)

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
    alg_bytes = unique * EXPERT_BYTES + T * H * 2 + T * H * 4
    timed = exp_ms if exp_ms else ms
    achieved = alg_bytes / (timed * 1e-3) / 1e9 / world
    result = {
        "metric": METRIC, "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "mxfp4",
        "data": "synthetic (seeded; generated in HBM by the library's generator)",
        "config": c2_config(cfg, f"expert parallel x{world}" if world > 1 else "single GPU"),
        "cuda_graph": used_graph,
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4 + 2 * T * K * 4},
        "roofline": {"bound": "hbm", "kernel": "expert FFN" + (" (timed alone)" if exp_ms else " (whole layer, per GPU)"),
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "alg_bytes_per_launch": alg_bytes, "unique_experts": unique, "launch_ms": timed,
                     "traffic": unique * EXPERT_BYTES * EXPERT_TRAFFIC_RATIO,
                     "traffic_source": "ncu dram__bytes_read+write per algorithmic byte of gate/up (64x96) and down (128x24), "
                                       "scaled by unique experts (profiles/expert_ffn_traffic_128x24.md)"},
        "gpu_launches": per_step * args.steps, "clocks": clk.summary(), "engine": args.engine,
        "mxf4_act_terms": args.act_terms or k3xb.default_act_terms(T * K, E),
    }
    if args.profile:
        result["phases"] = phase_profile(ctx, torch, step, max(3, args.steps))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline("c2")
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        ctx.ep_finalize()


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
    bf = lambda stream, *shape: (gpu_tensor(ctx, torch, ("bf16", shape, cfg["seed"], stream, 1.0)).to(torch.int32)
                                 << 16).view(torch.float32).contiguous()
    f32 = lambda stream, *shape: gpu_tensor(ctx, torch, ("f32", shape, cfg["seed"], stream, 1.0, 0.0))
    q, k, v = bf(1, S, Nn, P), bf(2, S, Nn, P), bf(3, S, Nn, P)
    # q, k L2-normalised per head (official_kda.cpp:259-290: q also x 1/sqrt(d))
    k = (k.view(S, Nn, h, d) / k.view(S, Nn, h, d).norm(dim=-1, keepdim=True)).view(S, Nn, P).contiguous()
    q = (q.view(S, Nn, h, d) / q.view(S, Nn, h, d).norm(dim=-1, keepdim=True) / d ** 0.5).view(S, Nn, P).contiguous()
    ld = torch.nn.functional.logsigmoid(f32(4, S, Nn, P)).contiguous()
    beta = torch.sigmoid(f32(5, S, Nn, h)).contiguous()
    # prefix state: the recurrence over a 1024-token linear prefix from zero
    T0 = cfg["prefix"]
    pq, pk, pv = bf(6, S, T0, P), bf(7, S, T0, P), bf(8, S, T0, P)
    pk = (pk.view(S, T0, h, d) / pk.view(S, T0, h, d).norm(dim=-1, keepdim=True)).view(S, T0, P).contiguous()
    pld = torch.nn.functional.logsigmoid(f32(9, S, T0, P)).contiguous()
    pbe = torch.sigmoid(f32(10, S, T0, h)).contiguous()
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


def run_attnres(args, rank, world, local, ctx, stream):
    """The block attention residual with many sources (model.cpp:645-666)
    over c5's 576 verify positions at H 7168, with `--sources` block
    sources (default 8). HBM-bound: every value row is read once and the
    output written once."""
    import torch
    T, H, S = C5["sequences"] * (C5["drafts"] + 1), C5["hidden"], args.sources
    values = gpu_tensor(ctx, torch, ("f32", (S + 1, T, H), 11, 1, 1.0, 0.0))
    norm = gpu_tensor(ctx, torch, ("f32", (H,), 11, 2, 0.1, 1.0))
    proj = gpu_tensor(ctx, torch, ("f32", (H,), 11, 3, 3.0 / H ** 0.5, 0.0))
    sources, prefix = (values[:S] if S else None), values[S]
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    eps = 1e-6

    def step():
        ctx.block_attention_residual(prefix, sources, norm, proj, eps, out)

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
    ctx.sync()
    ms = max_over_ranks(statistics.mean(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)), world)
    alg = (S + 2) * T * H * 4 + 2 * H * 4
    # DRAM bytes per algorithmic byte from one ncu capture of this command at
    # the default 8 sources (profiles/block_attnres_576x9.md): (249.28 + 8.14)
    # MB over 165.21 MB; other source counts were not captured
    traffic = alg * (249.280 + 8.138) / 165.208 if S == 8 else None
    hbm, peak_kind = peaks()
    result = {
        "metric": "attention-residual positions/s", "value": sum_over_ranks(T, world) / (ms * 1e-3),
        "unit": "positions/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (FP64 score sums)",
        "data": "synthetic (seeded, generated on the GPU)",
        "config": {"workload": "block attention residual over many sources", "positions": T, "hidden": H,
                   "sources": S, "l2": "flushed (256 MB write) before every timed step"},
        "roofline": {"bound": "hbm", "kernel": "block_attnres_kernel", "achieved": alg / (ms * 1e-3) / 1e9,
                     "peak": hbm, "unit": "GB/s", "frac": alg / (ms * 1e-3) / 1e9 / hbm,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})", "alg_bytes_per_launch": alg,
                     "traffic": traffic},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = attnres_cpu_baseline(S)
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_tc_sweep(args, rank, world, local, ctx, stream):
    """Tensor-core sweep of the expert GEMM: 8 experts x M tokens each (Top-8
    of 8, so every token uses every expert) for M in {256, 1024, 4096}, c2
    expert shapes. Reports useful TFLOP/s (2 * T * k * 3 * H * I per call)
    and the MMA work, which is `terms` times larger because each activation
    row enters as E2M1 terms."""
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
        terms = args.act_terms or k3xb.default_act_terms(T * K, E)
        lines.append({"tokens_per_expert": M, "ms": ms, "act_terms": terms,
                      "useful_tflops": useful / (ms * 1e-3) / 1e12, "mma_tflops": useful * terms / (ms * 1e-3) / 1e12})
        del w, desc, hidden, slot_out
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"metric": "expert GEMM tensor-core sweep (useful TFLOP/s)", "config":
                          {"workload": "8 experts x M tokens, Top-8 of 8, H 7168, I 2048, MXFP4",
                           "act_terms": args.act_terms or "library default"}, "sweep": lines,
                          "peak_note": "mxf4 dense peak 9 PFLOP/s nominal; MMA work = terms x useful"}), flush=True)


def run_ours(args):
    import torch

    import k3xb
    rank, world, local = dist_setup()
    torch.cuda.set_device(local)
    ctx = k3xb.Context(local)
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx.use_stream(stream)
    try:
        if args.config in ("c4", "c5"):
            cfg = dict(C5 if args.config == "c5" else C4, name=args.config)
            cfg["terms"] = args.act_terms or k3xb.default_act_terms(cfg["sequences"] * (cfg["drafts"] + 1) * cfg["top_k"],
                                                                  cfg["experts"])
            run_stack(args, rank, world, local, ctx, stream, cfg)
        elif args.config == "c3":
            run_c3(args, rank, world, local, ctx, stream)
        elif args.config == "tc":
            run_tc_sweep(args, rank, world, local, ctx, stream)
        elif args.config == "attnres":
            run_attnres(args, rank, world, local, ctx, stream)
        else:
            cfg = dict(C2)
            if args.experts:   # reduced c2 case for profiler captures (a few GB on the device)
                cfg["experts"] = args.experts
            if args.tokens:
                cfg["tokens"] = args.tokens
            run_c2(args, rank, world, local, ctx, stream, cfg)
    finally:
        ctx.close()
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def run_reference_attnres(args):
    """--impl reference --config attnres: the port (the reference's function
    is private to its engine) on all host threads, same metric and config."""
    sample = AttnResSample(args.sources)
    times = []
    for i in range(args.warmup + args.steps):
        dt = sample.step()
        if i >= args.warmup:
            times.append(dt)
    dt = statistics.mean(times)
    value = sample.units() / dt
    print(json.dumps({
        "impl": "reference", "metric": "attention-residual positions/s", "value": value, "unit": "positions/s",
        "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (FP64 squares; the reference's float chains)",
        "data": "synthetic (the same spec, built on the host by the generator's restatement)",
        "config": {"workload": "block attention residual over many sources", "positions": sample.T,
                   "hidden": C5["hidden"], "sources": sample.S,
                   "l2": "flushed (256 MB write) before every timed step"},
        "cpu_baseline": {"value": value, "unit": "positions/s", "cores": len(sample.chunks), "kind": "port",
                         "sample": sample.describe(dt)},
        "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference(args):
    """--impl reference: the reference's own CPU implementation of the path
    (oracle/_ref), on this host's cores, on a bounded sample of the same
    workload (the same spec, built on the host). Rank 0 alone runs."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.config in ("c3", "tc"):
        print(json.dumps({"impl": "reference", "unavailable": f"--config {args.config} has no reference CPU path "
                                                              "(the reference has no draft tree and no tensor cores)"}))
        return
    if args.config == "attnres":
        run_reference_attnres(args)
        return
    sample = reference_sample(args.config)
    if sample is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libk3x_ref.so was not built"}))
        return
    times = []
    for i in range(args.warmup + args.steps):
        dt = sample.step()
        if i >= args.warmup:
            times.append(dt)
    dt = statistics.mean(times)
    value = sample.units() / dt
    if args.config == "c2":
        config = c2_config(dict(C2), f"{sample.n} host threads")
    else:
        cfg = dict(C5 if args.config == "c5" else C4, name=args.config)
        config = stack_config(cfg, 1)
        config["parallelism"] = f"{sample.n} host threads"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32/fp64 (reference CPU)",
        "data": "synthetic (the same spec, built on the host by the generator's restatement)", "config": config,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": sample.n, "kind": "reference",
                         "sample": sample.describe(dt) + f"; built on the host in {sample.build_s:.1f} s"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--engine", choices=["mxf4", "simt"], default=os.environ.get("K3XB_ENGINE", "mxf4"))
    ap.add_argument("--act-terms", type=int, default=0,
                    help="E2M1 activation terms of the MXF4 engine (0: the library default, k3xb_default_act_terms)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", choices=["c5", "c4", "c2", "c3", "tc", "attnres"], default="c5",
                    help="c5 (default: 8-layer KDA+MoE verify step, expert parallel at N > 1), c4 (2 layers), "
                         "c2 (one MoE layer), c3 (KDA draft tree), tc (tensor-core sweep of the expert GEMM)")
    ap.add_argument("--sequences", type=int, default=1, help="c3: sequences sharing the draft tree")
    ap.add_argument("--sources", type=int, default=8, help="attnres: block sources besides the prefix")
    ap.add_argument("--experts", type=int, default=0, help="c2 with fewer experts (small profiler case)")
    ap.add_argument("--tokens", type=int, default=0, help="c2 with another verify-token count")
    ap.add_argument("--no-graph", action="store_true", help="c2: time eager launches instead of a CUDA graph")
    ap.add_argument("--profile", action="store_true", help="c2: add per-phase device times to the JSON line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
