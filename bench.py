"""Benchmark of the MoE-expert decode hot path (BASELINE config 1 on one B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one MoE-layer forward (router -> top-k -> gate/up dequant-GEMV +
SwiGLU -> down dequant-GEMV + weighted combine + shared expert) over one batch
of T seeded bf16 tokens, on the DeepSeek-V3-shape layer of config 1 (H 7168,
256 routed + 1 shared experts, top-8, I 2048, 4-bit g64 MLX affine). Weights
of several distinct seeded layers are resident and steps cycle through them,
so every step streams a different layer's experts (>= 227 MB, larger than
L2) — no L2 flush is needed.

Prints one JSON line (rank 0). `value` is tokens/s over the timed steps with
inputs resident in HBM; `e2e` is the same metric through the host-buffer
C-ABI call (pinned host x in, host out, copies inside the timed region);
`roofline` is for the dominant kernel (gate/up GEMV), from CUDA events on the
launching stream; `cpu_baseline` times the CPU oracle on the host cores.
Under torchrun (N > 1) the layer is expert-parallel: rank r holds routed
experts [r*E/N, (r+1)*E/N) of every layer and T tokens of an N*T-token
global batch (weak scaling: T per GPU fixed). The token exchange is one of
three modes: NCCL all-gather of the tokens with the router over all of them;
the same with an NCCL reduce-scatter of per-token sums; or a peer all-to-all
dispatch of each token to the GPUs holding its experts. In the fused modes
the rank's down GEMV stores each routed partial straight into the token's
home GPU over NVLink, followed by the shared expert and the slot-ordered
combine there. `--ep-mode auto` (default) times the three on the headline
batch after warm-up and runs the headline in the fastest; `ep_modes` reports
all three. The time is the max over ranks; `value` counts all N*T tokens.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "minirun-app_b200"))

METRIC = ("MoE-layer decode tokens/s; dequant-GEMV HBM GB/s (% of ~8 TB/s) at 1/2/4/8 GPUs")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# kernels one layer forward launches: logits(+prep), top-k(+plan), gate/up, down, combine.
# Expert parallel (NCCL collectives not counted): all-gather modes: logits, top-k, routed
# gate/up and down, shared gate/up and down, wait+combine (+ the partial-sum kernel on the
# NCCL path); all-to-all: logits, top-k, dispatch plan, dispatch copy, receive, prep, plan,
# routed gate/up and down, shared gate/up and down, wait+combine
LAUNCHES_PER_STEP = 5
LAUNCHES_PER_STEP_EP = {"allgather": 7, "nccl": 8, "alltoall": 12}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--layers", type=int, default=4, help="distinct resident layers cycled")
    p.add_argument("--sweep", default="1,8", help="extra token counts measured (no e2e)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--experts", type=int, default=0,
                   help="routed experts (0 = config 1's 256); smaller values only for "
                        "profiling captures that must fit a few GB")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--kernel-path", choices=["auto", "register", "tma", "umma", "v2"],
                   default="auto",
                   help="dequant-GEMV implementation (mr_ctx_set_kernel_path)")
    p.add_argument("--prefill-tokens", type=int, default=4096,
                   help="config-3 prefill batch measured beside the decode line (0 = skip)")
    p.add_argument("--k3-tokens", default="1,16",
                   help="token counts of the K3 latent-MoE layer line ('' = skip)")
    p.add_argument("--k3-experts", type=int, default=896,
                   help="routed experts of the K3 layer (flagship: 896)")
    p.add_argument("--ep-nccl", action="store_true",
                   help="expert parallel: NCCL reduce-scatter instead of the fused peer stores "
                        "(same as --ep-mode nccl)")
    p.add_argument("--ep-mode", choices=["auto", "allgather", "nccl", "alltoall"],
                   default="auto",
                   help="expert-parallel token exchange: NCCL all-gather + fused peer combine, "
                        "NCCL all-gather + reduce-scatter, or peer all-to-all dispatch + fused "
                        "peer combine; auto (default) times each on the headline batch after "
                        "warm-up and runs the headline in the fastest")
    p.add_argument("--no-ep-compare", action="store_true",
                   help="N > 1: skip timing the other exchange modes beside the headline")
    p.add_argument("--config", default="1", choices=["1", "2b2", "2b8"],
                   help="decode layer: config 1 (the headline) or config 2's wide 2-/8-bit "
                        "layers (384 experts)")
    p.add_argument("--cache-layers", type=int, default=0,
                   help="config 4: budgeted decode through this many layers via the HBM "
                        "expert cache (58 in BASELINE; 0 = skip)")
    p.add_argument("--cache-budget-gb", type=float, default=40.0,
                   help="config 4: HBM byte budget of the expert cache")
    p.add_argument("--cache-only", action="store_true",
                   help="measure only the config-4 cached decode line")
    p.add_argument("--k3-only", action="store_true",
                   help="measure only the K3 latent-MoE layer (profiling driver)")
    p.add_argument("--strong-tokens", type=int, default=64,
                   help="global batch of the strong-scaling line (64 / N tokens per GPU)")
    p.add_argument("--no-parity", action="store_true",
                   help="skip the in-run correctness check (oracle / one-GPU comparison)")
    p.add_argument("--parity-tokens", type=int, default=4,
                   help="tokens of every rank's batch checked against the CPU oracle")
    p.add_argument("--config2-tokens", type=int, default=64,
                   help="config-2 sub-line (2-/8-bit, 384 experts) at this global batch "
                        "(0 = skip)")
    p.add_argument("--config4-layers", type=int, default=8,
                   help="config-4 sub-line: budgeted decode through this many layers, budget "
                        "scaled from 40 GB for 58 layers (0 = skip)")
    p.add_argument("--config4-budget-gb", type=float, default=0.0,
                   help="config-4 sub-line budget (0 = 40 GB * layers / 58)")
    p.add_argument("--config4-ep-layers", type=int, default=58,
                   help="N >= 4: config-4 decode with every expert resident across the GPUs "
                        "(all-to-all mode, the token on GPU 0), this many layers (0 = skip)")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s (burst: the kernels are timed alone)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------- ours

def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist

    import minirun_moe as M
    from minirun_moe import synth as S

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))
    spec = S.CONFIGS[1 if args.config == "1" else args.config]
    if args.experts:
        import dataclasses
        spec = dataclasses.replace(spec, experts=args.experts)
    T = args.tokens
    NL = max(1, args.layers)
    # N > 1: expert parallelism, rank r holds experts [r*E/N, (r+1)*E/N) of
    # every layer; its T tokens are rows r*T.. of the seeded global batch
    ep = world > 1
    e0, e1 = (rank * spec.experts // world, (rank + 1) * spec.experts // world)
    layers = [S.synth_layer(spec, layer=l, device=local, shard=(rank, world) if ep else None)
              for l in range(NL)]
    NB = NL + 1
    # strong scaling: 64 tokens in the global batch whatever N is (64 / N per rank)
    Ts = args.strong_tokens // world if args.strong_tokens % world == 0 else 0
    token_counts = [T] + [int(t) for t in args.sweep.split(",") if t and int(t) != T]
    if Ts and Ts not in token_counts:
        token_counts.append(Ts)

    def xrows(t, b):
        full = S.synth_x(spec, t * world, layer=0, batch=b, device=local)
        return full[rank * t:(rank + 1) * t].contiguous()

    xs = {t: [xrows(t, b) for b in range(NB)] for t in token_counts}
    ctx = M.Context.get(local)
    ctx.set_kernel_path(args.kernel_path)
    if args.ep_nccl:
        args.ep_mode = "nccl"
    group = M.ExpertGroup(local, rank, world) if ep else None
    auto_mode = args.ep_mode == "auto"
    if auto_mode:
        args.ep_mode = "alltoall"  # until the probe below has measured the modes
    if group is not None:
        group.set_mode(args.ep_mode)
    torch.cuda.synchronize()

    def step(lay, x, out, ids=None):
        if ep:
            group.forward(lay, x, out=out, ids=ids)
        elif ids is None:
            lay.forward(x, out=out, selection=False)
        else:
            _, sel = lay.forward(x, out=out)
            ids.copy_(sel.ids)

    def barrier():
        if world > 1:
            dist.barrier()

    def schedule(i):
        return layers[i % NL], i % NB

    def max_over_ranks(v):
        if world > 1:
            t = torch.tensor([v], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = float(t.item())
        return v

    def timed(tok, steps, warm):
        outs = torch.empty((tok, spec.hidden), dtype=torch.bfloat16, device=dev)
        for i in range(warm):
            lay, b = schedule(i)
            step(lay, xs[tok][b], outs)
        torch.cuda.synchronize()
        barrier()
        st = torch.cuda.current_stream()
        a = torch.cuda.Event(enable_timing=True)
        z = torch.cuda.Event(enable_timing=True)
        a.record(st)
        for i in range(steps):
            lay, b = schedule(i)
            step(lay, xs[tok][b], outs)
        z.record(st)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(a.elapsed_time(z))

    def distinct_experts(tok, steps):
        """Distinct routed experts this GPU streams per step (its own range,
        selected by any token of the global batch)."""
        us = []
        outs = torch.empty((tok, spec.hidden), dtype=torch.bfloat16, device=dev)
        ids = torch.empty((tok, spec.top_k), dtype=torch.int32, device=dev)
        for i in range(steps):
            lay, b = schedule(i)
            step(lay, xs[tok][b], outs, ids)
            allids = ids
            if ep:
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                allids = torch.cat(parts)
            us.append(len({e for e in allids.cpu().view(-1).tolist() if e0 <= e < e1}))
        return us

    def step_bytes(tok, U):
        eb = spec.expert_bytes()
        return (U + 1) * eb + spec.router_bytes() + 2 * tok * spec.hidden * 2

    def gate_up_bytes(tok, U):
        return ((U + 1) * 2 * spec.proj_bytes(spec.inter, spec.hidden) + tok * spec.hidden * 2
                + (tok * spec.top_k + 2 * tok) * spec.inter * 2)

    hbm, peak_kind = peaks()
    K, W = args.steps, max(3, args.warmup)

    def phases(tok):
        """Per-step device time of each kernel class (CUDA events around each
        launch on the launching stream, max over ranks), and the gate/up
        roofline of this GPU's share."""
        ctx.profile(True)
        timed(tok, K, 0)
        prof = ctx.profile_read()
        ctx.profile(False)
        per = {k: {"ms_per_step": max_over_ranks(v[0] / K), "launches_per_step": v[1] / K}
               for k, v in prof.items() if v[1]}
        return prof, per

    # expert parallel, --ep-mode auto: every exchange mode on the headline
    # batch (same steps and warm-up as the headline, max over ranks, so every
    # rank picks the same), then the headline in the fastest
    mode_probe = None
    if ep and auto_mode:
        mode_probe = {}
        for mode in ("allgather", "nccl", "alltoall"):
            group.set_mode(mode)
            mode_probe[mode] = world * T * K / (timed(T, K, W) / 1e3)
        args.ep_mode = max(mode_probe, key=mode_probe.get)
        group.set_mode(args.ep_mode)

    with ClockSampler(local) as clk:
        ms = timed(T, K, W)
    clocks = clk.summary()
    us = distinct_experts(T, K)
    avg_bytes = sum(step_bytes(T, u) for u in us) / len(us)
    ms_step = ms / K
    value = world * T * K / (ms / 1e3)

    # per-kernel durations (CUDA events around each launch, same stream)
    prof, per_phase = phases(T)
    # gate/up time per step (expert-parallel steps launch it twice: the
    # rank's routed experts, then the shared expert) against its bytes per step
    gu_ms, gu_n = prof["gate_up"]
    gu_step_ms = gu_ms / K
    gu_bytes = sum(gate_up_bytes(T, u) for u in us) / len(us)
    achieved = gu_bytes / (gu_step_ms / 1e3) / 1e9
    kern = {k: {"ms_per_launch": v[0] / max(v[1], 1), "launches": v[1]} for k, v in prof.items()}
    # the ncu traffic summary is of the config-1 (4-bit) kernel
    traffic = read_traffic(gu_bytes) if args.config == "1" else None

    sweep = {}
    for tok in token_counts[1:]:
        m2 = timed(tok, K, W)
        u2 = distinct_experts(tok, K)
        b2 = sum(step_bytes(tok, u) for u in u2) / len(u2)
        sweep[str(tok)] = {"tokens_per_s": world * tok * K / (m2 / 1e3),
                           "ms_per_step": m2 / K,
                           "layer_gbs": b2 / (m2 / K / 1e3) / 1e9,
                           "layer_frac_of_hbm": b2 / (m2 / K / 1e3) / 1e9 / hbm,
                           "distinct_experts_avg": sum(u2) / len(u2)}

    # strong scaling: the same 64-token global batch on N GPUs, with its
    # per-phase split and, at N > 1, a one-GPU run of the whole layer on rank 0
    # in this same job (the speed-up is measured, not inferred across runs)
    strong = None
    full_layers = None
    if Ts:
        sw = sweep.get(str(Ts)) if Ts != T else {"tokens_per_s": value, "ms_per_step": ms_step,
                                                 "distinct_experts_avg": sum(us) / len(us)}
        sprof, sper = phases(Ts) if Ts != T else (prof, per_phase)
        su = distinct_experts(Ts, K) if Ts != T else us
        sgu = sum(gate_up_bytes(Ts, u) for u in su) / len(su)
        s_gu_ms = max_over_ranks(sprof["gate_up"][0] / K)
        strong = {"global_tokens": args.strong_tokens, "tokens_per_rank": Ts,
                  "tokens_per_s": sw["tokens_per_s"], "ms_per_step": sw["ms_per_step"],
                  "distinct_experts_per_gpu_avg": sum(su) / len(su),
                  "gate_up_frac_of_hbm_per_gpu": sgu / (s_gu_ms / 1e3) / 1e9 / hbm,
                  "phases_ms_per_step": {k: v["ms_per_step"] for k, v in sper.items()}}
        if world > 1:
            one = None
            if rank == 0:
                full_layers = [S.synth_layer(spec, layer=l, device=local) for l in range(NL)]
                x1 = [S.synth_x(spec, args.strong_tokens, layer=0, batch=b, device=local)
                      for b in range(NB)]
                o1 = torch.empty((args.strong_tokens, spec.hidden), dtype=torch.bfloat16,
                                 device=dev)
                for i in range(W):
                    full_layers[i % NL].forward(x1[i % NB], out=o1, selection=False)
                torch.cuda.synchronize()
                a = torch.cuda.Event(enable_timing=True)
                z = torch.cuda.Event(enable_timing=True)
                a.record()
                for i in range(K):
                    full_layers[i % NL].forward(x1[i % NB], out=o1, selection=False)
                z.record()
                torch.cuda.synchronize()
                one = args.strong_tokens * K / (a.elapsed_time(z) / 1e3)
            barrier()
            if rank == 0:
                strong["one_gpu_tokens_per_s"] = one
                strong["speedup_vs_one_gpu"] = strong["tokens_per_s"] / one

    parity = guarded("parity", parity_check, args, spec, S, M, torch, dist, world, rank, local,
                     dev, layers, full_layers, step, xs, T) if not args.no_parity else None
    if full_layers is not None:
        del full_layers
        torch.cuda.empty_cache()

    prefill = None
    # the exchange modes side by side (same run, same inputs): T per GPU and
    # the strong-scaling batch
    ep_modes = None
    if ep and not args.no_ep_compare:
        ep_modes = {}
        for mode in ("allgather", "nccl", "alltoall"):
            group.set_mode(mode)
            row = {}
            for tok in sorted({T, Ts} - {0}):
                m3 = timed(tok, K, W)
                row[str(tok)] = {"tokens_per_s": world * tok * K / (m3 / 1e3),
                                 "ms_per_step": m3 / K}
            ep_modes[mode] = row
        group.set_mode(args.ep_mode)
        # the strong-scaling batch in whichever exchange mode measured fastest
        # in this run (the line above it is in the default mode)
        if strong is not None and str(Ts) in ep_modes[args.ep_mode]:
            best = max(ep_modes, key=lambda m: ep_modes[m][str(Ts)]["tokens_per_s"])
            bt = ep_modes[best][str(Ts)]["tokens_per_s"]
            strong["mode"] = args.ep_mode
            strong["fastest_mode"] = best
            strong["fastest_mode_tokens_per_s"] = bt
            if strong.get("one_gpu_tokens_per_s"):
                strong["fastest_mode_speedup_vs_one_gpu"] = bt / strong["one_gpu_tokens_per_s"]
    if args.prefill_tokens > 0:
        prefill = guarded("prefill", prefill_run, args, S, M, torch, ctx, local, dev, group, world,
                          rank, dist)
    k3 = None
    if not ep and args.k3_tokens:
        k3 = guarded("k3", k3_run, args, M, torch, dev, hbm)
    config2 = None
    if args.config == "1" and args.config2_tokens > 0:
        config2 = guarded("config2", config2_run, args, S, M, torch, dist, world, rank, local, dev,
                          group, hbm, max_over_ranks, barrier)
    config4 = None
    if not ep and args.config4_layers > 0 and args.config == "1":
        config4 = guarded("config4", cache_run, args, M, S, torch, dev,
                          layers_n=args.config4_layers, budget_gb=args.config4_budget_gb,
                          check_identity=True)
    elif ep and world >= 4 and args.config4_ep_layers > 0 and args.config == "1":
        config4 = guarded("config4", config4_ep_run, args, S, M, torch, world, rank, local, dev,
                          group, max_over_ranks, barrier)

    e2e = e2e_run(args, spec, T, K, W, xs, schedule, barrier, world, dev, local,
                  group if ep else None)
    ctx.sync_check()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(T)

    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": f"bf16 activations, {spec.bits}-bit affine weights (u{spec.bits} codes, bf16 "
                 "scale/bias), fp32 "
                 "accumulate",
        "data": "synthetic (SplitMix64-seeded, BASELINE config 1 distributions)",
        "config": {
            "workload": f"config{args.config[0]} decode T={T}: H{spec.hidden}, "
                        f"{spec.experts}+1 experts, top-{spec.top_k}, I{spec.inter}, "
                        f"{spec.bits}-bit g{spec.group}",
            "tokens": T,
            "global_batch": world * T,
            "layers_cycled": NL,
            "l2": "inputs larger than L2: consecutive steps read different layers' experts "
                  "(>= 227 MB each)",
            "exchange_mode": args.ep_mode if ep else None,
            "exchange_mode_probe_tokens_per_s": mode_probe,
            "parallelism": "single GPU" if world == 1 else
                           f"ep{world}: {spec.experts // world} routed experts per GPU, " +
                           {"nccl": "NCCL all-gather of tokens, NCCL reduce-scatter of per-token "
                                    "sums",
                            "allgather": "NCCL all-gather of tokens, down GEMV storing routed "
                                         "partials into their home GPU over NVLink (fused), "
                                         "slot-ordered combine there",
                            "alltoall": "each GPU routes its own tokens and stores their rows "
                                        "into the GPUs holding their experts (NVLink peer "
                                        "all-to-all), down GEMV storing routed partials into "
                                        "their home GPU, slot-ordered combine there"}[args.ep_mode],
            "distinct_experts_avg": sum(us) / len(us),
            "layer_bytes_per_step": avg_bytes,
            "layer_gbs": avg_bytes / (ms_step / 1e3) / 1e9,
            "layer_frac_of_hbm": avg_bytes / (ms_step / 1e3) / 1e9 / hbm,
            "kernels": kern,
            "phases_ms_per_step": {k: v["ms_per_step"] for k, v in per_phase.items()},
            "sweep": sweep,
            "strong_T64": strong,
            "ep_modes": ep_modes,
            "prefill": prefill,
            "k3_latent_moe": k3,
            "config2": config2,
            "config4": config4,
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "gemv gate/up (+SwiGLU)",
            "achieved": achieved,
            "peak": hbm,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / hbm,
            "algorithmic_bytes_per_launch": gu_bytes,
            "launches_per_step": gu_n / K,
            "traffic": traffic,
        },
        "parity": parity,
        "e2e": e2e,
        "gpu_launches": K * (LAUNCHES_PER_STEP_EP[args.ep_mode] if ep else LAUNCHES_PER_STEP),
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        group.close()
        dist.destroy_process_group()


def guarded(name, fn, *a, **k):
    """Runs one optional sub-line; an exception becomes {"error": ...} in the
    JSON line instead of costing the headline (every rank takes the same
    steps, so an error that every rank meets keeps them in step)."""
    try:
        return fn(*a, **k)
    except Exception as e:  # noqa: BLE001 — reported, not swallowed
        print(f"bench: {name} failed: {type(e).__name__}: {e}", file=sys.stderr, flush=True)
        return {"error": f"{type(e).__name__}: {e}"}


def rel_l2(a, b):
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def parity_check(args, spec, S, M, torch, dist, world, rank, local, dev, layers, full_layers,
                 step, xs, T):
    """Correctness of the measured configuration, checked in the same run.

    vs_oracle: the first `--parity-tokens` tokens of every rank's batch (layer
    0, batch 0 of the bench's inputs) against the CPU oracle: expert ids equal
    as sets per token (a difference only where the oracle's margin shows a
    tie below 1e-5) and the outputs within the 1e-2 relative-L2 bound.
    vs_one_gpu (N > 1): the whole global batch of the expert-parallel step
    against the one-GPU layer on rank 0: ids identical and outputs
    bit-identical (fused path) or within 2e-3 (NCCL reduce-scatter path)."""
    import numpy as np
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    out = torch.empty((T, spec.hidden), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((T, spec.top_k), dtype=torch.int32, device=dev)
    step(layers[0], xs[T][0], out, ids)
    torch.cuda.synchronize()
    if world > 1:
        outs = [torch.empty_like(out) for _ in range(world)]
        idss = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(outs, out)
        dist.all_gather(idss, ids)
        gout, gids = torch.cat(outs), torch.cat(idss)
    else:
        gout, gids = out, ids
    res = {"ok": True}
    if rank == 0:
        xg = S.synth_x(spec, T * world, layer=0, batch=0, device=local)
        if world > 1:
            fl = full_layers[0] if full_layers else S.synth_layer(spec, layer=0, device=local)
            ref, sel = fl.forward(xg)
            torch.cuda.synchronize()
            same_ids = bool(torch.equal(torch.sort(sel.ids, 1)[0], torch.sort(gids, 1)[0]))
            bit = bool(torch.equal(ref, gout))
            err = rel_l2(gout.float().cpu().numpy(), ref.float().cpu().numpy())
            exact = args.ep_mode != "nccl"
            ok = same_ids and (bit if exact else err < 2e-3)
            res["vs_one_gpu"] = {"tokens": T * world, "ids_equal": same_ids,
                                 "bit_identical": bit, "rel_l2": err,
                                 "bound": "bit-identical" if exact else 2e-3,
                                 "ok": ok}
            res["ok"] = res["ok"] and ok
            del fl
        if args.config == "1" and args.parity_tokens > 0:
            cfg = O.CONFIGS[1]
            pick = sorted({r * T + j for r in range(world) for j in range(min(args.parity_tokens, T))})
            xn = xg.cpu().view(torch.int16).numpy().view(np.uint16)[pick]
            L = O.gen_layer(cfg, layer=0, experts=O.selected_experts(cfg, xn))
            o_out, o_f, o_ids, o_w, o_m = O.moe_layer_forward(L, xn)
            g = gout.cpu().view(torch.int16).numpy().view(np.uint16)[pick]
            gi = gids.cpu().numpy()[pick]
            flips, bad = 0, 0
            for t in range(len(pick)):
                if set(gi[t].tolist()) != set(o_ids[t].tolist()):
                    if abs(o_m[t]) < 1e-5:
                        flips += 1
                    else:
                        bad += 1
            err = rel_l2(O.bf16_to_f32(g), o_f)
            ok = bad == 0 and err < 1e-2
            res["vs_oracle"] = {"tokens": len(pick), "token_rows": pick[:16],
                                "ids_sets_equal": bad == 0 and flips == 0,
                                "excused_tie_flips": flips, "unexcused_flips": bad,
                                "rel_l2": err, "bound": 1e-2, "ok": ok}
            res["ok"] = res["ok"] and ok
    if world > 1:
        dist.barrier()
    return res if rank == 0 else None


def config2_run(args, S, M, torch, dist, world, rank, local, dev, group, hbm, max_over_ranks,
                barrier):
    """Config 2: the wide layer (384 routed + 1 shared experts, 2-bit and
    8-bit) at `--config2-tokens` global tokens; on N GPUs expert-parallel,
    384 / N experts per GPU (48 at N = 8). Two resident layers alternate so
    that consecutive steps stream different experts."""
    out = {}
    G = args.config2_tokens
    if G % world:
        return None
    t = G // world
    K, W = args.steps, max(3, args.warmup)
    for name in ("2b2", "2b8"):
        spec = S.CONFIGS[name]
        ep = world > 1
        lays = [S.synth_layer(spec, layer=l, device=local, shard=(rank, world) if ep else None)
                for l in range(2)]
        xb = [S.synth_x(spec, G, layer=0, batch=b, device=local)[rank * t:(rank + 1) * t]
              .contiguous() for b in range(3)]
        o = torch.empty((t, spec.hidden), dtype=torch.bfloat16, device=dev)
        ids = torch.empty((t, spec.top_k), dtype=torch.int32, device=dev)

        def fwd(i, want_ids=False):
            lay, x = lays[i % 2], xb[i % 3]
            if ep:
                group.forward(lay, x, out=o, ids=ids if want_ids else None)
            elif want_ids:
                _, sel = lay.forward(x, out=o)
                ids.copy_(sel.ids)
            else:
                lay.forward(x, out=o, selection=False)

        for i in range(W):
            fwd(i)
        torch.cuda.synchronize()
        barrier()
        a = torch.cuda.Event(enable_timing=True)
        z = torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(K):
            fwd(i)
        z.record()
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(a.elapsed_time(z)) / K
        e0, e1 = rank * spec.experts // world, (rank + 1) * spec.experts // world
        us = []
        for i in range(min(K, 6)):
            fwd(i, True)
            allids = ids
            if ep:
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                allids = torch.cat(parts)
            us.append(len({e for e in allids.cpu().view(-1).tolist() if e0 <= e < e1}))
        U = sum(us) / len(us)
        byt = (U + 1) * spec.expert_bytes() + spec.router_bytes() + 2 * t * spec.hidden * 2
        out[name] = {"bits": spec.bits, "tokens_per_s": G / (ms / 1e3), "ms_per_step": ms,
                     "experts_per_gpu": spec.experts // world,
                     "distinct_experts_per_gpu_avg": U,
                     "layer_gbs_per_gpu": byt / (ms / 1e3) / 1e9,
                     "layer_frac_of_hbm_per_gpu": byt / (ms / 1e3) / 1e9 / hbm}
        del lays, xb
        torch.cuda.empty_cache()
    return {"workload": f"config2 decode, {G} global tokens: H7168, 384+1 experts, top-8, "
                        f"I2048, g64; {384 // world} routed experts per GPU",
            "by_bits": out}


def prefill_run(args, S, M, torch, ctx, local, dev, group=None, world=1, rank=0, dist=None):
    """Config 3: one prefill-size batch (T tokens per GPU, Zipf-skewed
    routing) through the same layer call; reports tokens/s and the tcgen05
    GEMMs' TFLOP/s against the dense bf16 peak (tensor-bound). Algorithmic
    FLOPs: 2*H*I per (token, expert) and projection, over the k routed slots
    and the shared expert; the measured experts are whatever the router
    picked. On N GPUs the layer is expert-parallel through `group` (its
    current exchange mode; the all-to-all dispatch sends each GPU only the
    rows routed to it); rank 0's outputs are checked bit for bit against the
    one-GPU layer on the same tokens."""
    spec = S.CONFIGS[3]
    if args.experts:
        import dataclasses
        spec = dataclasses.replace(spec, experts=args.experts)
    T = args.prefill_tokens
    ep = world > 1
    # the Zipf router favours low expert ids: strided placement spreads the
    # hot experts over the GPUs (contiguous ranges would put them all on one)
    if ep:
        # the all-to-all dispatch: each GPU receives only the rows routed to
        # its experts (the all-gather modes would hand every GPU all N * T)
        group.set_placement("strided")
        group.set_mode("alltoall")
        try:
            return _prefill(args, S, torch, ctx, local, dev, group, world, rank, dist, spec, T)
        finally:
            group.set_placement("contiguous")
            group.set_mode(args.ep_mode)
    return _prefill(args, S, torch, ctx, local, dev, group, world, rank, dist, spec, T)


def _prefill(args, S, torch, ctx, local, dev, group, world, rank, dist, spec, T):
    ep = world > 1
    lay = S.synth_layer(spec, layer=0, device=local, shard=(rank, world) if ep else None,
                        strided=ep)
    x = S.synth_x(spec, T * world, layer=0, batch=0, device=local)[rank * T:(rank + 1) * T]
    x = x.contiguous()
    out = torch.empty((T, spec.hidden), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((T, spec.top_k), dtype=torch.int32, device=dev)

    def fwd(want_ids=False):
        if ep:
            group.forward(lay, x, out=out, ids=ids if want_ids else None)
        elif want_ids:
            _, sel = lay.forward(x, out=out)
            ids.copy_(sel.ids)
        else:
            lay.forward(x, out=out, selection=False)

    def barrier():
        if ep:
            dist.barrier()

    def max_over_ranks(v):
        if ep:
            t = torch.tensor([v], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = float(t.item())
        return v

    for _ in range(3):
        fwd()
    torch.cuda.synchronize()
    barrier()
    steps = 5
    ctx.profile(True)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fwd()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    prof = ctx.profile_read()
    ctx.profile(False)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    fwd(True)
    torch.cuda.synchronize()
    allids = ids
    if ep:
        parts = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(parts, ids)
        allids = torch.cat(parts)
    hist = torch.bincount(allids.view(-1).long(), minlength=spec.experts).cpu().tolist()
    distinct = sum(1 for c in hist if c)
    slots = world * T * (spec.top_k + (1 if spec.shared_inter else 0))
    gu_flops = slots * 2 * (2 * spec.hidden * spec.inter)
    dn_flops = slots * 2 * spec.hidden * spec.inter
    gu_ms = max_over_ranks(prof["gate_up"][0] / steps)   # per step (routed + shared launches)
    dn_ms = max_over_ranks(prof["down_combine"][0] / steps)
    peak, kind = tensor_peak()
    gu_tf = gu_flops / world / (gu_ms / 1e3) / 1e12        # per GPU
    one = None
    if ep:
        # rank 0's tokens through the one-GPU layer (routing is per token)
        same = None
        if rank == 0:
            full = S.synth_layer(spec, layer=0, device=local)
            ref, _ = full.forward(x)
            torch.cuda.synchronize()
            same = bool(torch.equal(ref, out))
            del full, ref
            torch.cuda.empty_cache()
        barrier()
        one = {"tokens": T, "bit_identical": same}
    per_rank = None
    if ep:
        per_rank = [sum(hist[r::world]) for r in range(world)]
    return {
        "workload": f"config3 prefill T={T} per GPU: config-1 layer, router biased to Zipf(1.1)"
                    + (f", ep{world}, strided expert placement (expert e on GPU e % {world})"
                       if ep else ""),
        "tokens_per_s": world * T / (ms / 1e3),
        "ms_per_step": ms,
        "distinct_experts": distinct,
        "top_expert_share": max(hist) / max(sum(hist), 1),
        "routed_pairs_per_gpu": per_rank,
        "gate_up_ms": gu_ms,
        "down_combine_ms": dn_ms,
        "roofline": {"bound": "tensor", "kernel": "gemm gate/up (+SwiGLU), tcgen05",
                     "achieved": gu_tf, "peak": peak, "peak_kind": kind, "unit": "TFLOP/s",
                     "frac": gu_tf / peak, "algorithmic_flops_per_step": gu_flops / world,
                     "note": "per GPU: the group's gate/up FLOPs / N over the slowest GPU's "
                             "gate/up time" if ep else "one GPU"},
        "layer_tflops_per_gpu": (gu_flops + dn_flops) / world / (ms / 1e3) / 1e12,
        "down_tflops": dn_flops / world / (dn_ms / 1e3) / 1e12,
        "vs_one_gpu": one,
    }


def k3_run(args, M, torch, dev, hbm):
    """K3's latent MoE layer (K3MoE.forward, MoE.swift:219-272) at the flagship
    geometry (hidden 7168, latent 3584, intermediate 3072, top-16, MXFP4 routed
    experts, bf16 dense latent projections and a 6144-wide bf16 shared expert),
    fp32 activations, seeded random weights generated on the GPU. One step =
    one layer forward over T tokens; L2 is flushed (a 256 MB write) between
    steps, outside the timed events."""
    E, H, Lt, I, S, k = args.k3_experts, 7168, 3584, 3072, 6144, 16
    g = torch.Generator(device=dev)
    g.manual_seed(20260801)

    def mx(e, o, i):
        shape = (e, o) if e else (o,)
        p = torch.randint(-2**31, 2**31 - 1, shape + (i // 8,), dtype=torch.int32, device=dev,
                          generator=g)
        sc = torch.randint(118, 122, shape + (i // 32,), dtype=torch.uint8, device=dev,
                           generator=g)
        return M.MXFP4Weights(p, sc)

    def dense(o, i):
        return (torch.randn(o, i, device=dev, generator=g) / i ** 0.5).to(torch.bfloat16)

    blk = M.K3MoE(dense(E, H), torch.zeros(E, device=dev), M.K3Projection(dense(Lt, H)),
                  M.K3Projection(dense(H, Lt)), torch.ones(Lt, device=dev), mx(E, I, Lt),
                  mx(E, I, Lt), mx(E, Lt, I),
                  (M.K3Projection(dense(S, H)), M.K3Projection(dense(S, H)),
                   M.K3Projection(dense(H, S))), k)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    dense_bytes = (E * H + 2 * Lt * H + 3 * S * H) * 2
    out = {}
    for T in [int(t) for t in args.k3_tokens.split(",") if t]:
        x = torch.randn(T, H, device=dev, generator=g)
        for _ in range(max(3, args.warmup)):
            blk.forward(x)
        times, us = [], []
        for _ in range(args.steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            _, sel = blk.forward(x)
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
            us.append(len(torch.unique(sel.ids)))
        ms = sum(times) / len(times)
        U = sum(us) / len(us)
        byt = U * 3 * I * Lt * (0.5 + 1 / 32) + dense_bytes
        out[str(T)] = {"ms_per_layer": ms, "tokens_per_s": T / (ms / 1e3),
                       "distinct_experts_avg": U, "layer_bytes": byt,
                       "layer_gbs": byt / (ms / 1e3) / 1e9,
                       "layer_frac_of_hbm": byt / (ms / 1e3) / 1e9 / hbm}
    return {"workload": f"K3 latent MoE layer: {E} MXFP4 experts, hidden {H}, latent {Lt}, "
                        f"inter {I}, top-{k}, bf16 dense projections, fp32 activations",
            "l2": "flushed between steps (256 MB write, outside the timed events)",
            "by_tokens": out}


def cache_run(args, M, S, torch, dev, layers_n=None, budget_gb=None, check_identity=False):
    """Config 4: one-token decode through `layers_n` config-1 layers whose
    routed experts live in pinned host memory and reach the GPU through the
    HBM expert cache (`mr_moe_layer_forward_cached`) under `budget_gb`.
    Each layer has its own seeded router (and so its own routing); to keep
    host memory at one layer's 6.4 GB, every layer registers the same seeded
    expert arrays under its own (layer, expert) keys, so the cache sees
    layers x 256 distinct experts and copies each miss from host memory as it
    would distinct weights. The shared expert stays resident. A step = one
    token position through all layers, each layer routing a seeded token of
    its own: with the BASELINE weight distributions (codes uniform, bias
    -8 * scale, so every weight has mean -scale/2) a layer's output is
    dominated by one common-mode direction, and chained layers would route
    every token to the same experts. Independent tokens make the routing as
    diverse as random choice, the hard case for the cache.
    With `check_identity`, the same tokens also run through a second cache
    whose budget holds every expert (all resident after the first pass), and
    the outputs of the timed steps must be byte-identical."""
    spec = S.CONFIGS[1]
    NL = layers_n if layers_n is not None else args.cache_layers
    gb = budget_gb if budget_gb is not None else args.cache_budget_gb
    if not gb:
        gb = 40.0 * NL / 58.0  # the BASELINE resident fraction (40 GB of 58 layers)
    base = S.synth_layer(spec, layer=0, device=dev.index)
    E, H = spec.experts, spec.hidden
    slot = M.ExpertCache.slot_bytes_for(base.gate, base.up, base.down)
    t0 = time.perf_counter()
    host = [tuple(tuple(t[e].contiguous().cpu().pin_memory() for t in (w.packed, w.scales,
                                                                        w.biases))
                  for w in (base.gate, base.up, base.down)) for e in range(E)]
    layers = []
    for l in range(NL):
        rw = torch.empty((E, H), dtype=torch.bfloat16, device=dev)
        S.synth_normal_bf16(S.derive(spec.seed, S.label(l, S.KIND_ROUTER, 0, 0)), E * H,
                            1.0 / 32.0, False, rw)
        layers.append(M.CachedLayer(rw, base.router, H, spec.inter, spec.bits, spec.group,
                                    shared=base.shared))

    def make_cache(budget_bytes):
        c = M.ExpertCache(dev.index, int(budget_bytes), slot)
        for l in range(NL):
            for e in range(E):
                c.register(l, e, host[e])
        return c

    cache = make_cache(gb * 1e9)
    setup_s = time.perf_counter() - t0
    steps = max(3, min(args.steps, 10))
    W = max(3, args.warmup)
    # a seeded token per (step, layer)
    xs = [[S.synth_x(spec, 1, layer=l, batch=i, device=dev.index) for l in range(NL)]
          for i in range(W + steps)]
    outs = [[torch.empty((1, H), dtype=torch.bfloat16, device=dev) for _ in range(NL)]
            for _ in range(W + steps)]

    def token(c, i):
        for l, lay in enumerate(layers):
            c.forward(l, lay, xs[i][l], out=outs[i][l])

    for i in range(W):  # first fills of the cache
        token(cache, i)
    torch.cuda.synchronize()
    s0 = cache.stats()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(W, W + steps):
        token(cache, i)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    s1 = cache.stats()
    d = {k: s1[k] - s0[k] for k in ("hits", "misses", "bytes_copied") if k in s1}
    uses = d.get("hits", 0) + d.get("misses", 0)
    slots = int(gb * 1e9) // slot
    cache.close()
    identity = None
    if check_identity:
        got = [torch.cat(outs[i]).clone() for i in range(W, W + steps)]
        big = make_cache(NL * E * slot + slot)  # every expert fits
        for i in range(W + steps):
            token(big, i)
        torch.cuda.synchronize()
        same = all(torch.equal(got[j], torch.cat(outs[W + j])) for j in range(steps))
        big.close()
        identity = {"vs_all_resident_budget_gb": (NL * E * slot + slot) / 1e9,
                    "byte_identical": same}
    return {"workload": f"config4: {NL} config-1 layers, 1-token decode, {E} routed experts "
                        f"per layer in pinned host memory, HBM cache budget "
                        f"{gb:g} GB ({slots} slots of {slot} B)",
            "tokens_per_s": 1e3 / ms, "ms_per_token": ms, "steps": steps,
            "hit_rate": d.get("hits", 0) / max(uses, 1),
            "h2d_gbs": d.get("bytes_copied", 0) / steps / (ms / 1e3) / 1e9,
            "setup_s": setup_s, "identity": identity,
            "note": "every layer registers the same seeded host arrays under its own keys"}


def config4_ep_run(args, S, M, torch, world, rank, local, dev, group, max_over_ranks, barrier):
    """Config 4 on N GPUs with every expert resident: `--config4-ep-layers`
    seeded config-1 layers, each GPU holding E/N routed experts of every
    layer; a one-token decode whose token lives on GPU 0 (the others pass no
    tokens, all-to-all mode with capacity 1). As in the one-GPU line each
    layer routes a seeded token of its own. GPU 0's outputs of the first two
    layers are checked bit for bit against the one-GPU layer."""
    group.set_mode("alltoall")
    group.set_placement("contiguous")
    group.set_capacity(1)
    try:
        return _config4_ep(args, S, torch, world, rank, local, dev, group, max_over_ranks,
                           barrier)
    finally:
        group.set_capacity(0)
        group.set_mode(args.ep_mode)
        torch.cuda.empty_cache()


def _config4_ep(args, S, torch, world, rank, local, dev, group, max_over_ranks, barrier):
    spec = S.CONFIGS[1]
    NL = args.config4_ep_layers
    layers = [S.synth_layer(spec, layer=l, device=local, shard=(rank, world)) for l in range(NL)]
    steps = max(3, min(args.steps, 10))
    W = max(3, args.warmup)
    H = spec.hidden
    empty = torch.empty((0, H), dtype=torch.bfloat16, device=dev)
    xs = [[S.synth_x(spec, 1, layer=l, batch=i, device=local) if rank == 0 else empty
           for l in range(NL)] for i in range(W + steps)]
    outs = [torch.empty((1 if rank == 0 else 0, H), dtype=torch.bfloat16, device=dev)
            for _ in range(NL)]

    def token(i):
        for l, lay in enumerate(layers):
            group.forward(lay, xs[i][l], out=outs[l])

    for i in range(W):
        token(i)
    torch.cuda.synchronize()
    barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(W, W + steps):
        token(i)
    b.record()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(a.elapsed_time(b) / steps)
    same = None
    if rank == 0:
        same = True
        for l in range(min(2, NL)):
            full = S.synth_layer(spec, layer=l, device=local)
            ref, _ = full(xs[W + steps - 1][l])
            torch.cuda.synchronize()
            same = same and bool(torch.equal(ref, outs[l]))
            del full
        torch.cuda.empty_cache()
    barrier()
    resident = sum(w.nbytes for lay in layers for w in (lay.gate, lay.up, lay.down))
    del layers
    return {"workload": f"config4: {NL} config-1 layers, 1-token decode, every routed expert "
                        f"resident ({spec.experts // world} per GPU per layer), the token on "
                        f"GPU 0, all-to-all dispatch",
            "tokens_per_s": 1e3 / ms, "ms_per_token": ms, "steps": steps,
            "routed_bytes_resident_per_gpu": resident,
            "identity": {"vs_one_gpu_layers": min(2, NL), "bit_identical": same}}


def e2e_run(args, spec, T, K, W, xs, schedule, barrier, world, dev, local, group=None):
    """Same metric with host buffers: pinned host x in, host out, both copies
    inside the timed region — through the host-buffer C-ABI call on one GPU,
    through copies + the expert-parallel call on N."""
    if args.no_e2e:
        return None
    import torch
    import torch.distributed as dist
    xh = [x.cpu().pin_memory() for x in xs[T]]
    oh = torch.empty((T, spec.hidden), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty((T, spec.hidden), dtype=torch.bfloat16, device=dev)
    od = torch.empty_like(xd)

    def host_step(lay, xhost):
        if group is None:
            lay.forward_host(xhost, oh, device=local)
        else:
            xd.copy_(xhost, non_blocking=True)
            group.forward(lay, xd, out=od)
            oh.copy_(od, non_blocking=True)

    for i in range(W):
        lay, b = schedule(i)
        host_step(lay, xh[b])
    torch.cuda.synchronize()
    barrier()
    st = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(K):
        lay, b = schedule(i)
        host_step(lay, xh[b])
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    return {
        "value": world * T * K / (e2e_ms / 1e3),
        "unit": "tokens/s",
        "h2d_bytes_per_step": T * spec.hidden * 2,
        "d2h_bytes_per_step": T * spec.hidden * 2,
    }


def read_traffic(algorithmic_bytes):
    """DRAM bytes per gate/up launch, scaled from the committed ncu summary.

    The summary records one captured launch (a small case that fits the capture
    rules): its dram read+write bytes and its algorithmic bytes. Traffic grows
    with the weight bytes a launch streams, so the bench launch's traffic is the
    captured ratio times its own algorithmic bytes."""
    path = os.path.join(ROOT, "profiles", "gemv_v2_gate_up_config1.md")
    vals = {}
    try:
        for line in open(path):
            for key in ("traffic_bytes_per_launch", "algorithmic_bytes_per_launch"):
                if line.startswith(key + ":"):
                    vals[key] = float(line.split(":", 1)[1].split()[0])
    except (OSError, ValueError):
        return None
    if len(vals) != 2 or vals["algorithmic_bytes_per_launch"] <= 0:
        return None
    return vals["traffic_bytes_per_launch"] / vals["algorithmic_bytes_per_launch"] * algorithmic_bytes


# ------------------------------------------------------------- CPU baseline

def cpu_baseline(T: int, steps: int = 1):
    """The CPU oracle (C, OpenMP, all host threads) on config 1 with T tokens."""
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    O.set_num_threads(os.cpu_count() or 1)
    cfg = O.CONFIGS[1]
    x = O.gen_x(cfg, T, layer=0, batch=0)
    L = O.gen_layer(cfg, layer=0, experts=O.selected_experts(cfg, x))
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        O.moe_layer_forward(L, x)
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    return {"value": T / dt, "unit": "tokens/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"config1 layer 0, one {T}-token batch, {steps} forward(s), "
                      f"{dt:.2f} s each (weights generation excluded)"}


def run_reference(args, world, rank, local):
    """The reference arm: the CPU restatement of the path (the reference's
    own implementation is Swift/MLX on Apple GPUs and cannot run here)."""
    if rank != 0:
        return
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    # torchrun sets OMP_NUM_THREADS=1 for every rank; the reference arm runs
    # on rank 0 alone and takes every host thread
    O.set_num_threads(os.cpu_count() or 1)
    cfg = O.CONFIGS[1]
    T = args.tokens
    x = O.gen_x(cfg, T, layer=0, batch=0)
    L = O.gen_layer(cfg, layer=0, experts=O.selected_experts(cfg, x))
    t0 = time.perf_counter()
    O.moe_layer_forward(L, x)
    est = time.perf_counter() - t0
    K = max(2, min(args.steps, int(150 / max(est, 1e-3))))
    W = max(3, min(args.warmup, int(60 / max(est, 1e-3))))  # >= 3 untimed steps
    for _ in range(W):
        O.moe_layer_forward(L, x)
    t0 = time.perf_counter()
    for _ in range(K):
        O.moe_layer_forward(L, x)
    dt = time.perf_counter() - t0
    value = T * K / dt
    cores = O.num_threads()
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": dt / K * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations, 4-bit affine weights, exact (fp64) accumulation",
        "data": "synthetic (SplitMix64-seeded, BASELINE config 1 distributions)",
        "config": {"workload": f"config1 decode T={T}: H7168, 256+1 experts, top-8, I2048, "
                               f"4-bit g64", "tokens": T,
                   "note": "the reference's MLX/Metal path is unavailable on this box (no "
                           "Apple GPU, Swift or mlx); the CPU restatement of its arithmetic "
                           "(oracle/, C + OpenMP) stands in"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"config1 layer 0, one {T}-token batch per step"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank, local)
    elif args.cache_only:
        import torch
        import minirun_moe as M
        from minirun_moe import synth as S
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        print(json.dumps({"config4_cached_decode": cache_run(args, M, S, torch, dev)}),
              flush=True)
    elif args.k3_only:
        import torch
        import minirun_moe as M
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        hbm, _ = peaks()
        print(json.dumps({"k3_latent_moe": k3_run(args, M, torch, dev, hbm)}), flush=True)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
