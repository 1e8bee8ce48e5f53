#!/usr/bin/env python3
"""Benchmark of the Hyperion hot path on B200 (one JSON line on rank 0).

Default workload (the metric's "12B-shaped decode tok/s at 1/2/4/8
GPUs"): the 48-layer Gemma-12B-shaped Q4/g64 decoder (seeded synthetic weights) prefills
a 4096-token context and then decodes greedily, one token per step, through the
reference-facing ABI call hyp_decode_block. With N GPUs the model is tensor-parallel
over the N ranks (column/row-parallel projections, KV heads sharded, vocab-parallel
lm_head, all-reduces over NVLink), so `value` is whole-job tokens/s at a fixed model
(strong scaling). The line also carries:
  * roofline: the decode projections' kernel (qmv_packed_kernel) over this rank's
    shapes, timed live with CUDA events on graphs of back-to-back launches over distinct
    weight copies (inputs larger than L2), mix-weighted by one token's launches;
  * qmv_sweep (N = 1): the config-1 qmv shapes, the metric's first half;
  * parity (N > 1): 16 greedy steps of the tensor-parallel run teacher-forced against
    the same model at TP = 1 on rank 0;
  * cpu_baseline (N = 1): a full 48-layer decode token on the host cores (the oracle's
    multithreaded C kernels; the reference's own CPU path is MLX, unavailable here).

Other workloads (profiling and config 2/4 measurements): `--workload qmv` (the config-1
sweep in 12B decode-token proportions, GB/s), `qmv-shape`, `attn-decode`, `qmm`,
`sdpa-prefill`, `spec-verify`, `tp-decode` (27B-shaped, config 4).

`--impl reference` times the CPU restatement of the default workload (full decode
tokens on all host cores) on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

PROJ = [("q", 3840, 4096), ("k", 3840, 2048), ("v", 3840, 2048), ("o", 4096, 3840),
        ("gate", 3840, 15360), ("up", 3840, 15360), ("down", 15360, 3840)]
LM_HEAD = ("lm_head", 3840, 262144)
N_LAYERS = 48
METRIC = "Q4/g64 qmv HBM GB/s (% of peak); 12B-shaped decode tok/s at 1/2/4/8 GPUs"


def qmv_bytes(K: int, N: int) -> int:
    """Algorithmic bytes of one batch-1 qmv: nibbles + bf16 scale/bias + x + y."""
    return K * N // 2 + 4 * N * K // 64 + 2 * K + 2 * N


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ CPU baseline (oracle)
def cpu_qmv_baseline(budget_s: float = 10.0):
    """The oracle's multithreaded qmv over the six cfg-1 shapes, looped for ~budget_s."""
    import numpy as np
    from oracle import gemma_oracle as go
    from hyperion_b200.synth import f32_to_bf16_bits
    rng = np.random.default_rng(0)
    shapes = [(3840, 4096), (3840, 2048), (4096, 3840), (3840, 15360), (15360, 3840), (3840, 262144)]
    data = []
    for K, N in shapes:
        w = rng.integers(0, 2 ** 32, size=(N, K // 8), dtype=np.uint32)
        s = f32_to_bf16_bits(np.abs(rng.standard_normal((N, K // 64), dtype=np.float32)) * 0.02)
        b = f32_to_bf16_bits(-8 * (s.astype(np.uint32) << 16).view(np.float32))
        x = f32_to_bf16_bits(rng.standard_normal(K, dtype=np.float32))
        data.append((K, N, x, w, s, b))
    threads = go.host_threads()
    for K, N, x, w, s, b in data:  # warm-up pass
        go.qmv_fast(x, w, s, b, threads)
    total_bytes, t0, passes = 0, time.perf_counter(), 0
    while True:
        for K, N, x, w, s, b in data:
            go.qmv_fast(x, w, s, b, threads)
            total_bytes += qmv_bytes(K, N)
        passes += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    el = time.perf_counter() - t0
    return {"value": round(total_bytes / el / 1e9, 2), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{passes} passes over the six cfg-1 qmv shapes (655 MB each), {el:.1f} s, "
                      f"oracle/hyp_oracle.c orc_qmv_fast, OpenMP {threads} threads"}


class CpuDecode:
    """Full 12B-shaped decode tokens on the host cores: the reference's CPU path restated
    with the oracle's multithreaded C kernels (orc_qmv_fast: fp32 group dots, the way a
    tuned CPU quantized matmul accumulates; orc_sdpa: fp32-or-better attention).

    Every step runs all 48 layers: input norm, the fused q/k/v projection, QK-norm, RoPE,
    cache append, attention over 1024 ring keys (sliding) or every cached key (global),
    o_proj, residual and norms, gate/up, GeGLU, down_proj, layer scalar, then the final
    norm, the 262144-row lm_head, the soft-cap and the greedy scan. Weights are the
    seeded synthetic model; the caches hold random keys for a `ctx`-token context. The
    ring is read in slot order rather than position order (same cost, no gather), so
    this is a timing port, not a parity path (parity lives in tests/)."""

    def __init__(self, ctx: int, threads: int, extra_steps: int = 256, seed: int = 1):
        import numpy as np
        from oracle import gemma_oracle as go
        from hyperion_b200.synth import config3
        self.go, self.np = go, np
        self.geo = geo = config3()
        self.threads = threads
        ztab = go.normal_table()
        H, I, nh, hd = geo.hidden_size, geo.intermediate_size, geo.num_attention_heads, geo.head_dim_local
        rng = np.random.default_rng(seed)
        tag = [seed * 1000003]

        def nxt():
            tag[0] += 1
            return tag[0]

        self.lm = go.synth_q4(nxt(), geo.vocab_size, H, ztab=ztab, nthreads=threads)
        self.final_norm = go.synth_norm(nxt(), H, ztab)
        self.layers = []
        for i, kind in enumerate(geo.layer_types):
            nkv = geo.n_kv(i)
            rows = nh * hd + (1 if kind == 1 else 2) * nkv * hd
            cap = geo.sliding_window + 8 if kind == 0 else ctx + extra_steps
            lay = {"kind": kind, "qkv": go.synth_q4(nxt(), rows, H, ztab=ztab, nthreads=threads),
                   "o": go.synth_q4(nxt(), H, nh * hd, ztab=ztab, nthreads=threads),
                   "gate": go.synth_q4(nxt(), I, H, ztab=ztab, nthreads=threads),
                   "up": go.synth_q4(nxt(), I, H, ztab=ztab, nthreads=threads),
                   "down": go.synth_q4(nxt(), H, I, ztab=ztab, nthreads=threads),
                   "norms": [go.synth_norm(nxt(), n, ztab) for n in (hd, hd, H, H, H, H, 1)],
                   "k": rng.integers(0x3800, 0x3F00, size=(cap, nkv, hd), dtype=np.uint16),
                   "v": rng.integers(0x3800, 0x3F00, size=(cap, nkv, hd), dtype=np.uint16)}
            self.layers.append(lay)
        self.inv_l = go.rope_inv_freq(hd, geo.rope_theta_local, False, 0.0)
        self.inv_g = go.rope_inv_freq(geo.head_dim_global, geo.rope_theta_global, True,
                                      geo.partial_rotary_factor_global)
        self.pos = ctx
        self.token = 7

    def step(self) -> int:
        go, np, geo, nt = self.go, self.np, self.geo, self.threads
        H, nh, eps = geo.hidden_size, geo.num_attention_heads, geo.rms_norm_eps
        w, s, b = self.lm
        codes = np.zeros(H, dtype=np.float32)
        for i in range(8):
            codes[i::8] = ((w[self.token] >> np.uint32(4 * i)) & np.uint32(15)).astype(np.float32)
        g = codes.reshape(-1, 64) * go.fl(s[self.token])[:, None] + go.fl(b[self.token])[:, None]
        h = go.bf(go.fl(go.bf(g.reshape(-1))) * 62.0)
        pos = self.pos
        for lay in self.layers:
            qn, kn, in_ln, post_attn, pre_ff, post_ff, scal = lay["norms"]
            kind = lay["kind"]
            k_c, v_c = lay["k"], lay["v"]
            nkv, hd = k_c.shape[1], k_c.shape[2]
            xn = go.rms_norm(h.reshape(1, H), in_ln, eps)
            qkv = go.qmv_fast(xn, *lay["qkv"], nt)
            q = go.rope(go.rms_norm(qkv[:nh * hd].reshape(1, nh, hd), qn, eps), pos, self.inv_l if kind == 0 else self.inv_g)
            kr = qkv[nh * hd:(nh + nkv) * hd].reshape(1, nkv, hd)
            k = go.rope(go.rms_norm(kr, kn, eps), pos, self.inv_l if kind == 0 else self.inv_g)
            v = go.rms_norm(kr if kind == 1 else qkv[(nh + nkv) * hd:].reshape(1, nkv, hd), None, eps)
            slot = pos % k_c.shape[0]
            k_c[slot], v_c[slot] = k[0], v[0]
            n = min(geo.sliding_window, pos + 1) if kind == 0 else pos + 1
            att = go.sdpa(q, k_c[:n], v_c[:n], pos, pos - n + 1, 0, nthreads=nt)
            o = go.qmv_fast(att.reshape(-1), *lay["o"], nt)
            h1 = go.bf(go.fl(h) + go.fl(go.rms_norm(o.reshape(1, H), post_attn, eps)).reshape(-1))
            xin = go.rms_norm(h1.reshape(1, H), pre_ff, eps)
            act = go.bf(go.fl(go.gelu_tanh(go.qmv_fast(xin, *lay["gate"], nt))) * go.fl(go.qmv_fast(xin, *lay["up"], nt)))
            dn = go.qmv_fast(act, *lay["down"], nt)
            h2 = go.bf(go.fl(h1) + go.fl(go.rms_norm(dn.reshape(1, H), post_ff, eps)).reshape(-1))
            h = go.bf(go.fl(h2) * go.fl(scal)[0])
        logits = go.softcap(go.qmv_fast(go.rms_norm(h.reshape(1, H), self.final_norm, eps), *self.lm, nt),
                            geo.final_logit_softcapping)
        self.token = go.greedy(logits)[0]
        self.pos += 1
        return self.token


def cpu_decode_baseline(ctx: int, budget_s: float = 10.0):
    """CPU tokens/s of full 12B-shaped decode tokens (CpuDecode) for about budget_s."""
    from oracle import gemma_oracle as go
    threads = go.host_threads()
    cpu = CpuDecode(ctx, threads)
    cpu.step()  # warm-up (first touch of the caches, thread pool start)
    t0, n = time.perf_counter(), 0
    while True:
        cpu.step()
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    el = time.perf_counter() - t0
    return {"value": round(n / el, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} full cfg3 decode tokens (48 layers + lm_head) at ctx {ctx} in {el:.1f} s, oracle C "
                      f"kernels (orc_qmv_fast, orc_sdpa) on {threads} host threads"}


def run_reference(args):
    """The reference arm: the default workload's CPU restatement (full 12B-shaped decode
    tokens, all host cores) on rank 0; other ranks exit at once."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import gemma_oracle as go
    threads = go.host_threads()
    cpu = CpuDecode(args.ctx, threads, extra_steps=args.warmup + args.steps + 8)
    for _ in range(args.warmup):
        cpu.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.step()
    el = time.perf_counter() - t0
    v = args.steps / el
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u4/bf16->f32",
            "data": "synthetic",
            "config": {"workload": f"cfg3 12B-shaped decode, ctx {args.ctx}, batch 1", "l2": "inputs larger than L2"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} full decode tokens (48 layers + lm_head) at ctx {args.ctx}, "
                                       f"oracle C kernels on {threads} host threads (the reference's MLX CPU path "
                                       f"is not installable here)"},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ qmv sweep (ours)
def make_q4(N, K, gen, device):
    import torch
    w = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // 8), dtype=torch.int32, device=device, generator=gen)
    s = (torch.randn((N, K // 64), device=device, generator=gen) * 0.02).abs().to(torch.bfloat16)
    b = (-8.0 * s.float()).to(torch.bfloat16)
    return w, s, b


def run_qmv(args, rank, world, local):
    """`--workload qmv`: the config-1 sweep as one graph of 337 launches per step (every
    projection of a 12B decode token with its own weights), replicated per rank."""
    import torch
    import ctypes
    import hyperion_b200 as hb
    from hyperion_b200 import ops
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    # weights: 48 layers x 7 projections + lm_head, all distinct
    layers = []
    for _ in range(N_LAYERS):
        lay = []
        for name, K, N in PROJ:
            w, s, b = make_q4(N, K, gen, dev)
            x = torch.randn(K, device=dev, generator=gen).to(torch.bfloat16)
            y = torch.empty(N, dtype=torch.bfloat16, device=dev)
            lay.append((name, K, N, w, s, b, x, y))
        layers.append(lay)
    K, N = LM_HEAD[1], LM_HEAD[2]
    lw, ls, lb = make_q4(N, K, gen, dev)
    lx = torch.randn(K, device=dev, generator=gen).to(torch.bfloat16)
    ly = torch.empty(N, dtype=torch.bfloat16, device=dev)
    items = [it for lay in layers for it in lay] + [("lm_head", K, N, lw, ls, lb, lx, ly)]
    step_bytes = sum(qmv_bytes(it[1], it[2]) for it in items)
    launches = len(items)
    # the decode engine's resident layout: every matrix repacked once (not timed)
    packs = [ops.qmv_pack(it[3], it[4], it[5]) for it in items]
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device=dev)

    def launch_all():
        for it, pk in zip(items, packs):
            name, K_, N_, w, s, b, x, y = it
            ops.qmv_packed(x, pk, K_, N_, out=y)

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        launch_all()  # sets kernel attributes outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch_all()
    # ---- device-resident timing (graph replays go to the current stream)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        torch.cuda.synchronize()
        barrier(world)
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = max_over_ranks(ms, world)
    value = step_bytes * world / (ms_max * 1e-3) / 1e9

    # ---- per-shape kernel timing (each shape over its distinct copies, graph of back-to-back launches)
    per_shape = []
    shape_time = {}
    for (name, K_, N_), layout in [(sh, lay) for sh in PROJ + [LM_HEAD] for lay in ("packed", "mlx")]:
        sel = [(it, pk) for it, pk in zip(items, packs) if it[0] == name]
        reps = max(1, 48 // len(sel))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                for it, pk in sel:
                    if layout == "packed":
                        ops.qmv_packed(it[6], pk, K_, N_, out=it[7])
                    else:
                        ops.quantized_matmul(it[6].view(1, K_), it[3], it[4], it[5], out=it[7].view(1, N_))
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            R = 5
            for _ in range(R):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        per_launch_us = e0.elapsed_time(e1) * 1e3 / (R * reps * len(sel))
        gbs = qmv_bytes(K_, N_) / (per_launch_us * 1e-6) / 1e9
        if layout == "packed":
            shape_time[name] = per_launch_us
        per_shape.append({"shape": f"{name} K={K_} N={N_}", "layout": layout, "us": round(per_launch_us, 2),
                          "GB/s": round(gbs, 1), "frac": round(gbs / peaks()[0], 3)})
        del g
    # mix-weighted kernel achieved bandwidth (kernel time only, no inter-launch gaps)
    kern_us = sum(shape_time[it[0]] for it in items)
    achieved = step_bytes / (kern_us * 1e-6) / 1e9

    # ---- e2e: the C-ABI call per projection with host activations/results
    hx = torch.empty(sum(it[1] for it in items), dtype=torch.bfloat16).pin_memory()
    hy = torch.empty(sum(it[2] for it in items), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(hx, device=dev)
    dy = torch.empty_like(hy, device=dev)
    hx.copy_(torch.randn(hx.numel()).to(torch.bfloat16))
    offs_x, offs_y, ox, oy = [], [], 0, 0
    for it in items:
        offs_x.append(ox)
        offs_y.append(oy)
        ox += it[1]
        oy += it[2]
    L = hb.lib()
    s_ptr = ctypes.c_void_p(stream.cuda_stream)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        for i, it in enumerate(items):
            _, K_, N_, w, s, b, _, _ = it
            L.hyb_qmv_packed(ctypes.c_void_p(dx.data_ptr() + 2 * offs_x[i]), ctypes.c_void_p(packs[i].data_ptr()),
                             ctypes.c_void_p(dy.data_ptr() + 2 * offs_y[i]), K_, N_, 0, 0, None, None, None, None,
                             None, 1e-6, s_ptr)
        hy.copy_(dy, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    e2e_val = step_bytes * world / (e2e_ms * 1e-3) / 1e9

    if rank != 0:
        return
    hbm, _, src = peaks()
    traffic = None
    tp = os.path.join(REPO, "profiles", "qmv_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get("dram_bytes_per_launch_mix")
    line = {
        "metric": "cfg1 Q4/g64 qmv HBM GB/s (12B decode-token mix)", "value": round(value, 1), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4/bf16->f32", "data": "synthetic",
        "config": {"workload": "cfg1 qmv sweep in 12B decode-token proportions: 48 x {q,k,v,o,gate,up,down} "
                               "+ lm_head, distinct weights (6.62 GB/step)",
                   "l2": "inputs larger than L2 (no reuse across steps)",
                   "step_bytes": step_bytes, "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": src,
                     "kernel": "qmv_packed_kernel (mix-weighted over the step's 337 launches)"},
        "per_shape": per_shape,
        "gpu_launches": launches * args.steps,
        "e2e": {"value": round(e2e_val, 1), "unit": "GB/s",
                "h2d_bytes_per_step": int(hx.numel() * 2), "d2h_bytes_per_step": int(hy.numel() * 2),
                "path": "hyb_qmv_packed per projection via ctypes, host x/y copied each step"},
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_qmv_baseline(args.cpu_seconds)
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ prefill qmm (config 2)
def run_qmm(args, rank, world, local):
    """Config 2: the 12B-shaped projections of one decoder layer (q/k/v fused 3840x8192,
    o 4096x3840, gate/up fused 3840x30720, down 15360x3840) at M tokens, through
    hyb_quantized_matmul (tcgen05 tensor cores). value = useful TFLOP/s (2 M K N)."""
    import torch
    from hyperion_b200 import ops
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    shapes = [("qkv", 3840, 8192), ("o", 4096, 3840), ("gate_up", 3840, 30720), ("down", 15360, 3840)]
    Ms = [int(m) for m in args.qmm_m.split(",")]
    weights = {nm: make_q4(N, K, gen, dev) for nm, K, N in shapes}
    stream = torch.cuda.Stream(device=dev)
    rows, flop_tot, us_tot = [], 0.0, 0.0
    for M in Ms:
        xs = {K: torch.randn((M, K), device=dev, generator=gen).to(torch.bfloat16) for _, K, _ in shapes}
        ys = {nm: torch.empty((M, N), dtype=torch.bfloat16, device=dev) for nm, _, N in shapes}

        def layer():
            for nm, K, N in shapes:
                w, s, b = weights[nm]
                ops.quantized_matmul(xs[K], w, s, b, out=ys[nm], stream=stream)

        with torch.cuda.stream(stream):
            layer()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                layer()
            for _ in range(args.warmup):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as clk:
                e0.record(stream)
                for _ in range(args.steps):
                    g.replay()
                e1.record(stream)
                torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        flops = sum(2.0 * M * K * N for _, K, N in shapes)
        rows.append({"M": M, "us_per_layer": round(us, 1), "TFLOP/s": round(flops / (us * 1e-6) / 1e12, 1)})
        flop_tot += flops
        us_tot += us
        del g
    _, tf_peak, src = peaks()
    value = flop_tot / (us_tot * 1e-6) / 1e12
    print(json.dumps({"metric": "prefill Q4/g64 qmm TFLOP/s (cfg2 12B layer projections)", "value": round(value, 1),
                      "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(us_tot / 1e3, 4), "higher_is_better": True, "dtype": "u4->f16, f32 acc",
                      "data": "synthetic",
                      "config": {"workload": "cfg2 prefill qmm: qkv 3840x8192, o 4096x3840, gate/up 3840x30720, "
                                             f"down 15360x3840 at M = {args.qmm_m}"},
                      "roofline": {"bound": "tensor", "achieved": round(value, 1), "peak": tf_peak, "unit": "TFLOP/s",
                                   "frac": round(value / tf_peak, 4), "traffic": None, "peak_source": src,
                                   "kernel": "qmm_tc_kernel"},
                      "per_m": rows, "gpu_launches": 4 * len(Ms) * args.steps, "clocks": clk.summary()}), flush=True)


# ------------------------------------------------------------------ prefill causal SDPA (config 2)
def run_sdpa_prefill(args, rank, world, local):
    """Config 2's attention: causal SDPA at M tokens over 16 query / 8 KV heads, head_dim
    256, on a local layer (window 1024) and a global layer (full context), one M-token
    chunk at position 0 through hyb_sdpa_prefill. value = useful TFLOP/s (4 H hd per
    visible query-key pair: QK^T and PV)."""
    import torch
    from hyperion_b200 import ops
    H, Hkv, hd = 16, 8, 256
    rows = []
    flop_tot = us_tot = 0.0
    g = torch.Generator(device="cuda").manual_seed(3)
    for M in [int(m) for m in args.qmm_m.split(",")]:
        q = torch.randn((M, H, hd), generator=g, device="cuda").to(torch.bfloat16)
        k = torch.randn((M, Hkv, hd), generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn((M, Hkv, hd), generator=g, device="cuda").to(torch.bfloat16)
        for window in (1024, 0):
            vis = sum(min(i + 1, window) if window else i + 1 for i in range(M))
            flops = 4.0 * H * hd * vis
            ops.sdpa_prefill(q, k, v, 0, 0, window)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                ops.sdpa_prefill(q, k, v, 0, 0, window)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / args.steps
            rows.append({"M": M, "window": window, "us": round(us, 1), "TFLOP/s": round(flops / (us * 1e-6) / 1e12, 1)})
            flop_tot += flops
            us_tot += us
    _, tf_peak, src = peaks()
    value = flop_tot / (us_tot * 1e-6) / 1e12
    print(json.dumps({"metric": "prefill causal SDPA TFLOP/s (cfg2: 16/8 heads, hd 256, window 1024 and global)",
                      "value": round(value, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
                      "higher_is_better": True, "dtype": "bf16, f32 acc", "data": "synthetic",
                      "config": {"workload": f"cfg2 causal SDPA at M = {args.qmm_m}"},
                      "roofline": {"bound": "tensor", "achieved": round(value, 1), "peak": tf_peak, "unit": "TFLOP/s",
                                   "frac": round(value / tf_peak, 4), "traffic": None, "peak_source": src,
                                   "kernel": "prefill_attn_tc_kernel"},
                      "per_case": rows}), flush=True)


# ------------------------------------------------------------------ single qmv shape (profiling)
def run_qmv_shape(args, rank, world, local):
    """One cfg-1 shape over enough distinct copies to exceed 2x L2 (the workload the
    committed ncu summaries under profiles/ capture)."""
    import torch
    from hyperion_b200 import ops
    K, N = (int(v) for v in args.shape.split(","))
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    nbytes = qmv_bytes(K, N)
    copies = max(1, -(-2 * 126 * 2 ** 20 // nbytes))
    bufs = []
    for _ in range(copies):
        w, s, b = make_q4(N, K, gen, dev)
        pk = ops.qmv_pack(w, s, b) if args.layout == "packed" else None
        if pk is not None:
            del w, s, b
            w = s = b = None
        bufs.append((w, s, b, pk, torch.randn(1, K, device=dev, generator=gen).to(torch.bfloat16),
                     torch.empty(1, N, dtype=torch.bfloat16, device=dev)))

    def one(w, s, b, pk, x, y):
        if pk is not None:
            ops.qmv_packed(x, pk, K, N, out=y)
        else:
            ops.quantized_matmul(x, w, s, b, out=y)

    for bf in bufs:  # warm-up launches (also what ncu's -s skips)
        one(*bf)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, args.steps)
    e0.record()
    for _ in range(reps):
        for bf in bufs:
            one(*bf)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    if rank == 0:
        print(json.dumps({"workload": f"qmv K={K} N={N} ({args.layout} layout)", "copies": copies,
                          "us_per_launch": round(us, 2),
                          "GB/s": round(nbytes / (us * 1e-6) / 1e9, 1), "bytes_per_launch": nbytes}), flush=True)


# ------------------------------------------------------------------ 12B decode (ours, default)
L2_BYTES = 126 * 2 ** 20


def time_qmv_shapes(shapes, dev, stream, rounds=5):
    """Per-launch time of qmv_packed_kernel for each (name, K, N, prologue, epilogue):
    a CUDA graph of back-to-back launches over distinct packed weight copies (together
    more than 2x L2, so every launch streams its weights from HBM), timed with CUDA events
    on the launching stream after a warm-up replay. Returns {name: microseconds}."""
    import torch
    from hyperion_b200 import ops
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321)
    out = {}
    for name, K, N, prologue, epilogue in shapes:
        copies = max(2, -(-2 * L2_BYTES // qmv_bytes(K, N)))
        bufs = []
        for _ in range(copies):
            w, sc, bi = make_q4(N, K, gen, dev)
            pk = ops.qmv_pack(w, sc, bi)
            del w, sc, bi
            x = torch.randn(K, device=dev, generator=gen).to(torch.bfloat16)
            y = torch.empty(N // 2 if epilogue else N, dtype=torch.bfloat16, device=dev)
            nw = (1 + 0.02 * torch.randn(K, device=dev, generator=gen)).to(torch.bfloat16)
            rs = torch.randn(K, device=dev, generator=gen).to(torch.bfloat16)
            ho = torch.empty(K, dtype=torch.bfloat16, device=dev)
            bufs.append((pk, x, y, nw, rs, ho))

        def launch_all():
            for pk, x, y, nw, rs, ho in bufs:
                if prologue == 2:
                    ops.qmv_packed(x, pk, K, N, prologue=2, epilogue=epilogue, norm_w=nw, resid=rs, post_w=nw,
                                   h_out=ho, out=y, stream=stream)
                else:
                    ops.qmv_packed(x, pk, K, N, prologue=prologue, epilogue=epilogue, norm_w=nw, out=y,
                                   stream=stream)

        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            launch_all()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch_all()
        with torch.cuda.stream(stream):
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(rounds):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) * 1e3 / (rounds * copies)
        del g, bufs
    torch.cuda.empty_cache()
    return out


def decode_shapes(T: int):
    """The decode projections of the 12B-shaped model on one of T tensor-parallel ranks,
    as the engine launches them: (name, K, N, prologue, epilogue, launches per token).
    Prologue 1 = norm, 2 = residual + norm; epilogue 1 = GeGLU over interleaved rows."""
    return [("qkv_sliding", 3840, 8192 // T, 2, 0, 40), ("qkv_global", 3840, 6144 // T, 2, 0, 8),
            ("o", 4096 // T, 3840, 0, 0, 48), ("gate_up", 3840, 30720 // T, 2, 1, 48),
            ("down", 15360 // T, 3840, 0, 0, 48), ("lm_head", 3840, 262144 // T, 2, 0, 1)]


def run_decode(args, rank, world, local):
    """The default workload: cfg3 decode through hyp_decode_block, tensor-parallel over
    the job's ranks (see the module docstring)."""
    import torch
    import hyperion_b200 as hb
    from hyperion_b200.synth import config3
    geo = config3()
    why = hb.tp_shard_check(geo, world)
    if why:
        raise SystemExit(f"config 3 does not split over {world} ranks: {why}")
    tp = None
    if world > 1:
        import torch.distributed as dist
        obj = [hb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp = (rank, world, obj[0])
    dev = torch.device("cuda", local)
    seed = 1
    t0 = time.perf_counter()
    eng = hb.Engine(geo, synthetic_seed=seed, tp=tp)
    load_s = max_over_ranks(time.perf_counter() - t0, world)
    ctx = args.ctx
    prompt = [int(t) for t in torch.randint(0, geo.vocab_size, (ctx,), generator=torch.Generator().manual_seed(5))]
    warm = eng.new_kv()  # the first prefill pays one-time costs (module load, pools, tensor maps)
    warm.prefill(prompt)
    warm.close()
    kv = eng.new_kv()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    f0, _ = kv.prefill(prompt)
    prefill_s = max_over_ranks(time.perf_counter() - t0, world)

    # parity of the tensor-parallel run: 16 greedy steps, teacher-forced against TP = 1
    parity = None
    if world > 1:
        toks = [f0.token_id]
        for _ in range(16):
            f, _ = kv.decode(1)
            toks.append(f.token_id)
        barrier(world)
        if rank == 0:
            ref = hb.Engine(geo, synthetic_seed=seed)
            rkv = ref.new_kv()
            rf, _ = rkv.prefill(prompt)
            agree = [rf.token_id == toks[0]]
            for i in range(16):
                f, _ = rkv.decode(1, forced=toks[i])
                agree.append(f.token_id == toks[i + 1])
            rkv.close()
            ref.close()
            torch.cuda.empty_cache()
            parity = {"vs": "same model at TP 1 on rank 0, teacher-forced", "steps": 17,
                      "greedy_agreement": round(sum(agree) / len(agree), 4)}
        barrier(world)

    stream = torch.cuda.ExternalStream(eng.stream())
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            kv.decode(1)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            kv.decode(1)  # hyp_decode_block: host token in, greedy result read back every step
        e1.record(stream)
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - w0) * 1e3 / args.steps
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
        wall_ms = max_over_ranks(wall_ms, world)
        # the dominant kernel, live: the decode projections at this rank's shapes
        qstream = torch.cuda.Stream(device=dev)
        shapes = decode_shapes(world)
        per = time_qmv_shapes([sh[:5] for sh in shapes], dev, qstream)
        sweep = None
        if world == 1 and not args.no_sweep:
            cfg1 = PROJ + [LM_HEAD]
            sp = time_qmv_shapes([(nm, K, N, 0, 0) for nm, K, N in cfg1], dev, qstream)
            sb = 48 * sum(qmv_bytes(K, N) for _, K, N in PROJ) + qmv_bytes(LM_HEAD[1], LM_HEAD[2])
            st = 48 * sum(sp[nm] for nm, _, _ in PROJ) + sp[LM_HEAD[0]]
            sweep = {"workload": "cfg1 shapes in 12B decode-token proportions (48 x q,k,v,o,gate,up,down + "
                                 "lm_head), no prologue",
                     "value": round(sb / (st * 1e-6) / 1e9, 1), "unit": "GB/s",
                     "frac": round(sb / (st * 1e-6) / 1e9 / peaks()[0], 4),
                     "per_shape": [{"shape": f"{nm} K={K} N={N}", "us": round(sp[nm], 2),
                                    "frac": round(qmv_bytes(K, N) / (sp[nm] * 1e-6) / 1e9 / peaks()[0], 3)}
                                   for nm, K, N in cfg1]}
    tok_s = 1e3 / ms
    if rank != 0:
        return
    hbm, _, src = peaks()
    mix_bytes = sum(c * qmv_bytes(K, N) for _, K, N, _, _, c in shapes)
    mix_us = sum(c * per[nm] for nm, _, _, _, _, c in shapes)
    achieved = mix_bytes / (mix_us * 1e-6) / 1e9
    # whole-step bytes per token on this rank: its weight shard + its KV heads
    kv_bytes = 0
    for i, kind in enumerate(geo.layer_types):
        n = min(geo.sliding_window, ctx + args.warmup) if kind == 0 else ctx + args.warmup
        kv_bytes += 2 * n * geo.n_kv(i) * geo.head_dim(i) * 2 // world
    step_bytes = mix_bytes + kv_bytes
    traffic = None
    tp_path = os.path.join(REPO, "profiles", "qmv_traffic.json")
    if os.path.exists(tp_path) and world == 1:
        with open(tp_path) as f:
            traffic = json.load(f).get("dram_bytes_per_launch_decode_mix")
    # our kernels per token: embed, 5 per layer (qkv, fused attention, o, gate/up, down),
    # lm_head, soft-cap/top-k stages 1 and 2, and with TP the candidate kernel
    launches_per_step = 1 + 5 * len(geo.layer_types) + 3 + (1 if world > 1 else 0)
    line = {"metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u4/bf16->f32", "data": "synthetic",
            "config": {"workload": f"cfg3 12B-shaped decode, ctx {ctx}, batch 1", "parallelism": f"tp{world}",
                       "load_s": round(load_s, 2), "prefill_s": round(prefill_s, 3),
                       "prefill_tok_s": round(ctx / prefill_s, 1), "l2": "inputs larger than L2 (6.6 GB of "
                       "weights per token; roofline copies > 2x L2)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": src,
                         "kernel": "qmv_packed_kernel, mix-weighted over one token's decode projections at this "
                                   "rank's shapes (CUDA events, back-to-back graph launches)"},
            "per_shape": [{"shape": f"{nm} K={K} N={N}", "launches_per_token": c, "us": round(per[nm], 2),
                           "frac": round(qmv_bytes(K, N) / (per[nm] * 1e-6) / 1e9 / hbm, 3)}
                          for nm, K, N, _, _, c in shapes],
            "step_roofline": {"bytes_per_token_per_rank": step_bytes,
                              "achieved": round(step_bytes / (ms * 1e-3) / 1e9, 1),
                              "frac": round(step_bytes / (ms * 1e-3) / 1e9 / hbm, 4)},
            "gpu_launches": launches_per_step * args.steps,
            "e2e": {"value": round(1e3 / wall_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 64 if world == 1 else 16 * world,
                    "path": "hyp_decode_block(n_tokens=1) via ctypes on every rank (token id in, greedy result "
                            "out each step), host wall clock, max over ranks"},
            "clocks": clk.summary()}
    if parity is not None:
        line["parity"] = parity
    if sweep is not None:
        line["qmv_sweep"] = sweep
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_baseline(ctx, args.cpu_seconds)
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ speculative verify
def run_spec_verify(args, rank, world, local):
    """Greedy speculative verify on the 12B-shaped model after a --ctx prefill: one pass
    checks D draft tokens (D = 1, 3, 7 by default, --drafts) by running D + 1 rows through
    the chunked forward and sampling every row (hyb_verify). Each pass is timed with CUDA
    events on the engine stream beside a plain decode step of the same state; value = rows
    per second of the largest D (the tokens/s speculative decoding reaches when every draft
    is accepted)."""
    import numpy as np
    import torch
    import hyperion_b200 as hb
    from hyperion_b200.synth import config3
    geo = config3()
    eng = hb.Engine(geo, synthetic_seed=1 + rank)
    ctx = args.ctx
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, geo.vocab_size, ctx).tolist()
    kv = eng.new_kv()
    kv.prefill(prompt)
    stream = torch.cuda.ExternalStream(eng.stream())
    drafts = [int(d) for d in args.drafts.split(",")]

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps, (time.perf_counter() - w0) * 1e3 / args.steps

    with ClockSampler(local) as clk:
        dec_ms, _ = timed(lambda: kv.decode(1))
        per, wall = {}, {}
        for d in drafts:
            draws = [rng.integers(0, geo.vocab_size, d).tolist() for _ in range(args.warmup + args.steps)]
            it = iter(draws)
            per[d], wall[d] = timed(lambda: kv.verify(next(it)))
    if rank != 0:
        return
    d = max(drafts)
    rows_s = (d + 1) / (per[d] * 1e-3)
    w_bytes = 48 * sum(qmv_bytes(K, N) for _, K, N in PROJ) + qmv_bytes(3840, 262144)
    hbm, _, src = peaks()
    print(json.dumps({
        "metric": "speculative verify rows/s (12B-shaped, all drafts accepted)", "value": round(rows_s, 1),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per[d], 4),
        "higher_is_better": True, "vs_baseline": None, "dtype": "u4/bf16->f32", "data": "synthetic",
        "config": {"workload": f"cfg3 12B-shaped verify of {drafts} drafts at ctx ~{ctx}, batch 1",
                   "decode_ms": round(dec_ms, 4),
                   "verify_ms": {str(k): round(v, 4) for k, v in per.items()},
                   "verify_wall_ms": {str(k): round(v, 4) for k, v in wall.items()},
                   "speedup_at_full_acceptance": {str(k): round((k + 1) * dec_ms / v, 2) for k, v in per.items()},
                   "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": round(w_bytes / (per[d] * 1e-3) / 1e9, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(w_bytes / (per[d] * 1e-3) / 1e9 / hbm, 4), "traffic": None,
                     "peak_source": src, "kernel": "whole verify pass (weight bytes per pass)"},
        "e2e": {"value": round((d + 1) / (wall[d] * 1e-3), 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * d,
                "d2h_bytes_per_step": 8 * (d + 1), "path": "hyb_verify via ctypes, host wall clock"},
        "clocks": clk.summary()}), flush=True)


# ------------------------------------------------------------------ decode attention alone (profiling)
def run_attn_decode(args, rank, world, local):
    """The fused decode attention over the 48 layers of the 12B-shaped model at --ctx:
    40 sliding layers (1024 keys) and 8 global layers (ctx + 1 keys), each with its own
    K/V cache, one token per step, captured in a CUDA graph. value = K/V bytes / time."""
    import torch
    from hyperion_b200 import ops
    from hyperion_b200.synth import config3
    geo = config3()
    H, ctx = 16, args.ctx
    g = torch.Generator(device="cuda").manual_seed(7)
    layers = []
    for i, kind in enumerate(geo.layer_types):
        hkv, hd = geo.n_kv(i), geo.head_dim(i)
        cap = 1032 if kind == 0 else (ctx + 1 + 255) // 256 * 256
        n_keys = min(1024, ctx + 1) if kind == 0 else ctx + 1
        kc = torch.randn((cap, hkv, hd), generator=g, device="cuda").to(torch.bfloat16)
        vc = torch.randn((cap, hkv, hd), generator=g, device="cuda").to(torch.bfloat16)
        qkv = (3 * torch.randn((H + 2 * hkv) * hd, generator=g, device="cuda")).to(torch.bfloat16)
        nw = (1 + 0.02 * torch.randn(hd, generator=g, device="cuda")).to(torch.bfloat16)
        inv = (1.0 / (10000.0 ** (torch.arange(0, hd, 2, device="cuda").float() / hd))).contiguous()
        out = torch.empty((H, hd), dtype=torch.bfloat16, device="cuda")
        layers.append((qkv, nw, inv, kc, vc, n_keys, out, 2 * 2 * n_keys * hkv * hd))
    stream = torch.cuda.Stream()

    def step():
        for qkv, nw, inv, kc, vc, n_keys, out, _ in layers:
            ops.sdpa_decode_fused(qkv, False, nw, nw, inv, kc, vc, ctx, n_keys, H, out=out, stream=stream)

    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    kv_bytes = sum(l[7] for l in layers)
    hbm, _, src = peaks()
    gbs = kv_bytes / (us * 1e-6) / 1e9
    print(json.dumps({"metric": "fused decode attention K/V GB/s (48 cfg3 layers per step)", "value": round(gbs, 1),
                      "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(us / 1e3, 4), "higher_is_better": True,
                      "config": {"workload": f"cfg3 decode attention, ctx {ctx}: 40 x 1024-key sliding + 8 x "
                                             f"{ctx + 1}-key global layers", "kv_bytes_per_step": kv_bytes,
                                 "l2": "inputs larger than L2"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                   "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src,
                                   "kernel": "decode_attn_fused_kernel"},
                      "us_per_layer_avg": round(us / len(layers), 2), "gpu_launches": len(layers) * args.steps,
                      "clocks": clk.summary()}), flush=True)


# ------------------------------------------------------------------ 27B-shaped tensor-parallel decode (config 4)
def run_tp_decode(args, rank, world, local):
    """Config 4: the 27B-shaped decoder split over the job's GPUs (one rank per GPU,
    column/row-parallel projections, NCCL all-reduce after o_proj and down_proj,
    vocab-parallel lm_head), greedy decode after a --ctx prefill. --batch B > 1 decodes B
    sequences per step through hyb_decode_batch: the prefilled context is cloned B times
    (hyb_kvstate_clone) with distinct next tokens, so every sequence attends over ctx keys."""
    import torch
    import hyperion_b200 as hb
    from hyperion_b200.synth import config4
    geo = config4()
    why = hb.tp_shard_check(geo, world)
    if why:
        raise SystemExit(f"config 4 does not split over {world} ranks: {why}")
    tp = None
    if world > 1:
        import torch.distributed as dist
        obj = [hb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        tp = (rank, world, obj[0])
    eng = hb.Engine(geo, synthetic_seed=1, tp=tp)
    ctx = args.ctx
    prompt = [int(t) for t in torch.randint(0, geo.vocab_size, (ctx,), generator=torch.Generator().manual_seed(5))]
    kv = eng.new_kv()
    barrier(world)
    t0 = time.perf_counter()
    kv.prefill(prompt)
    prefill_s = max_over_ranks(time.perf_counter() - t0, world)
    B = args.batch
    seqs = [kv] if B == 1 else [kv.clone(last_token=int(t)) for t in
                                torch.randint(0, geo.vocab_size, (B,), generator=torch.Generator().manual_seed(9))]
    step = (lambda: kv.decode(1)) if B == 1 else (lambda: eng.decode_batch(seqs))
    stream = torch.cuda.ExternalStream(eng.stream())
    for _ in range(args.warmup):
        step()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            step()  # host tokens in, greedy results read back every step
        e1.record(stream)
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - w0) * 1e3 / args.steps
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    wall_ms = max_over_ranks(wall_ms, world)
    if rank != 0:
        return
    # bytes each rank streams per step: its shard of the projections and lm_head rows once,
    # plus its KV heads of every sequence
    per_layer = (qmv_bytes(5376, 8192 + 2 * 4096) + qmv_bytes(4096, 5376) + qmv_bytes(5376, 2 * 21504) +
                 qmv_bytes(21504, 5376)) / world
    w_bytes = 62 * per_layer + qmv_bytes(5376, 262144) / world
    kv_bytes = 0
    for i, kind in enumerate(geo.layer_types):
        n = min(geo.sliding_window, ctx + args.warmup) if kind == 0 else ctx + args.warmup
        kv_bytes += 2 * n * geo.n_kv(i) * geo.head_dim(i) * 2
    step_bytes = w_bytes + B * kv_bytes / world
    hbm, _, src = peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    launches = (1 + 5 * 62 + 4) if B == 1 else (2 + 11 * 62 + 4 + (1 if world > 1 else 0))
    print(json.dumps({"metric": f"27B-shaped tensor-parallel decode tok/s (cfg4, batch {B})",
                      "value": round(B * 1e3 / ms, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
                      "scaling": "strong", "vs_baseline": None, "dtype": "u4/bf16->f32", "data": "synthetic",
                      "config": {"workload": f"cfg4 27B-shaped decode, ctx {ctx}, batch {B}",
                                 "parallelism": f"tp{world}", "prefill_s": round(prefill_s, 3),
                                 "l2": "inputs larger than L2"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                   "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src,
                                   "kernel": "whole decode step per rank (its weight shard + its KV heads of "
                                             "every sequence)"},
                      "gpu_launches": launches * args.steps,
                      "e2e": {"value": round(B * 1e3 / wall_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                              "d2h_bytes_per_step": (64 if B == 1 else 8 * B) * world,
                              "path": ("hyp_decode_block(n_tokens=1)" if B == 1 else "hyb_decode_batch") +
                                      " on every rank, host wall clock"},
                      "clocks": clk.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode",
                    choices=["qmv", "decode", "qmv-shape", "attn-decode", "qmm", "tp-decode", "sdpa-prefill",
                             "spec-verify"])
    ap.add_argument("--drafts", default="1,3,7", help="draft lengths for --workload spec-verify (1..8)")
    ap.add_argument("--qmm-m", default="512,2048,8192", help="token counts for --workload qmm")
    ap.add_argument("--shape", default="3840,262144", help="K,N for --workload qmv-shape")
    ap.add_argument("--layout", default="packed", choices=["packed", "mlx"], help="weights for qmv-shape")
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=1, help="tp-decode: sequences decoded per step (1..64)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="decode: skip the config-1 qmv sweep keys")

    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return
    from hyperion_b200.build import LIB
    if not os.path.exists(LIB):
        raise SystemExit("libhyperion_mlx.so is not built (python -m hyperion_b200.build)")
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.workload == "qmv":
            run_qmv(args, rank, world, local)
        elif args.workload == "tp-decode":
            run_tp_decode(args, rank, world, local)
        elif args.workload == "sdpa-prefill":
            run_sdpa_prefill(args, rank, world, local)
        elif args.workload == "qmm":
            run_qmm(args, rank, world, local)
        elif args.workload == "attn-decode":
            run_attn_decode(args, rank, world, local)
        elif args.workload == "qmv-shape":
            run_qmv_shape(args, rank, world, local)
        elif args.workload == "spec-verify":
            run_spec_verify(args, rank, world, local)
        else:
            run_decode(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            barrier(world)
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
