#!/usr/bin/env python
"""Benchmark of the B200 decode hot path (rdna4-quant INT4/INT8 dequant-GEMV).

Headline workload (benchmark config 1): the Qwen3-14B decode-layer INT4 GEMV
set — qkv 5120->7168, o 5120->5120, gate_up 5120->34816, down 17408->5120 (the
reference's fused runtime shapes, int4_engine_v5.py:136-162) — at batch 1, with
the H32 FWHT (qkv/o/gate_up inputs) and SiLU*up+FWHT (down input) fused into
the GEMV prologue.  One step runs that set over 40 distinct layers (8.3 GB of
weights, far above the 126 MB L2, so every step streams from HBM).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun as independent replicas (the GEMV set does not
shard; no collective), value = bytes of all ranks / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "rdna4-quant_b200"))

HID, INTER, NQ, NKV, HD = 5120, 17408, 40, 8, 128
QKV_N = (NQ + 2 * NKV) * HD
LAYER_SHAPES = [  # (name, N, K, prologue)
    ("qkv", QKV_N, HID, "fwht"),
    ("o", HID, NQ * HD, "fwht"),
    ("gate_up", 2 * INTER, HID, "fwht"),
    ("down", HID, INTER, "silu_fwht"),
]
METRIC = "INT4 GEMV HBM GB/s (Qwen3-14B decode-layer GEMV set)"
# dram__bytes_read.sum + dram__bytes_write.sum of one gate_up launch at B=1,
# from the ncu capture summarised in profiles/gemv_tma_int4_gate_up_b1.md
TRAFFIC_GATE_UP_B1 = 111478016 + 4093696


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-ctx", default="128,2048",
                    help="prompt lengths for the Qwen3-14B decode tok/s measurement ('' skips it)")
    ap.add_argument("--decode-tokens", type=int, default=256)
    ap.add_argument("--prefill-tokens", type=int, default=512,
                    help="prompt length of the prefill tok/s measurement (0 skips it)")
    ap.add_argument("--decode-probe", action="store_true",
                    help="build the 40-layer model, decode 3 tokens eagerly and exit (for ncu)")
    ap.add_argument("--moe-batches", default="1,16,64",
                    help="batches of the config-4 MoE decode measurement ('' skips it)")
    ap.add_argument("--moe-tokens", type=int, default=32)
    ap.add_argument("--gemv-batches", default="4,16",
                    help="extra batch sizes of the GEMV set (config 1 names B = 1, 4, 16); '' skips")
    ap.add_argument("--moe-probe", type=int, default=0,
                    help="ncu target: 3 eager MoE decode steps of a 2-layer config-4 model at this batch")
    ap.add_argument("--gemm-probe", action="store_true",
                    help="run the INT4 tcgen05 prefill GEMM (M=512, qkv shape) 4 times and exit (for ncu)")
    ap.add_argument("--kernel-probe", default=None, choices=[n for n, *_ in LAYER_SHAPES],
                    help="run one GEMV of this shape 4 times and exit (for ncu captures)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def step_bytes(B, layers):
    from r4q.synth import gemv_bytes
    return layers * sum(gemv_bytes("int4", B, N, K) for _, N, K, _ in LAYER_SHAPES)


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        try:
            rows = [r.split(",") for r in Path(self.f.name).read_text().strip().splitlines()]
        except Exception:
            rows = []
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ ours ----
def build_layers(B, layers, device, seed=1234):
    import torch
    from r4q import synth
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(layers):
        L = {}
        for name, N, K, _ in LAYER_SHAPES:
            _, w, s = synth.linear_int4(N, K, g, device)
            L[name] = (w, s)
        out.append(L)
    return out


def gemv_set_batches(a, dev, layers, peak, Lpro, ws):
    """Config 1 at the other batch sizes it names: the same 40-layer GEMV set
    (same weights) through a CUDA graph, B activation rows per GEMV; GB/s of
    algorithmic bytes per GPU and the fraction of the measured copy peak."""
    import torch
    from r4q import ops
    res = []
    for B in [int(b) for b in a.gemv_batches.split(",") if b]:
        g = torch.Generator(device=dev).manual_seed(7 + B)
        x = torch.randn(B, HID, generator=g, device=dev).half()
        att = torch.randn(B, NQ * HD, generator=g, device=dev).half()
        qkv = torch.empty(B, QKV_N, device=dev, dtype=torch.float16)
        o = torch.empty(B, HID, device=dev, dtype=torch.float16)
        gu = torch.randn(B, 2 * INTER, generator=g, device=dev).half()
        d = torch.empty(B, HID, device=dev, dtype=torch.float16)
        bufs = (x, qkv, att, o, gu, d)
        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            for _ in range(2):
                run_set(ops, Lpro, layers, bufs)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            run_set(ops, Lpro, layers, bufs)
        with torch.cuda.stream(s):
            for _ in range(3):
                graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        with torch.cuda.stream(s):
            e0.record(s)
            for _ in range(reps):
                graph.replay()
            e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        gbs = step_bytes(B, a.layers) / (ms * 1e-3) / 1e9
        res.append({"batch": B, "GBps_per_gpu": round(gbs, 1), "ms_per_step": round(ms, 4),
                    "frac": round(gbs / peak, 4)})
        del graph
    return {"workload": f"cfg1 GEMV set x{a.layers} layers (same weights as the headline)",
            "gpus": ws, "parallelism": f"replicas x{ws}", "results": res}


def run_set(ops, Lpro, layers, bufs):
    """Launch the GEMV set of every layer once (no host sync)."""
    x, qkv, att, o, gu, d = bufs
    for L in layers:
        ops.gemv("int4", x, *L["qkv"], QKV_N, HID, prologue=Lpro["fwht"], out=qkv)
        ops.gemv("int4", att, *L["o"], HID, NQ * HD, prologue=Lpro["fwht"], out=o)
        ops.gemv("int4", x, *L["gate_up"], 2 * INTER, HID, prologue=Lpro["fwht"], out=gu)
        ops.gemv("int4", gu, *L["down"], HID, INTER, prologue=Lpro["silu_fwht"], out=d)


def cpu_port_setup(B):
    """Random nibbles/scales for one layer's GEMV set (values do not change the
    CPU cost of dequant + matmul)."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "oracle"))
    import r4q_oracle as O
    rng = np.random.default_rng(0)
    mats = []
    for _, N, K, _ in LAYER_SHAPES:
        packed = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
        s = (rng.random((N, K // 32)) * 0.01 + 1e-3).astype(np.float16)
        z = rng.integers(0, 16, size=(N, K // 32)).astype(np.uint8)
        mats.append((N, K, packed, O.interleave_scale_zero(s, z)))
    x = rng.standard_normal((B, 2 * INTER)).astype(np.float16)
    return mats, x, B


def cpu_port_run(setup, threads, only=None):
    """The reference's CPU math for the GEMV set — dequant to fp16
    (int4_quant_v2.py:105-127) then fp32 matmul — through the oracle port,
    threaded over row chunks.  Returns (algorithmic bytes, seconds)."""
    import numpy as np
    import r4q_oracle as O
    from concurrent.futures import ThreadPoolExecutor
    from r4q.synth import gemv_bytes
    mats, x, B = setup
    sel = mats if only is None else [mats[only]]
    t0 = time.perf_counter()
    nbytes = 0
    with ThreadPoolExecutor(max_workers=threads) as pool:
        for (N, K, packed, sz) in sel:
            xin = x[:, :K].astype(np.float32)

            def part(r, packed=packed, sz=sz, xin=xin):
                W = O.dequant_int4_runtime(packed[r[0]:r[-1] + 1], sz[r[0]:r[-1] + 1])
                return xin @ W.astype(np.float32).T
            ys = list(pool.map(part, np.array_split(np.arange(N), threads)))
            np.concatenate(ys, axis=1).astype(np.float16)
            nbytes += gemv_bytes("int4", B, N, K)
    return nbytes, time.perf_counter() - t0


def main_ours(a):
    import torch
    import torch.distributed as dist
    from r4q import lib as Lb
    from r4q import ops
    ws, rank, local = dist_env()
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B = a.batch
    layers = build_layers(B, a.layers, dev)
    Lpro = {"fwht": Lb.PRO_FWHT, "silu_fwht": Lb.PRO_SILU_FWHT}
    gx = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(B, HID, generator=gx, device=dev).half()
    att = torch.randn(B, NQ * HD, generator=gx, device=dev).half()
    qkv = torch.empty(B, QKV_N, device=dev, dtype=torch.float16)
    o = torch.empty(B, HID, device=dev, dtype=torch.float16)
    gu = (torch.randn(B, 2 * INTER, generator=gx, device=dev)).half()
    d = torch.empty(B, HID, device=dev, dtype=torch.float16)
    bufs = (x, qkv, att, o, gu, d)
    nlaunch = 4 * a.layers

    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        for _ in range(2):
            run_set(ops, Lpro, layers, bufs)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        run_set(ops, Lpro, layers, bufs)
    torch.cuda.synchronize()

    with torch.cuda.stream(s):
        for _ in range(a.warmup):
            graph.replay()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        time.sleep(0.3)
        with torch.cuda.stream(s):
            e0.record(s)
            for _ in range(a.steps):
                graph.replay()
            e1.record(s)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
        torch.cuda.synchronize()

    per_rank = step_bytes(B, a.layers)
    value = per_rank * ws / (ms * 1e-3) / 1e9

    # ---- e2e through the public API with host buffers (pinned) ----
    xh = x.cpu().pin_memory()
    yh = torch.empty(B, HID, dtype=torch.float16).pin_memory()
    with torch.cuda.stream(s):
        for _ in range(2):
            x.copy_(xh, non_blocking=True)
            run_set(ops, Lpro, layers, bufs)
            yh.copy_(d, non_blocking=True)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, a.steps // 4)
    with torch.cuda.stream(s):
        ee0.record(s)
        for _ in range(e2e_steps):
            x.copy_(xh, non_blocking=True)
            run_set(ops, Lpro, layers, bufs)
            yh.copy_(d, non_blocking=True)
        ee1.record(s)
    torch.cuda.synchronize()
    e2e_ms = ee0.elapsed_time(ee1) / e2e_steps
    if ws > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = per_rank * ws / (e2e_ms * 1e-3) / 1e9

    peak, peak_kind = peaks()
    # dominant kernel: the gate_up GEMV (54 % of the step's bytes), timed alone
    # with CUDA events on its own stream over the 40 layers' distinct weights
    from r4q.synth import gemv_bytes
    gg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gg, stream=s):
        for L in layers:
            ops.gemv("int4", x, *L["gate_up"], 2 * INTER, HID, prologue=Lpro["fwht"], out=gu)
    with torch.cuda.stream(s):
        gg.replay()
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kreps = 5
    with torch.cuda.stream(s):
        k0.record(s)
        for _ in range(kreps):
            gg.replay()
        k1.record(s)
    torch.cuda.synchronize()
    k_us = k0.elapsed_time(k1) * 1e3 / (kreps * a.layers)
    k_bytes = gemv_bytes("int4", B, 2 * INTER, HID)
    achieved = k_bytes / (k_us * 1e-6) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xfp16->fp32",
        "data": "synthetic (seeded N(0,0.02)+0.1% x20 outliers, H32-rotated, RTN INT4 asym)",
        "config": {"workload": f"cfg1 Qwen3-14B decode-layer GEMV set x{a.layers} layers, B={B}",
                   "batch": B, "layers": a.layers, "shapes": [f"{n}:{K}->{N}" for n, N, K, _ in LAYER_SHAPES],
                   "prologues": "fwht on qkv/o/gate_up inputs, silu*up+fwht on down input",
                   "l2": "inputs larger than L2 (8.3 GB distinct weights per step)",
                   "parallelism": f"replicas x{ws}", "timing": "CUDA graph replay, CUDA events"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": TRAFFIC_GATE_UP_B1 if B == 1 else None,
                     "kernel": "gemv_tma_kernel<INT4> gate_up 5120->34816",
                     "launch_us": round(k_us, 2), "algorithmic_bytes_per_launch": k_bytes,
                     "peak_source": peak_kind + " (burst copy; of measured)",
                     "step_avg_GBps": round(per_rank / (ms * 1e-3) / 1e9, 1)},
        "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": 2 * B * HID,
                "d2h_bytes_per_step": 2 * B * HID,
                "api": "r4q.ops.gemv per call (ctypes C ABI), pinned host x in, y out"},
        "gpu_launches": nlaunch * a.steps,
        "clocks": clk.summary(),
    }
    if a.gemv_batches:
        line["gemv_batches"] = gemv_set_batches(a, dev, layers, peak, Lpro, ws)
    if a.decode_ctx:
        del layers
        torch.cuda.empty_cache()
        line["decode"] = decode_tok_s(a, dev, peak, ws, rank)
    if a.moe_batches:
        torch.cuda.empty_cache()
        line["moe"] = moe_tok_s(a, dev, peak, ws, rank)
    if rank == 0 and ws == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        setup = cpu_port_setup(B)
        nb, dt, reps = 0, 0.0, 0
        while dt < 10.0 and reps < 200:          # about 10 s of host work
            b_, t_ = cpu_port_run(setup, threads)
            nb, dt, reps = nb + b_, dt + t_, reps + 1
        line["cpu_baseline"] = {"value": round(nb / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
                                "kind": "port", "seconds": round(dt, 2),
                                "sample": f"{reps} passes over one layer's GEMV set (qkv,o,gate_up,down) "
                                          f"of the {a.layers}, B={B}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def main_reference(a):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    mats = cpu_port_setup(a.batch)
    tot_b, tot_t, per = 0, 0.0, []
    for i in range(a.warmup + a.steps):
        nb, dt = cpu_port_run(mats, threads, only=i % len(LAYER_SHAPES))
        if i >= a.warmup:
            tot_b += nb
            tot_t += dt
            per.append(dt)
    value = tot_b / tot_t / 1e9
    ms = statistics.median(per) * 1e3
    sample = "one GEMV of the layer set per step, cycling qkv/o/gate_up/down"
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": ws, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4xfp16->fp32", "data": "synthetic random nibbles/scales",
            "config": {"workload": f"cfg1 Qwen3-14B decode-layer GEMV set, B={a.batch}",
                       "batch": a.batch, "shapes": [f"{n}:{K}->{N}" for n, N, K, _ in LAYER_SHAPES],
                       "sample": "1 layer per step (of 40)"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def decode_tok_s(a, dev, peak, ws=1, rank=0):
    """benchmark config 3: 40-layer Qwen3-14B-shaped decode (random-init,
    80 % INT4 / 20 % INT8 groups by seed, fp16 embedding + lm_head), KV cache
    pre-filled for `ctx` prompt positions, greedy decode of `tokens` tokens,
    each one CUDA-graph launch of step + device argmax + embedding lookup
    (r4q_decode_loop, the engine of int4_hip.decode_loop).  TP=ws>1
    (torchrun, one rank per GPU): each rank holds its shard (r4q.tp) and the
    step's exchanges run over NVLink peer memory (r4q_comm); time is the max
    over ranks."""
    import torch
    import torch.distributed as dist
    from r4q import synth, tp
    cfg = synth.qwen3_14b_config()
    ctxs = [int(c) for c in a.decode_ctx.split(",") if c]
    max_seq = max(ctxs) + a.decode_tokens + 16
    m = synth.build_decode_model(cfg, dev, seed=3, max_seq=max_seq)
    wbytes, int8_groups = m['weight_bytes'], m['int8_groups']
    dec = None
    if ws > 1:
        sh = tp.shard_decode_model(m, cfg, rank, ws)
        del m
        torch.cuda.empty_cache()
        m = sh
        comm = tp.Comm(rank, ws, max_batch=1, hidden=cfg['hidden'], vocab=cfg['vocab'])
        dec = tp.TPDecoder(m, cfg, comm, batch=1)
    res = []
    from r4q import decode as rdec
    for ctx in ctxs:
        gen = torch.Generator(device=dev).manual_seed(ctx)
        if ws == 1:
            # the prompt through the prefill path: its K/V fill positions 0..ctx-1
            from r4q import prefill as rpre
            ids = torch.randint(0, cfg['vocab'], (ctx,), generator=gen, device=dev)
            last = rpre.prefill_logits(m['embed'][ids], m['qkv_w'], m['qkv_s'], m['o_w'], m['o_s'], m['gu_w'],
                                       m['gu_s'], m['down_w'], m['down_s'], m['in_norm_w'], m['post_norm_w'],
                                       m['q_norm_w'], m['k_norm_w'], m['rope_cos'], m['rope_sin'],
                                       cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'], cfg['hidden'],
                                       cfg['intermediate'], cfg['rms_eps'], m['final_norm_w'], m['lm_w'], m['lm_s'],
                                       cfg['vocab'], k_caches=m['k_caches'], v_caches=m['v_caches'],
                                       last_only=True)
            tok = last.reshape(-1).argmax().reshape(1)
        else:
            synth.fill_kv_synthetic(m, ctx, seed=ctx)
            tok = torch.randint(0, cfg['vocab'], (1,), generator=gen, device=dev)
        h0 = m['embed'][tok].reshape(1, -1).contiguous()
        if dec is not None:
            loop = lambda start, n: dec.loop(m['embed'], h0, start, n)
        else:
            c1 = rdec.get_context(
                m['qkv_w'], m['qkv_s'], m['o_w'], m['o_s'], m['gu_w'], m['gu_s'], m['down_w'], m['down_s'],
                m['in_norm_w'], m['post_norm_w'], m['q_norm_w'], m['k_norm_w'], m['rope_cos'], m['rope_sin'],
                cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'], cfg['hidden'], cfg['intermediate'],
                cfg['rms_eps'], m['k_caches'], m['v_caches'], m['final_norm_w'], m['lm_w'], m['lm_s'],
                cfg['vocab'], batch=1)
            loop = lambda start, n: c1.loop(m['embed'], h0, start, n)
        loop(ctx, 3)                                   # warm-up (graph capture)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        toks = loop(ctx, a.decode_tokens)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / a.decode_tokens
        if ws > 1:
            comm.status()
            tt = torch.tensor([ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        kv = cfg['num_layers'] * 2 * cfg['num_kv_heads'] * cfg['head_dim'] * (ctx + a.decode_tokens // 2)
        byt = (wbytes + kv) // ws + 2 * cfg['hidden']          # per GPU
        res.append({"ctx": ctx, "tok_s": round(1e3 / ms, 1), "ms_per_token": round(ms, 4),
                    "bytes_per_token_per_gpu": byt, "GBps_per_gpu": round(byt / ms / 1e6, 1),
                    "roofline_tok_s": round(peak * 1e9 / byt, 1),
                    "frac": round((byt / ms / 1e6) / peak, 4)})
    pre = None
    if ws == 1 and a.prefill_tokens:
        pre = prefill_tok_s(a, dev, m, cfg)
    if dec is not None:
        dec = None
        from r4q import decode
        decode.clear_contexts()
        dist.barrier()
        comm.close()
    return {"model": "Qwen3-14B shape, random init", "int8_groups": int8_groups,
            "lm_head": "fp16", "batch": 1, "tokens": a.decode_tokens, "tp": ws,
            "kv": ("prompt of seeded random ids through prefill_logits (writes K/V of positions 0..ctx-1)"
                   if ws == 1 else "prompt K/V pre-filled with seeded FP8 values (prefill is single-GPU)"),
            "api": ("r4q decode_loop (int4_hip.decode_loop's engine): one CUDA-graph launch per token "
                    "= step + device argmax + embedding lookup" if ws == 1 else
                    "r4q.tp.TPDecoder.loop: one CUDA-graph launch per token per rank (NVLink P2P "
                    "exchanges fused into the GEMVs) + device argmax + embedding lookup"),
            "results": res, "prefill": pre}


def prefill_tok_s(a, dev, m, cfg):
    """Prompt processing (pp) of `prefill_tokens` tokens through
    int4_hip.prefill_logits (tcgen05 GEMM for every projection, logits for
    every position as the reference returns), timed with CUDA events."""
    import torch
    from r4q import prefill
    M = a.prefill_tokens
    gen = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, cfg['vocab'], (M,), generator=gen, device=dev)

    def run():
        x = m['embed'][ids]
        return prefill.prefill_logits(x, m['qkv_w'], m['qkv_s'], m['o_w'], m['o_s'], m['gu_w'], m['gu_s'],
                                      m['down_w'], m['down_s'], m['in_norm_w'], m['post_norm_w'], m['q_norm_w'],
                                      m['k_norm_w'], m['rope_cos'], m['rope_sin'], cfg['num_heads'],
                                      cfg['num_kv_heads'], cfg['head_dim'], cfg['hidden'], cfg['intermediate'],
                                      cfg['rms_eps'], m['final_norm_w'], m['lm_w'], m['lm_s'], cfg['vocab'])
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    L, D, I, H, Hk, hd = (cfg['num_layers'], cfg['hidden'], cfg['intermediate'], cfg['num_heads'],
                          cfg['num_kv_heads'], cfg['head_dim'])
    flops = 2 * M * (L * (D * (H + 2 * Hk) * hd + H * hd * D + D * 2 * I + I * D) + D * cfg['vocab'])
    return {"tokens": M, "ms": round(ms, 3), "tok_s": round(M * 1e3 / ms, 1),
            "gemm_TFLOPs": round(flops / ms / 1e9, 1),
            "api": "int4_hip.prefill_logits (r4q.prefill): tcgen05 GEMM per projection, torch SDPA attention"}


def moe_tok_s(a, dev, peak, ws=1, rank=0):
    """benchmark config 4: 48-layer Qwen3-30B-A3B-shaped MoE decode (random
    init, INT4 experts, top-8 of 128), KV cache of ctx 2048 filled with seeded
    FP8 values, batches from --moe-batches; each token one CUDA-graph replay
    of the whole step (routing on the device).  ws > 1: expert parallelism,
    E / ws experts per rank, attention and router replicated, fp32 expert
    partials all-reduced over NVLink; time = max over ranks.  Bytes per step
    and GPU count the dense weights, the router, the lm_head, the KV read and
    this GPU's share of the distinct experts the step's routing selects
    (expected count for uniform routing: E (1 - (1 - k/E)^B) per layer)."""
    import torch
    import torch.distributed as dist
    from r4q import moe, synth, tp
    cfg = moe.qwen3_30b_a3b_config()
    bs = [int(b) for b in a.moe_batches.split(",") if b]
    ctx, steps = 2048, a.moe_tokens
    m = moe.build_moe_model(cfg, dev, seed=11, max_seq=ctx + steps + 16, batch=max(bs))
    synth.fill_kv_synthetic(m, ctx, seed=5)
    E, k, D = cfg['experts'], cfg['topk'], cfg['hidden']
    comm = tp.Comm(rank, ws, max_batch=max(bs), hidden=D, sa_cap=max(bs) * D) if ws > 1 else None
    res = []
    for B in bs:
        dec = moe.MoEDecoder(m, cfg, batch=B, comm=comm)
        h = m['embed'][torch.arange(B, device=dev) * 31 + 1]
        for w in range(3):
            dec.step(h, ctx + w)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for t in range(steps):
            dec.step(h, ctx + t)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        if ws > 1:
            comm.status()
            tm = torch.tensor([ms], device=dev)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ms = float(tm.item())
        distinct = E * (1 - (1 - k / E) ** B)
        byt = int(m['dense_weight_bytes'] + cfg['num_layers'] * (E * D * 2 + moe.expert_bytes(cfg, 1) * distinct / ws)
                  + 2 * cfg['vocab'] * D + cfg['num_layers'] * 2 * B * cfg['num_kv_heads'] * 128 * (ctx + steps // 2))
        res.append({"batch": B, "tok_s": round(B * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                    "bytes_per_step_per_gpu": byt, "GBps_per_gpu": round(byt / ms / 1e6, 1),
                    "frac": round(byt / ms / 1e6 / peak, 4)})
        del dec
    if comm is not None:
        comm.close()
    return {"model": "Qwen3-30B-A3B shape (48 layers, 128 experts, top-8), random init, INT4 experts",
            "ctx": ctx, "tokens": steps, "gpus": ws,
            "parallelism": f"expert parallel x{ws} (all-reduce of fp32 expert partials)" if ws > 1 else "1 GPU",
            "results": res,
            "api": "r4q.moe.MoEDecoder.step (one CUDA graph per step: router, top-k, grouped expert GEMVs)"}


def moe_probe(a):
    """Config-4 layer shapes (hidden 2048, 128 experts, top-8) with 2 layers,
    KV at ctx 2048, batch --moe-probe: 3 eager steps (each layer's kernels
    launch separately), for an ncu launch list / capture on a small case."""
    import torch
    from r4q import moe, synth
    dev = torch.device("cuda", 0)
    cfg = moe.qwen3_30b_a3b_config(layers=2)
    B = a.moe_probe
    m = moe.build_moe_model(cfg, dev, seed=11, max_seq=2048 + 16, batch=B)
    synth.fill_kv_synthetic(m, 2048, seed=5)
    dec = moe.MoEDecoder(m, cfg, batch=B)
    h = m['embed'][torch.arange(B, device=dev) * 31 + 1]
    for t in range(3):
        dec.step(h, 2048 + t, use_graph=False)
    torch.cuda.synchronize()
    print(f"moe probe B={B} ok")


def kernel_probe(a):
    import torch
    from r4q import lib as Lb, ops, synth
    dev = torch.device("cuda", 0)
    name, N, K, pro = next(t for t in LAYER_SHAPES if t[0] == a.kernel_probe)
    g = torch.Generator(device=dev).manual_seed(0)
    _, w, sc = synth.linear_int4(N, K, g, dev)
    kin = 2 * K if pro == "silu_fwht" else K
    x = torch.randn(a.batch, kin, device=dev, generator=g).half()
    prol = Lb.PRO_SILU_FWHT if pro == "silu_fwht" else Lb.PRO_FWHT
    for _ in range(4):
        ops.gemv("int4", x, w, sc, N, K, prologue=prol)
    torch.cuda.synchronize()
    print(f"probe {name} N={N} K={K} B={a.batch} ok")


def decode_probe(a):
    import torch
    import int4_hip
    from r4q import synth
    dev = torch.device("cuda", 0)
    int4_hip.USE_GRAPH = False
    cfg = synth.qwen3_14b_config()
    m = synth.build_decode_model(cfg, dev, seed=3, max_seq=2304)
    synth.fill_kv_synthetic(m, 2048, seed=1)
    tok = torch.zeros(1, dtype=torch.long, device=dev)
    for t in range(3):
        h = m['embed'][tok].reshape(1, 1, -1)
        lg = int4_hip.decode_step_logits(
            h, m['qkv_w'], m['qkv_s'], 0, m['o_w'], m['o_s'], 0, m['gu_w'], m['gu_s'], 0,
            m['down_w'], m['down_s'], 0, m['in_norm_w'], m['post_norm_w'], m['q_norm_w'],
            m['k_norm_w'], m['rope_cos'], m['rope_sin'], 2048 + t, cfg['num_heads'],
            cfg['num_kv_heads'], cfg['head_dim'], cfg['hidden'], cfg['intermediate'],
            cfg['rms_eps'], m['k_caches'], m['v_caches'], m['final_norm_w'], m['lm_w'], m['lm_s'],
            cfg['vocab'], cfg['hidden'], None)
        tok = lg.reshape(-1).argmax().reshape(1)
    torch.cuda.synchronize()
    print("decode probe ok")


def gemm_probe(a):
    """Four INT4 prefill GEMMs, M = 512, qkv shape (7168 x 5120), for ncu."""
    import torch
    from r4q import ops, synth
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    _, w, sc = synth.linear_int4(QKV_N, HID, g, dev)
    x = torch.randn(512, HID, device=dev, generator=g).half()
    for _ in range(4):
        ops.gemm(x, w, sc, QKV_N)
    torch.cuda.synchronize()
    print("gemm probe ok")


if __name__ == "__main__":
    args = parse()
    if args.gemm_probe:
        gemm_probe(args)
    elif args.decode_probe:
        decode_probe(args)
    elif args.kernel_probe:
        kernel_probe(args)
    elif args.moe_probe:
        moe_probe(args)
    elif args.impl == "reference":
        main_reference(args)
    else:
        main_ours(args)
