"""Benchmark of the quantised MoE expert FFN on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the routed-expert FFN of a
Qwen3-30B-A3B-shaped MoE layer at batch 1 - 128 experts, top-8 softmax
routing, gate/up [768 x 2048] Q4_K, down [2048 x 768] Q6_K, x ~ N(0,1) f32
quantised to Q8_K on the device, router logits ~ N(0,1). All experts of 48
such layers (18.8 GB) are resident in HBM; one step is one token through the
48 layers' expert FFNs (48 independent layer-tokens), so each step walks
1.17 GB of selected expert weights and nothing is reused from the 126 MB L2.

Metric: expert weight bytes per second (24,477,696 algorithmic bytes per
layer-token), the reference's own matvec unit. `value` runs with inputs
resident in HBM; `e2e` runs the same steps through the public C ABI call
(tlmg_expert_ffn_many) with pinned host buffers, host<->device copies inside
the timed region. The reference arm (--impl reference) times the
reference's own AVX-512 kernels through its worker pool on the host cores.

Under torchrun each rank runs an independent replica on its own GPU (the
bs=1 path does not shard: no collective on the data path); value is the sum
over ranks divided by the slowest rank's time.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D, DE, E, K = 2048, 768, 128, 8
DT_GATE, DT_DOWN = 12, 14                       # Q4_K gate/up, Q6_K down
BYTES_LAYER_TOKEN = K * (2 * DE * (D // 256 * 144) + D * (DE // 256 * 210))   # 24,477,696
METRIC = "expert GEMV HBM GB/s, bs=1 MoE expert FFN (Qwen3-30B-A3B layer shape, Q4_K gate/up + Q6_K down)"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per layer-token of the persistent kernel, from
# ncu (dram__bytes_read.sum + dram__bytes_write.sum) over three consecutive
# 4-layer-token launches of the kernel as last changed in commit b5603b9
# (captured at a95d757): reads 98,118,912 / 98,110,976 / 98,109,184 B,
# writes 3,106,560 / 484,864 / 455,424 B (the share of the written rows that
# leaves L2 within the launch varies); the mean of the three, per layer-token.
TRAFFIC_LAYER_TOKEN = ((98_118_912 + 98_110_976 + 98_109_184) + (3_106_560 + 484_864 + 455_424)) // (3 * 4)


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, earlier measurement on this pool)"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
def cpu_reference_run(seconds: float, layers_host: int = 2, threads: int = 0, steps: int | None = None,
                      warmup: int = 0, step_layers: int = 48):
    """Time the reference's CPU path on the host cores: its own kernels
    (tlm_quantize_act / tlm_matvec_rows, AVX-512 tier) orchestrated like
    run_batch() through its worker pool, all threads, rotating over
    layers_host x 128 host-resident experts (>> L3). Returns a dict."""
    import oracle
    from tierlm_b200 import synth
    R = oracle.ref()
    kind = "reference"
    if R is None:
        raise RuntimeError("oracle/_ref/libtlmref.so is not built (make -C oracle ref)")
    R.tlmref_open(threads)
    nthreads = R.tlmref_threads()
    rng = np.random.default_rng(1234)
    layers = [[synth.rand_expert(rng, D, DE, (DT_GATE, DT_GATE, DT_DOWN)) for _ in range(E)]
              for _ in range(layers_host)]
    dt = (C.c_int * 3)(DT_GATE, DT_GATE, DT_DOWN)
    ffn = np.zeros(D, np.float32)
    inputs = [(rng.standard_normal(D).astype(np.float32), rng.standard_normal(E).astype(np.float32))
              for _ in range(64)]

    def one(i):
        x, lg = inputs[i % len(inputs)]
        ids, w = oracle.route(0, lg, K)     # routing: negligible next to the matvecs
        experts = layers[i % layers_host]
        g = (C.c_void_p * K)(*[experts[e][0].ctypes.data + experts[e][1][0] for e in ids])
        u = (C.c_void_p * K)(*[experts[e][0].ctypes.data + experts[e][1][1] for e in ids])
        d = (C.c_void_p * K)(*[experts[e][0].ctypes.data + experts[e][1][2] for e in ids])
        R.tlmref_expert_ffn(D, DE, K, dt, g, u, d, x.ctypes.data, w.ctypes.data, ffn.ctypes.data)

    for i in range(8):
        one(i)
    if steps is None:
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            one(n)
            n += 1
        el = time.perf_counter() - t0
        units = n
        sample = f"{n} layer-tokens over {el:.1f} s, rotating {layers_host} host layers x {E} experts"
    else:
        for i in range(warmup * step_layers):
            one(i)
        t0 = time.perf_counter()
        for i in range(steps * step_layers):
            one(i)
        el = time.perf_counter() - t0
        units = steps * step_layers
        sample = (f"{steps} steps x {step_layers} layer-tokens, rotating {layers_host} host layers x {E} "
                  f"experts ({layers_host * E * 3.06:.0f} MB > L3)")
    gbs = units * BYTES_LAYER_TOKEN / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": nthreads, "kind": kind,
            "tier": R.tlmref_tier().decode(), "cpu": R.tlmref_cpu_model().decode().strip(),
            "sample": sample, "seconds": el, "units": units}


def run_reference_arm(args, rank: int) -> None:
    if rank != 0:
        return
    r = cpu_reference_run(0, layers_host=2, steps=args.steps, warmup=args.warmup)
    ms = r["seconds"] * 1e3 / args.steps
    line = {"metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/int32+f32", "data": "synthetic", "impl": "reference",
            "config": config_dict(args),
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "tier", "cpu")},
            "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(args) -> dict:
    return {"workload": "BASELINE config 2: isolated expert FFN (GEMV+SwiGLU+combine), Qwen3-30B-A3B layer "
                        "shape, bs=1; one step = one token through 48 layers' expert FFNs",
            "layers": args.layers, "n_experts": E, "top_k": K, "d_model": D, "d_expert": DE, "batch": 1,
            "weights": "gate/up Q4_K, down Q6_K (random codes, finite random f16 scales)",
            "inputs": "x ~ N(0,1) f32 -> Q8_K on device; router logits ~ N(0,1), softmax top-8 renorm",
            "l2": f"inputs larger than L2: {args.layers} layers x {E} experts resident "
                  f"({args.layers * E * 3.06e-3:.1f} GB) walked once per step",
            "parallelism": f"replicas x{args.gpus} (bs=1 does not shard)"}


# ---------------------------------------------------------------------------
def build_context(args, dev, seed: int):
    import torch

    from tierlm_b200 import synth
    from tierlm_b200.moe import MoeContext
    ctx = MoeContext(args.layers, D, DE, E, K, router=0, device=dev.index)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    rb_g, rb_d = D // 256 * 144, DE // 256 * 210
    og, ou, od = 0, DE * rb_g, 2 * DE * rb_g
    per = 2 * DE * rb_g + D * rb_d
    for layer in range(args.layers):
        gu = synth.device_rows(DT_GATE, E * 2 * DE, D, gen, dev).view(E, 2 * DE * rb_g)
        dn = synth.device_rows(DT_DOWN, E * D, DE, gen, dev).view(E, D * rb_d)
        buf = torch.cat([gu, dn], dim=1).contiguous()          # [E, per]: gate | up | down
        for e in range(E):
            p = buf[e]
            ctx._lib.tlmg_set_expert(ctx._h, layer, e, (C.c_int32 * 3)(DT_GATE, DT_GATE, DT_DOWN),
                                     C.c_void_p(p.data_ptr()), per, (C.c_uint64 * 3)(og, ou, od))
        del gu, dn, buf
    torch.cuda.synchronize(dev)
    return ctx


def slot_cache_section(args, dev, rank: int, world: int, stream, timed) -> dict:
    """The reference's expert store on the GPU (BASELINE config 5 expert
    size: D 4096, d_expert 1536, Q4_K gate/up/down, 10.6 MB per expert, 128
    experts top-8): every expert of CL layers registered in pinned host
    memory, cache_frac of them fit in HBM slots, and each step is one token
    through the CL layers' whole moe() blocks (tlmg_moe_layer on a device h).
    Arms: demand loads only, and the router lookahead (tlmg_cache_lookahead:
    next layer's RMSNorm + router on the current residual, its top-k
    prefetched while this layer computes). Random inputs: no temporal
    locality beyond what the lookahead predicts."""
    import torch

    from tierlm_b200 import synth
    from tierlm_b200.moe import MoeContext
    D5, DE5, CL = 4096, 1536, args.cache_layers
    rb_g, rb_d = D5 // 256 * 144, DE5 // 256 * 144
    per = 2 * DE5 * rb_g + D5 * rb_d                        # 10,616,832 bytes per expert
    cctx = MoeContext(CL, D5, DE5, E, K, router=0, device=dev.index)
    cctx.set_stream(stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242 + rank)
    n_slots = max(K + 1, int(args.cache_frac * CL * E))
    cctx.cache_enable(n_slots, per + 3 * 512)
    rng = np.random.default_rng(99 + rank)
    host = []
    for layer in range(CL):
        gu = synth.device_rows(DT_GATE, E * 2 * DE5, D5, gen, dev).view(E, 2 * DE5 * rb_g)
        dn = synth.device_rows(DT_GATE, E * D5, DE5, gen, dev).view(E, D5 * rb_d)
        hb = torch.cat([gu, dn], dim=1).cpu().pin_memory()            # [E, per]: gate | up | down
        del gu, dn
        host.append(hb)
        for e in range(E):
            cctx.set_expert_host(layer, e, (DT_GATE, DT_GATE, DT_GATE), hb[e], (0, DE5 * rb_g, 2 * DE5 * rb_g))
        cctx.set_layer(layer, (1.0 + 0.1 * rng.standard_normal(D5)).astype(np.float32), 0,
                       (rng.standard_normal((E, D5)) / np.sqrt(D5)).astype(np.float32), 4 * D5)
    NR = args.warmup + args.steps                           # every token of both arms distinct
    hs = torch.randn((2 * NR, D5), generator=gen, device=dev)
    h = torch.empty(D5, device=dev)
    base = [0]

    def cstep(s):
        h.copy_(hs[base[0] + s % NR])
        for layer in range(CL):
            cctx.moe_layer(layer, h)
        cctx.cache_tick()                                  # one model step (frequency decay clock)

    res = {}
    for arm, (name, depth) in enumerate((("demand", 0), ("lookahead", 1))):
        base[0] = arm * NR
        cctx.cache_lookahead(depth, K)
        for s in range(args.warmup):
            cstep(s)
        st0 = cctx.cache_stats()
        cms = timed(cstep, args.steps)
        st1 = cctx.cache_stats()
        d = {k2: st1[k2] - st0[k2] for k2 in st1}
        res[name] = {"tokens_per_s": round(world * args.steps / (cms * 1e-3), 2),
                     "ms_per_token": round(cms / args.steps, 3),
                     "hit_rate": round(d["hits"] / max(1, d["hits"] + d["misses"]), 3),
                     "prefetch_issued": d["prefetched"], "prefetch_used": d["prefetch_hits"],
                     "h2d_GBps": round(d["bytes"] / (cms * 1e-3) / 1e9, 1)}
    cctx.close()
    del host
    return {"config": "BASELINE config 5 expert size: D 4096, d_expert 1536, Q4_K gate/up/down "
                      f"({per:,} bytes per expert), 128 experts top-8, {CL} layers",
            "slots": n_slots, "cold_fraction": round(1 - n_slots / (CL * E), 3),
            "policy": "the reference store's (LFU with decay, hint rules, demand reserve)",
            "workload": "bs=1 decode, whole moe() per layer on a device residual, random inputs", **res}


def decode_step_section(ctx, args, dev, g, peak: float) -> dict:
    """BASELINE config 3 through tlmg_decode_step: Qwen3-30B-A3B shape
    (48 layers, D 2048, 32 q / 4 KV heads x 128 with qk-norm, 128 experts
    top-8, de 768, vocab 151,936), attention and down Q6_K, gate/up and
    embedding Q4_K, router f32, lm_head Q6_K, random weights; bf16 KV pages
    and split attention. A random prompt is stepped position by position
    (no lm_head, as the reference's prefill), then greedy decode: each token
    is the argmax of the previous step's logits, read by the host."""
    import torch

    from tierlm_b200 import synth
    H, KVH, HD, V = 32, 4, 128, 151936
    DT_ATT, DT_EMB, DT_HEAD, BF16, SPLIT = 14, 12, 14, 2, 1
    L, P, NG = args.layers, args.step_prompt, args.step_gen
    rng = np.random.default_rng(77)
    inv = np.array([np.float32(1e6 ** (-2.0 * j / HD)) for j in range(HD // 2)], np.float32)
    ctx.step_open(H, KVH, HD, V, inv, 1.0, max_ctx=P + NG, kv_dtype=BF16, attn_mode=SPLIT)
    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    for layer in range(L):
        ctx.set_layer(layer, norm(D), 0, (0.02 * rng.standard_normal((E, D))).astype(np.float32), 4 * D)
        mats = [synth.device_rows(DT_ATT, r, c, g, dev) for r, c in ((H * HD, D), (KVH * HD, D), (KVH * HD, D),
                                                                     (D, H * HD))]
        ctx.set_attention(layer, norm(D), (DT_ATT,) * 4, *mats, q_norm=norm(HD), k_norm=norm(HD))
        del mats
    emb = synth.device_rows(DT_EMB, V, D, g, dev)
    ctx.set_embedding(DT_EMB, emb)
    del emb
    head = synth.device_rows(DT_HEAD, V, D, g, dev)
    ctx.set_output(norm(D), DT_HEAD, head)
    del head
    torch.cuda.synchronize(dev)
    prompt = [int(t) for t in rng.integers(0, V, P)]
    logits = torch.empty(V, device=dev)
    st = torch.cuda.current_stream(dev)

    def run(n_warm=0):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(st)
        for pos, tok in enumerate(prompt):
            ctx.decode_step(tok, pos, logits if pos == P - 1 else None)
        ev[1].record(st)
        toks = []
        tok = int(torch.argmax(logits))
        h0 = time.perf_counter()
        for i in range(NG):
            ctx.decode_step(tok, P + i, logits)
            tok = int(torch.argmax(logits))            # the host needs the token for the next step
            toks.append(tok)
        wall = time.perf_counter() - h0
        ev[2].record(st)
        torch.cuda.synchronize(dev)
        return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), wall, toks

    run()                                                   # warm-up pass (same positions)
    n0 = ctx.launches
    i0 = ctx.step_info()
    pre_ms, dec_ms, wall, toks = run()
    launches = ctx.launches - n0
    i1 = ctx.step_info()
    # algorithmic bytes per decode token: weights read once + the KV rows read
    rb = lambda dt, n: n // 256 * {12: 144, 14: 210}[dt]   # noqa: E731
    attn_w = (H * HD + 2 * KVH * HD) * rb(DT_ATT, D) + D * rb(DT_ATT, H * HD)
    per_layer = attn_w + E * D * 4 + BYTES_LAYER_TOKEN + 4 * (2 * D + 2 * HD)
    T_mean = P + (NG + 1) / 2
    kv = 2 * KVH * HD * 2 * T_mean
    bytes_tok = L * (per_layer + kv) + V * rb(DT_HEAD, D) + rb(DT_EMB, D) + 4 * D
    tps = NG / (dec_ms * 1e-3)
    return {"metric": "decode tok/s, bs=1, whole step (BASELINE config 3)",
            "tokens_per_s": round(tps, 1), "ms_per_token": round(dec_ms / NG, 3),
            "prefill_tokens_per_s": round(P / (pre_ms * 1e-3), 1),
            "host_wall_tokens_per_s": round(NG / wall, 1),
            "bytes_per_token": int(bytes_tok), "GBps": round(bytes_tok * tps / 1e9, 1),
            "roofline_tokens_per_s": round(peak * 1e9 / bytes_tok, 1),
            "frac": round(bytes_tok * tps / 1e9 / peak, 4),
            "gpu_launches_per_token": round(launches / (P + NG), 1),
            "graph_replays": i1["replays"] - i0["replays"], "graphs_off": i1["graphs_off"],
            "prompt": P, "generated": NG, "kv": "bf16 pages, split attention", "distinct_tokens": len(set(toks)),
            "api": "tlmg_decode_step per position; greedy token read by the host each step",
            "weights": "random: attention/down/lm_head Q6_K, gate/up/embedding Q4_K, router f32"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=64, help="batched-decode section: tokens per layer call (<= 1: off)")
    ap.add_argument("--prefill", type=int, default=2048, help="prefill section: prompt tokens per layer call (0: off)")
    ap.add_argument("--ep-exchange", choices=["peer", "nccl"], default="peer",
                    help="batched-decode section at N > 1: expert-parallel exchange over peer memory or NCCL")
    ap.add_argument("--step-prompt", type=int, default=512,
                    help="decode-step section (config 3): prompt positions before the timed decode (0: off)")
    ap.add_argument("--step-gen", type=int, default=256, help="decode-step section: greedy tokens timed")
    ap.add_argument("--cache-layers", type=int, default=0, help="slot-cache section: layers (0: off)")
    ap.add_argument("--cache-frac", type=float, default=0.5, help="slot-cache section: HBM slots / experts")
    ap.add_argument("--attn-ctx", default="",
                    help="decode-attention section: context lengths, comma-separated, e.g. 768,4096,32768 "
                         "(empty: off)")
    args = ap.parse_args()
    assert args.warmup >= 3 or args.impl == "reference" or os.environ.get("TLMG_BENCH_ALLOW_SHORT"), \
        "use at least 3 warm-up steps"
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    args.gpus = max(args.gpus, world)

    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from tierlm_b200 import _lib
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _lib.check(_lib.load().tlmg_init(local))

    ctx = build_context(args, dev, seed=1000 + rank)
    stream = torch.cuda.current_stream(dev)
    ctx.set_stream(stream)
    L = args.layers
    P = 8                                              # distinct token input sets, rotated
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    xs = torch.randn((P, L, D), generator=g, device=dev)
    lgs = torch.randn((P, L, E), generator=g, device=dev)
    out = torch.empty((P, L, D), device=dev)

    def step(s):
        i = s % P
        ctx.expert_ffn_many(0, xs[i], lgs[i], out[i])

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, n):
        torch.cuda.synchronize(dev)
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for s in range(n):
            fn(s)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ms = t0.elapsed_time(t1)
        if world > 1:
            tm = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ms = float(tm.item())
        return ms

    # ---- value: inputs resident in HBM
    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = ctx.launches
    ms = timed(step, args.steps)
    launches = ctx.launches - launches0
    clk = clocks.stop()
    bytes_step = L * BYTES_LAYER_TOKEN
    value = world * args.steps * bytes_step / (ms * 1e-3) / 1e9

    # ---- roofline of the dominant kernel: per-launch CUDA events, second pass
    kern = ctx.kernel_times(lambda: [step(s) for s in range(args.steps)])
    peak, peak_src = peaks()

    # ---- e2e: the same steps through the C ABI with pinned host buffers
    hx = xs.cpu().pin_memory()
    hl = lgs.cpu().pin_memory()
    ho = torch.empty((P, L, D)).pin_memory()

    def step_host(s):
        i = s % P
        ctx.expert_ffn_many(0, hx[i], hl[i], ho[i])

    for s in range(args.warmup):
        step_host(s)
    ms_e2e = timed(step_host, args.steps)
    e2e = world * args.steps * bytes_step / (ms_e2e * 1e-3) / 1e9
    h2d = L * (D + E) * 4
    d2h = L * D * 4

    # ---- batched decode (bs = BATCH tokens per GPU through each layer, one call per layer);
    # at N > 1 expert-parallel: each GPU owns E / N experts of every layer and exchanges
    # the (token, expert) records with NCCL all-to-all
    batch = None
    if args.batch > 1:
        B = args.batch
        bx = torch.randn((2, L, B, D), generator=g, device=dev)
        bl = torch.randn((2, L, B, E), generator=g, device=dev)
        bo = torch.empty((2, L, B, D), device=dev)
        # distinct experts each layer call reads (softmax top-k = the k largest logits),
        # over the tokens of every GPU
        sel = torch.topk(bl, K, dim=-1).indices                               # [2, L, B, K]
        hit = torch.zeros((2, L, E), dtype=torch.bool, device=dev)
        hit.scatter_(2, sel.reshape(2, L, B * K), True)
        if world > 1:
            hits = hit.to(torch.uint8)
            dist.all_reduce(hits, op=dist.ReduceOp.MAX)
            hit = hits.bool()
        uniq = hit.sum(-1).double()                                            # [2, L]
        bytes_expert = BYTES_LAYER_TOKEN // K
        ep = None
        if world > 1:
            from tierlm_b200.ep import ExpertParallel, PeerExpertParallel
            ep = (PeerExpertParallel(ctx, D, E, K, B, device=dev) if args.ep_exchange == "peer"
                  else ExpertParallel(ctx, D, E, K, device=dev))

        def layer_call(layer, xi, li, oi):
            if ep is None:
                ctx.expert_ffn_batch(layer, xi, li, oi)
            else:   # device errors of layer l surface in the call of l + 1, the step's last is checked
                ep.ffn_batch(layer, xi, li, oi, check=layer == L - 1)

        def bstep(s):
            i = s % 2
            for layer in range(L):
                layer_call(layer, bx[i, layer], bl[i, layer], bo[i, layer])

        for s in range(args.warmup):
            bstep(s)
        torch.cuda.synchronize(dev)
        n0 = ctx.launches
        bms = timed(bstep, args.steps)
        blaunch = ctx.launches - n0
        ubytes = sum(float(uniq[s % 2].sum()) for s in range(args.steps)) * bytes_expert
        hbx, hbl = bx.cpu().pin_memory(), bl.cpu().pin_memory()
        hbo = torch.empty((2, L, B, D)).pin_memory()
        dx_, dl_, do_ = torch.empty((B, D), device=dev), torch.empty((B, E), device=dev), torch.empty((B, D), device=dev)

        def bstep_host(s):
            i = s % 2
            for layer in range(L):
                if ep is None:
                    ctx.expert_ffn_batch(layer, hbx[i, layer], hbl[i, layer], hbo[i, layer])
                else:   # the exchange needs device buffers: the copies are part of the step
                    dx_.copy_(hbx[i, layer], non_blocking=True)
                    dl_.copy_(hbl[i, layer], non_blocking=True)
                    ep.ffn_batch(layer, dx_, dl_, do_, check=layer == L - 1)
                    hbo[i, layer].copy_(do_, non_blocking=True)

        for s in range(args.warmup):
            bstep_host(s)
        bms_e2e = timed(bstep_host, args.steps)
        if hasattr(ep, "close"):
            torch.cuda.synchronize(dev)
            dist.barrier()   # every rank's layer calls are done before any exchange buffer is unmapped
            ep.close()
        exch = ("peer-memory exchange, device barriers" if args.ep_exchange == "peer"
                else "NCCL all-to-all")
        batch = {"batch": B, "metric": f"decode tok/s, bs={B} per GPU, expert FFN of {L} layers per token",
                 "tokens_per_s": round(world * args.steps * B / (bms * 1e-3), 1),
                 "ms_per_step": bms / args.steps,
                 "unique_expert_GBps": round(ubytes / (bms * 1e-3) / 1e9, 1),
                 "unique_experts_per_layer": round(float(uniq.mean()), 2),
                 "gpu_launches": blaunch,
                 "kernels": "tcgen05.mma kind::i8 gate/up and down (one TMEM accumulator per sub-block)",
                 "parallelism": "single GPU" if world == 1 else f"expert-parallel x{world} ({exch})",
                 "e2e": {"tokens_per_s": round(world * args.steps * B / (bms_e2e * 1e-3), 1),
                         "h2d_bytes_per_step": L * B * (D + E) * 4, "d2h_bytes_per_step": L * B * D * 4,
                         "api": "tlmg_expert_ffn_batch (pinned host buffers)" if world == 1 else
                                f"{type(ep).__name__}.ffn_batch with pinned host copies in the step"},
                 "note": "one call per layer serves all B tokens; each selected expert is read once per call"}

    # ---- prefill: PREFILL tokens of one GPU's prompt through each layer's experts, one call per layer
    prefill = None
    if args.prefill > 0 and world == 1:
        T = args.prefill
        px = torch.randn((L, T, D), generator=g, device=dev)
        pl = torch.randn((L, T, E), generator=g, device=dev)
        po = torch.empty((L, T, D), device=dev)

        def pstep(s):
            for layer in range(L):
                ctx.expert_ffn_batch(layer, px[layer], pl[layer], po[layer])

        for s in range(args.warmup):
            pstep(s)
        psteps = max(1, min(args.steps, 5))
        pms = timed(pstep, psteps)
        pbytes = L * E * (BYTES_LAYER_TOKEN // K)           # every expert is selected at 2048 tokens
        flops = 2.0 * T * K * (2 * DE * D + D * DE) * L      # int8 MACs x 2 per step
        prefill = {"tokens": T, "metric": f"prefill tok/s, {T}-token prompt, expert FFN of {L} layers",
                   "tokens_per_s": round(world * psteps * T / (pms * 1e-3), 1),
                   "ms_per_step": pms / psteps, "steps": psteps,
                   "int8_tops": round(world * psteps * flops / (pms * 1e-3) / 1e12, 2),
                   "weight_GBps": round(world * psteps * pbytes / (pms * 1e-3) / 1e9, 1),
                   "note": "tlmg_expert_ffn_batch with all prompt tokens of a layer in one call (tensor-core kernels)"}

    # ---- HBM slot cache (BASELINE config 5 expert size): cold experts in pinned host memory, bs=1
    # decode through CL layers whose 128 experts share cache_frac x (CL x 128) HBM slots
    cache = None
    if args.cache_layers > 0:
        cache = slot_cache_section(args, dev, rank, world, stream, timed)

    # ---- decode attention over a paged KV cache (config-3 attention shape: 32 query heads,
    # 4 KV heads, head_dim 128, 64-position pages), one layer per call, replicated per GPU
    attn = None
    ctxs = [int(v) for v in str(args.attn_ctx).split(",") if v.strip()]
    if ctxs:
        from tierlm_b200 import attention as A
        AH, AKV, AHD, APG = 32, 4, 128, 64
        astream = torch.cuda.Stream(dev)   # graphs are captured on a side stream
        astream.wait_stream(stream)
        attn = {"heads": AH, "kv_heads": AKV, "head_dim": AHD, "page": APG, "contexts": {},
                "timing": "CUDA graph of R calls over R distinct KV pools (working set > L2), CUDA events",
                "kv_bytes": "2 x T x kv_heads x head_dim x element size per call (K and V read once)"}
        for T in ctxs:
            row = {}
            for name, dtype, mode in (("split_bf16", torch.bfloat16, A.SPLIT), ("split_f32", torch.float32, A.SPLIT),
                                      ("exact_f32", torch.float32, A.EXACT)):
                if mode == A.EXACT and T > 4096:
                    continue
                n_pages = -(-T // APG)
                esz = torch.tensor([], dtype=dtype).element_size()
                pool_b = 2 * n_pages * AKV * APG * AHD * esz
                R = int(min(256, max(1, -(-400_000_000 // pool_b))))
                pools = [(torch.randn((n_pages, AKV, APG, AHD), generator=g, device=dev).to(dtype),
                          torch.randn((n_pages, AKV, APG, AHD), generator=g, device=dev).to(dtype)) for _ in range(R)]
                table = torch.randperm(n_pages, device=dev).to(torch.int32)
                aq = torch.randn((AH, AHD), generator=g, device=dev)
                holder = A.PagedKV.__new__(A.PagedKV)
                holder._work = torch.empty(A.work_bytes(mode, dtype, T, AH, AKV, AHD), dtype=torch.uint8, device=dev)
                aout = torch.empty((AH, AHD), device=dev)
                with torch.cuda.stream(astream):
                    for kp_, vp_ in pools:
                        A.decode_attention(aq, kp_, vp_, table, T, mode, out=aout, work=holder)
                    astream.synchronize()
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=astream):
                        for kp_, vp_ in pools:
                            A.decode_attention(aq, kp_, vp_, table, T, mode, out=aout, work=holder)
                    for _ in range(3):
                        graph.replay()
                    reps = 5
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(astream)
                    for _ in range(reps):
                        graph.replay()
                    e1.record(astream)
                    astream.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (reps * R)
                gbs = pool_b / (us * 1e-6) / 1e9
                row[name] = {"us_per_layer": round(us, 2), "kv_GBps": round(gbs, 1),
                             "hbm_frac": round(gbs / peak, 4), "pools": R}
                del graph, pools
            attn["contexts"][str(T)] = row

    # ---- the whole decoder step: embedding, 48 x (attention + MoE), lm_head
    dstep = None
    if args.step_prompt > 0 and world == 1:
        dstep = decode_step_section(ctx, args, dev, g, peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_reference_run(args.cpu_seconds)
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "tier", "cpu")}
        except Exception as ex:   # the baseline is reported, never required
            cpu = {"value": None, "unit": "GB/s", "cores": None, "kind": "reference", "sample": f"failed: {ex}"}

    if rank == 0:
        kname, kms, kn, kbytes = kern
        achieved = kbytes / (kms / kn * 1e-3) / 1e9 if kn else None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/int32+f32", "data": "synthetic", "config": config_dict(args),
            "tokens_per_s": round(world * args.steps / (ms * 1e-3), 2),
            "layer_tokens_per_s": round(world * args.steps * L / (ms * 1e-3), 1),
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e / args.steps, "api": "tlmg_expert_ffn_many (pinned host buffers)"},
            "roofline": {"bound": "hbm", "kernel": kname,
                         "achieved": None if achieved is None else round(achieved, 1),
                         "peak": peak, "unit": "GB/s",
                         "frac": None if achieved is None else round(achieved / peak, 4),
                         "traffic": None if not kbytes else int(kbytes // BYTES_LAYER_TOKEN * TRAFFIC_LAYER_TOKEN),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-layer-token "
                                           "launch, scaled by layer-tokens per launch",
                         "peak_source": peak_src,
                         "launches": kn, "avg_us": None if not kn else round(kms / kn * 1e3, 3),
                         "algorithmic_bytes_per_launch": kbytes,
                         "timing": "per-launch CUDA events on the launch stream, second pass of the same steps"},
            "cpu_baseline": cpu, "clocks": clk, "gpu_launches": launches,
            "prefill": prefill, "decode_step": dstep, "slot_cache": cache, "decode_attention": attn,
            # last key: the bs=64 (expert-parallel at N > 1) decode section
            "batched_decode": batch,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
