"""Benchmark: 12B-shaped Q4_0 batch-1 greedy decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One step = one decode token of the 48-layer 12B-shaped model (Q4_0 layers, Q8_0 LM head,
640-slot ring with every slot live) on synthetic weights.  Prints one JSON line.

value : tokens/s with the step's inputs resident in HBM (device-timed CUDA graph replays)
e2e   : tokens/s through the public C ABI sx_forward_token (gpuDispatchForwardToken) with
        host buffers: the per-token host->device copy of x / slot list / step params and the
        device->host read of the sampled token are inside the timed region
roofline : dominant kernel (fused gate+up GeGLU Q4 GEMV) bytes / CUDA-event launch time
cpu_baseline : the CPU checker (restatement of the reference's CPU path) on the host cores

N > 1: one process per GPU (torchrun), the model tensor-parallel over the ranks (column-
parallel q/k/v/gate/up, row-parallel o/down with an NCCL all-reduce of the hidden vector twice
per layer, vocabulary-parallel LM head with an all-gather of argmax candidates); value is the
one token stream's tokens/s (strong scaling), timed as the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "ai-research_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "12B-shape Q4_0 decode tok/s"
UNIT = "tok/s"
SEED = 1234 + 4
START_CLOCK = 50000


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sx", choices=["sx", "reference"])
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-lines", action="store_true",
                    help="skip the stand-alone config 1-3 kernel measurements")
    ap.add_argument("--graph", choices=["stream", "persistent", "fused", "block"],
                    default="fused",
                    help="stream: one launch per token with a producer warp per SM streaming "
                         "the weights through a shared-memory ring (one GPU); persistent: one "
                         "cooperative launch per token with grid barriers; fused: 5 kernels "
                         "per layer chained with programmatic dependent launch; block: the fused "
                         "graph with q|k|v, attention and o as one attention-block kernel (one "
                         "GPU)")
    ap.add_argument("--case", choices=["geglu", "q4_head", "attn", "prefill", "sessions", "c1",
                                       "c3"],
                    help="profiling case: launch one kernel of the step standalone "
                         "(--launches times) on synthetic data and exit; prints no JSON line")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--rows", type=int, default=15360,
                    help="--case geglu: gate/up rows (15360 / N is one tensor-parallel rank's)")
    ap.add_argument("--allreduce", choices=["peer", "nccl"], default="peer",
                    help="tensor parallel (N > 1): the one-shot peer all-reduce (NCCL when its "
                         "workspaces cannot be mapped) or NCCL")
    return ap.parse_args()


def c5_config(**kw):
    import sx

    # config 5: H 1536, 35 layers, 8 q / 1 kv heads x 256, I 6144, Q4_0 layers, Q8_0 head
    d = dict(hidden_size=1536, intermediate_size=6144, num_layers=35, num_q_heads=8,
             num_kv_heads=1, num_global_kv_heads=1, head_dim=256, global_head_dim=256,
             num_sessions=8)
    d.update(kw)
    return sx.model_config(**d)


def run_sessions(eng, args, rank=0, print_lines=True):
    import torch
    import sx

    cfg = c5_config()
    model = sx.Model(eng, cfg)
    model.synth_weights(SEED + 1)
    H, V = cfg.hidden_size, cfg.vocab_size
    rng = np.random.default_rng(SEED + 1)
    lens = rng.integers(16, 513, 64)[8 * rank: 8 * rank + 8]
    prompts = [np.stack([sx.synth_embed_row(H, int(t), SEED + 1)
                         for t in rng.integers(0, V, n)]) for n in lens]
    stream = torch.cuda.ExternalStream(eng.stream)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    rings = [sx.Ring(1, cfg.num_anchors, cfg.window_size, cfg.num_recall) for _ in lens]
    # warm-up prefill of the same prompts on scratch rings (allocates the prefill scratch for
    # all the call's tokens, so the timed call does no allocation), then the timed one
    model.prefill_batch(prompts, [sx.Ring(1, cfg.num_anchors, cfg.window_size, cfg.num_recall)
                                  for _ in lens], [0] * 8)
    eng.sync()
    plan = model.prefill_plan(prompts, rings, [0] * 8)  # host ring bookkeeping, untimed
    ev[0].record(stream)
    toks = model.prefill_run(plan)  # uploads, 35 layers of GEMMs + per-token kernels, LM head
    ev[1].record(stream)
    eng.sync()
    T = int(lens.sum())
    ms_p = ev[0].elapsed_time(ev[1])
    flops = T * cfg.num_layers * 2.0 * H * (cfg.num_q_heads * 256 + 2 * 256 + 8 * 256 + 3 * 6144)
    if print_lines:
        print(json.dumps({"case": "c5_prefill", "sessions": 8, "tokens": T, "ms": ms_p,
                          "tok_s": T / (ms_p / 1e3), "gemm_tflops": flops / (ms_p / 1e3) / 1e12}),
              flush=True)
    clocks = [int(n) for n in lens]
    tokens = [int(t) for t in toks]
    steps = 128

    def step():
        nonlocal clocks, tokens
        xs = np.stack([sx.synth_embed_row(H, tokens[s], SEED + 1) for s in range(8)])
        slots = [rings[s].activate_slot(0, clocks[s]) for s in range(8)]
        lists = [rings[s].get_active_slots(0, clocks[s]) for s in range(8)]
        got = model.decode_batch(xs, clocks, slots, lists, True)
        tokens = [int(t) for t in got]
        clocks = [c + 1 for c in clocks]

    for _ in range(3):
        step()
    eng.sync()
    ev[2].record(stream)
    for _ in range(steps - 3):
        step()
    ev[3].record(stream)
    eng.sync()
    ms_d = ev[2].elapsed_time(ev[3]) / (steps - 3)
    # device time of the same step: replays of the batched graph from its staged inputs
    reps = 50
    ev[2].record(stream)
    for _ in range(reps):
        model.launch_batch(8, True)
    ev[3].record(stream)
    eng.sync()
    ms_dev = ev[2].elapsed_time(ev[3]) / reps
    if print_lines:
        print(json.dumps({"case": "c5_decode_batch8", "sessions": 8, "steps": steps,
                          "e2e_ms_per_step": ms_d, "e2e_tok_s": 8 / (ms_d / 1e3),
                          "device_ms_per_step": ms_dev, "device_tok_s": 8 / (ms_dev / 1e3)}),
              flush=True)
    model.close()
    return {"prompt_tokens": T, "prefill_ms": ms_p, "decode_e2e_ms_per_step": ms_d,
            "decode_device_ms_per_step": ms_dev, "steps": steps}


def run_case(args):
    """Small standalone workloads for ncu captures of the step's kernels:
    geglu   -- the fused gate+up GeGLU GEMV of one 12B layer (2 x rows x 3840 Q4_0; rows 15360
               is 73.8 MB, one GPU; 15360 / N is a tensor-parallel rank's share)
    q4_head -- a 262144 x 3840 Q4_0 GEMV (629 MB), the steady-state streaming case
    c1      -- BASELINE config 1: the 6144 x 1536 Q4_0 GEMV
    c3      -- BASELINE config 3: the fused attention over 256 independent 640-slot rings
    attn    -- one 12B-width layer token (16 q / 8 kv heads x 256, 640 live slots), whose
               second kernel is the fused attention
    prefill -- the tcgen05 Q4_0 GEMM on config 5's projection shapes (TFLOP/s per shape)
    sessions -- config 5 on one GPU: this GPU's 8 of the 64 seeded prompts prefilled with
               sx_prefill_batch, then 128 greedy tokens x 8 sessions with sx_decode_batch
               (host buffers in and out, timed with CUDA events on the engine stream)"""
    import torch
    import sx

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    eng = sx.Engine(local)
    g = torch.Generator(device="cuda").manual_seed(SEED)

    def packed(m, k):
        n = sx.packed_bytes(m, k, sx.QUANT_Q4)
        return torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)

    if args.case == "prefill":
        # config-5 batch-prefill projections: ~16.9k packed tokens x (q|k|v, o, gate|up, down);
        # prints one JSON line per shape (TFLOP/s of the tcgen05 GEMM vs the measured peak)
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
            if (ROOT / "MEASURED_PEAKS.json").exists() else {"bf16_tflops": 1590.0}
        t = 66 * 256
        x = torch.randn((t, 6144), device="cuda", generator=g).to(torch.bfloat16)
        for n, k in ((2560, 1536), (1536, 2048), (12288, 1536), (1536, 6144)):
            w = packed(n, k)
            xs = x[:, :k].contiguous()
            y = torch.empty((t, n), device="cuda")
            for _ in range(2):
                eng.prefill_gemm(w, xs, y, t, n, k)
            eng.sync()
            stream = torch.cuda.ExternalStream(eng.stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.launches):
                eng.prefill_gemm(w, xs, y, t, n, k)
            e1.record(stream)
            eng.sync()
            ms = e0.elapsed_time(e1) / args.launches
            tflops = 2.0 * t * n * k / (ms / 1e3) / 1e12
            print(json.dumps({"case": "prefill_q4_gemm", "t": t, "n": n, "k": k, "ms": ms,
                              "tflops": tflops, "frac_of_measured_bf16": tflops / peaks["bf16_tflops"]}),
                  flush=True)
        eng.close()
        return
    if args.case == "sessions":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world == 1:
            run_sessions(eng, args)
        else:
            # BASELINE config 5 across the node: rank r prefills and decodes sessions
            # 8r .. 8r + 7 of the 64 seeded prompts on its own GPU (its own weight copy, no
            # collective on the data path); the process group only gathers the timings
            import torch.distributed as dist
            from datetime import timedelta

            rank = int(os.environ.get("RANK", "0"))
            dist.init_process_group("gloo", timeout=timedelta(seconds=300))
            r = run_sessions(eng, args, rank=rank, print_lines=False)
            allr = [None] * world
            dist.all_gather_object(allr, r)
            if rank == 0:
                T = sum(x["prompt_tokens"] for x in allr)
                pm = max(x["prefill_ms"] for x in allr)
                dm = max(x["decode_e2e_ms_per_step"] for x in allr)
                dd = max(x["decode_device_ms_per_step"] for x in allr)
                print(json.dumps({"case": "c5_sessions_multi_gpu", "n_gpus": world,
                                  "sessions": 8 * world, "prompt_tokens": T,
                                  "prefill_ms_max_over_ranks": pm,
                                  "prefill_tok_s": T / (pm / 1e3),
                                  "decode_tok_s_e2e": 8 * world / (dm / 1e3),
                                  "decode_tok_s_device": 8 * world / (dd / 1e3),
                                  "decode_steps": allr[0]["steps"], "per_rank": allr}),
                      flush=True)
            dist.barrier()
            dist.destroy_process_group()
        eng.close()
        return
    if args.case == "attn":
        cfg = model_cfg_dict(1)
        cfg["vocab_size"] = 4096
        model = sx.Model(eng, sx.model_config(**cfg))
        model.synth_weights(SEED)
        model.fill_kv(SEED)
        ring = sx.Ring(1, 32, 512, 96)
        ring.prefill(0, START_CLOCK)
        for r in range(96):
            ring.write_recall(0, r, START_CLOCK - 1 - r)
        for t in range(args.launches):
            c = START_CLOCK + t
            s = ring.activate_slot(0, c)
            model.forward_token(sx.synth_embed_row(3840, 5, SEED), c, s,
                                ring.get_active_slots(0, c), want_logits=False)
    elif args.case == "c3":
        # 256 independent 640-slot rings in one launch of the fused kernel
        n, G, D, total = 256, 8, 256, 640
        stride = (G + 2) * D
        qkv = torch.randn(n * stride, device="cuda", generator=g)
        kc = torch.randn(n * total * D, device="cuda", generator=g).to(torch.bfloat16)
        vc = torch.randn(n * total * D, device="cuda", generator=g).to(torch.bfloat16)
        ones = torch.ones(D, device="cuda")
        slots = torch.arange(total, dtype=torch.int32, device="cuda").repeat(n)
        steps = torch.tensor([[50000 + i, 40 + i % 500, total, 0] for i in range(n)],
                             dtype=torch.int32, device="cuda")
        out = torch.empty(n * G * D, device="cuda")
        p0 = qkv.data_ptr()
        for _ in range(args.launches):
            eng.qkv_rope_attn(p0, p0 + 4 * G * D, p0 + 4 * (G + 1) * D, ones, ones, kc, vc, slots,
                              steps, out, G, 1, D, 64, 0, 1e6, 1e-6, 1.0 / 16, total, n, stride)
    else:
        m, k = {"geglu": (args.rows, 3840), "c1": (6144, 1536)}.get(args.case, (262144, 3840))
        w0, w1 = packed(m, k), (packed(m, k) if args.case == "geglu" else None)
        x = torch.randn(k, device="cuda", generator=g)
        y = torch.empty(m, device="cuda")
        for _ in range(args.launches):
            if args.case == "geglu":
                eng.gate_up(w0, w1, x, y, m, k, 1)
            else:
                eng.gemv(sx.QUANT_Q4, w0, x, y, m, k, 1)
    eng.sync()
    eng.close()


def model_cfg_dict(layers=48):
    return dict(
        vocab_size=262144, hidden_size=3840, intermediate_size=15360, num_layers=layers,
        num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8, head_dim=256, global_head_dim=256,
        num_anchors=32, window_size=512, num_recall=96, kv_bf16=1, has_post_norms=1, full_every=5,
        attention_k_eq_v=0, rms_norm_eps=1e-6, rope_theta=10000.0, rope_theta_full=1000000.0,
        attn_scale=1.0,
    )


def algorithmic_bytes_per_token(cfg) -> dict:
    H, I, V, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"], cfg["num_layers"]
    q = cfg["num_q_heads"] * cfg["head_dim"]
    kv = cfg["num_kv_heads"] * cfg["head_dim"]
    q4 = lambda r, c: r * c // 32 * 20  # noqa: E731
    layer_w = q4(q, H) + 2 * q4(kv, H) + q4(H, q) + 2 * q4(I, H) + q4(H, I)
    head = V * H // 32 * 36
    slots = cfg["num_anchors"] + cfg["window_size"] + cfg["num_recall"]
    kv_bytes = L * slots * kv * 2 * 2  # K and V, bf16
    norms = L * (6 * H + 2 * cfg["head_dim"]) * 4 + H * 4
    return dict(weights=L * layer_w, lm_head=head, kv=kv_bytes, norms=norms,
                total=L * layer_w + head + kv_bytes + norms)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(key: str):
    """dram read + write bytes per launch of one kernel at one shape, from the ncu captures
    recorded in profiles/dram_traffic.json (None when that shape was not captured)."""
    f = ROOT / "profiles" / "dram_traffic.json"
    if not f.exists():
        return None
    entry = json.loads(f.read_text()).get("kernels", {}).get(key)
    return int(entry["dram_bytes_per_launch"]) if entry else None


def graph_time_ms(torch, eng, launch, reps=5):
    """Device time of one call of `launch()` (which issues work on the engine stream): the
    calls are captured once into a CUDA graph and the graph is replayed `reps` times between
    CUDA events on the replay stream."""
    s = torch.cuda.Stream()
    eng.set_stream(s.cuda_stream)
    try:
        with torch.cuda.stream(s):
            launch()  # warm-up outside the capture (first-use set-up)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            launch()
        with torch.cuda.stream(s):
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                g.replay()
            e1.record(s)
        s.synchronize()
        return e0.elapsed_time(e1) / reps
    finally:
        eng.set_stream(None)


def kernel_lines(torch, eng, peak) -> dict:
    """BASELINE configs 1-3 as stand-alone kernels, each over copies larger than L2 so that the
    bytes come from HBM: c1, the 6144 x 1536 Q4_0 GEMV over 64 weight copies in one graph; c2,
    the GeGLU MLP (gate+up, then down; H 1536, I 6144) over 64 weight sets at batch 1 and 8; c3,
    the fused q/k norm + RoPE + cache write + attention over 256 independent 640-slot rings
    (8 q heads, 1 kv head, D 256, bf16 cache) in one launch."""
    import sx

    out = {}

    def synth(m, k, copies, seed):
        """`copies` device copies (torch uint8 tensors) of one synthetic packed Q4_0 matrix."""
        words = sx.quantized_row_words(k, sx.QUANT_Q4)
        ref = torch.empty(m * words, dtype=torch.int32, device="cuda")
        eng.synth_weights(sx.QUANT_Q4, ref, 0, m, k, seed, 1)
        nb = sx.packed_bytes(m, k, sx.QUANT_Q4)
        first = torch.empty(nb, dtype=torch.uint8, device="cuda")
        eng.sync()
        torch.cuda.synchronize()
        buf = eng.wrap(first.data_ptr(), nb)
        buf.repack_device(ref.data_ptr(), m, k, sx.QUANT_Q4)
        eng.sync()
        buf.close()
        return [first] + [first.clone() for _ in range(copies - 1)], nb

    # ---- c1
    M, K, C = 6144, 1536, 64
    w, nb = synth(M, K, C, SEED + 11)
    x = torch.randn(K, device="cuda").to(torch.bfloat16).float()
    y = torch.empty(M, device="cuda")
    ms = graph_time_ms(torch, eng, lambda: [eng.gemv(sx.QUANT_Q4, b, x, y, M, K, 1)
                                             for b in w])
    alg = M * K // 32 * 20 + 4 * K + 4 * M
    per = ms / C
    out["c1_gemv_q4_6144x1536"] = {
        "us_per_call": per * 1e3, "algorithmic_bytes_per_call": alg,
        "achieved_gbs": alg / (per / 1e3) / 1e9, "frac": alg / (per / 1e3) / 1e9 / peak,
        "copies": C, "working_set_mb": C * nb / 1e6,
        "traffic": profiled_traffic("gemv_q4_6144x1536"),
        "timing": "64 launches on distinct weight copies captured in one CUDA graph"}
    del w
    # ---- c2
    H, I = 1536, 6144
    wg, _ = synth(I, H, 2 * C, SEED + 12)
    wd, _ = synth(H, I, C, SEED + 13)
    sets = [(wg[2 * i], wg[2 * i + 1], wd[i]) for i in range(C)]
    for batch in (1, 8):
        xb = torch.randn(batch, H, device="cuda")
        act = torch.empty(batch, I, device="cuda")
        yb = torch.empty(batch, H, device="cuda")

        def mlp():
            for g, u, d in sets:
                eng.gate_up(g, u, xb, act, I, H, batch)
                eng.gemv(sx.QUANT_Q4, d, act, yb, H, I, batch)

        ms = graph_time_ms(torch, eng, mlp)
        alg = 3 * (I * H // 32 * 20) + batch * 4 * (2 * H + 2 * I)
        per = ms / C
        out[f"c2_geglu_mlp_b{batch}"] = {
            "us_per_step": per * 1e3, "algorithmic_bytes_per_step": alg,
            "achieved_gbs": alg / (per / 1e3) / 1e9, "frac": alg / (per / 1e3) / 1e9 / peak,
            "tokens_per_s": batch / (per / 1e3), "copies": C,
            "timing": "64 (gate+up, down) launch pairs on distinct weight sets in one CUDA graph"}
    del sets, wg, wd
    # ---- c3
    n, G, D, total = 256, 8, 256, 640
    rng = np.random.default_rng(SEED + 3)
    stride = (G + 2) * D
    qkv = torch.randn(n * stride, device="cuda")
    kc = torch.randn(n * total * D, device="cuda").to(torch.bfloat16).view(torch.int16)
    vc = torch.randn(n * total * D, device="cuda").to(torch.bfloat16).view(torch.int16)
    qn = torch.ones(D, device="cuda")
    kn = torch.ones(D, device="cuda")
    slots = np.zeros((n, total), np.uint32)
    steps = np.zeros((n, 4), np.uint32)
    for i in range(n):
        ring = sx.Ring(1, 32, 512, 96)
        c = int(rng.integers(544, 100000))
        ring.prefill(0, c)
        for r in range(96):
            ring.write_recall(0, r, int(rng.integers(0, c)))
        sl = ring.activate_slot(0, c)
        a = ring.get_active_slots(0, c)
        slots[i, :len(a)] = a
        steps[i] = (c, sl, len(a), 0)
        ring.close()
    d_slots = torch.from_numpy(slots.view(np.int32)).cuda()
    d_steps = torch.from_numpy(steps.view(np.int32)).cuda()
    att = torch.empty(n * G * D, device="cuda")
    p0 = qkv.data_ptr()

    def attn():
        eng.qkv_rope_attn(p0, p0 + 4 * G * D, p0 + 4 * (G + 1) * D, qn, kn, kc, vc, d_slots,
                          d_steps, att, G, 1, D, 64, 0, 1e6, 1e-6, 1.0 / 16, total, n, stride)

    ms = graph_time_ms(torch, eng, attn, reps=10)
    live = int(steps[:, 2].sum())
    alg = live * D * 2 * 2 + n * (stride + G * D) * 4 + n * total * 4
    out["c3_attention_640slot_x256"] = {
        "us_per_launch": ms * 1e3, "instances": n, "live_slots": live,
        "algorithmic_bytes_per_launch": alg, "achieved_gbs": alg / (ms / 1e3) / 1e9,
        "frac": alg / (ms / 1e3) / 1e9 / peak, "working_set_mb": 2 * n * total * D * 2 / 1e6,
        "traffic": profiled_traffic("attn_cluster_c3_x256"),
        "timing": "one launch over 256 independent rings (168 MB of bf16 K/V), graph replays"}
    return out


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.lines: list[str] = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

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
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------
class CpuToken:
    """The CPU checker (restatement of the reference's Q4 decode path, oracle/) running whole
    decode tokens of the benchmarked workload: 48 12B-width layers with 640 live ring slots, the
    full 262144-row Q8_0 LM head and the argmax, on all host cores."""

    def __init__(self, layers: int = 48):
        from oracle import oracle as orc

        self.cores = os.cpu_count() or 1
        t0 = time.perf_counter()
        cfg = model_cfg_dict(layers)
        self.m = orc.Model(cfg, SEED, nthreads=self.cores)
        self.m.fill_kv(SEED)
        self.m.ring.prefill(0, START_CLOCK)
        self.m.synth_recall(START_CLOCK, 96, SEED)
        self.setup_s = time.perf_counter() - t0
        self.layers = layers
        self.token = 5
        self.k = 0

    def step(self) -> float:
        """Seconds for one whole token (greedy: the sampled token feeds the next step)."""
        from oracle import oracle as orc

        x = orc.synth_embed_row(3840, self.token, SEED)
        t0 = time.perf_counter()
        tok, _, _ = self.m.forward(x, START_CLOCK + self.k, want_logits=True)
        dt = time.perf_counter() - t0
        self.token = int(tok)
        self.k += 1
        return dt

    def describe(self, n) -> str:
        return (f"{n} whole tokens of the c4 workload ({self.layers} layers, 640 live slots, "
                f"262144-row Q8_0 head + argmax) on the CPU checker with {self.cores} threads "
                f"(model set-up {self.setup_s:.1f} s, untimed)")


def cpu_baseline(tokens: int = 4) -> dict:
    ct = CpuToken()
    ct.step()  # warm-up token
    times = [ct.step() for _ in range(tokens)]
    per_token = sum(times) / len(times)
    return {"value": 1.0 / per_token, "unit": UNIT, "cores": ct.cores, "kind": "port",
            "sample": ct.describe(tokens)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    ct = CpuToken()
    for _ in range(args.warmup):
        ct.step()
    steps = [ct.step() for _ in range(args.steps)]
    per_token = sum(steps) / len(steps)
    value = 1.0 / per_token
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_token * 1e3,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "c4: 12B-shape Q4_0 greedy decode, batch 1, 48 layers, H 3840, "
                               "16q/8kv x 256, I 15360, vocab 262144 (Q8_0 head), 640 live ring "
                               "slots",
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": ct.cores, "kind": "port",
                         "sample": ct.describe(args.steps)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timed_s": sum(steps),
        "note": ("the reference's own CPU path is Zig and cannot be built here (no zig "
                 "toolchain); timed the C restatement of its Q4 decode path instead, whole "
                 "tokens"),
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.case:
        run_case(args)
        return

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import sx

    cfgd = model_cfg_dict(args.layers)
    cfgd["reference_graph"] = {"persistent": 2, "stream": 3, "block": 4}.get(args.graph, 0)
    eng = sx.Engine(local)
    comm = None
    if world > 1:
        # tensor parallel over the ranks: NCCL id made on rank 0, shared through the process group
        obj = [sx.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = sx.Comm(eng, obj[0], world, rank)
        try:
            comm.set_allreduce(args.allreduce == "nccl")
        except sx.SxError:
            # sx_comm_create agreed on the peer workspaces across the ranks, so this happens on
            # every rank or on none: all keep NCCL
            args.allreduce = "nccl"
        picks = [None] * world
        dist.all_gather_object(picks, args.allreduce)
        if len(set(picks)) != 1:
            raise RuntimeError(f"ranks chose different all-reduces: {picks}")
        cfgd.update(tp_size=world, tp_rank=rank, reference_graph=0)
    stream = torch.cuda.ExternalStream(eng.stream)
    model = sx.Model(eng, sx.model_config(**cfgd), comm)
    model.synth_weights(SEED)
    model.fill_kv(SEED)
    total_slots = model.total_slots
    ring = sx.Ring(1, 32, 512, 96)
    ring.prefill(0, START_CLOCK)
    rng = np.random.default_rng(SEED)
    for r in range(96):  # synthetic recall tier: every slot live (640)
        ring.write_recall(0, r, int(rng.integers(0, START_CLOCK)))

    # ---- per-step inputs staged in HBM (value run)
    nsteps = args.warmup + args.steps
    H = cfgd["hidden_size"]
    xs = np.stack([sx.synth_embed_row(H, int(rng.integers(0, 262144)), SEED) for _ in range(nsteps)])
    slot_tab = np.zeros((nsteps, total_slots), np.uint32)
    step_tab = np.zeros((nsteps, 4), np.uint32)
    vring = sx.Ring(1, 32, 512, 96)
    vring.prefill(0, START_CLOCK)
    for r in range(96):
        vring.write_recall(0, r, START_CLOCK - 1 - r)
    for i in range(nsteps):
        c = START_CLOCK + i
        s = vring.activate_slot(0, c)
        a = vring.get_active_slots(0, c)
        slot_tab[i, : len(a)] = a
        step_tab[i] = (c, s, len(a), 0)
    d_x = torch.from_numpy(xs.astype(np.float32)).cuda()
    d_slots = torch.from_numpy(slot_tab.view(np.int32)).cuda()
    d_step = torch.from_numpy(step_tab.view(np.int32)).cuda()
    io = model.io()

    import ctypes

    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_int, ctypes.c_void_p]
    cudart.cudaMemcpyAsync.restype = ctypes.c_int
    copies = []
    for i in range(nsteps):
        copies.append(((io.x, d_x[i].data_ptr(), 4 * H),
                       (io.slots, d_slots[i].data_ptr(), 4 * total_slots),
                       (io.step, d_step[i].data_ptr(), 16)))

    def stage(i):
        # device-to-device staging of this step's resident inputs on the engine stream
        for dst, src, nb in copies[i]:
            rc = cudart.cudaMemcpyAsync(dst, src, nb, 3, eng.stream)
            if rc != 0:
                raise RuntimeError(f"cudaMemcpyAsync failed ({rc})")

    kernels_per_token = model.kernels_per_token(True)
    for i in range(args.warmup):
        stage(i)
        model.launch(True)
    eng.sync()
    if dist is not None:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.warmup, nsteps):
        stage(i)
        model.launch(True)
    ev1.record(stream)
    eng.sync()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    # one token stream, sharded over the ranks (tensor parallel) or on one GPU
    value = args.steps / (ms_max / 1e3)

    # ---- e2e through the public API (host buffers, copies inside the timed region)
    token = 7
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.warmup):
        c = START_CLOCK + nsteps + i
        x = sx.synth_embed_row(H, token, SEED)
        s = ring.activate_slot(0, c)
        token = model.forward_token(x, c, s, ring.get_active_slots(0, c), True)
    stream_tokens = []
    t0 = time.perf_counter()
    for i in range(args.steps):
        c = START_CLOCK + nsteps + args.warmup + i
        x = sx.synth_embed_row(H, token, SEED)
        s = ring.activate_slot(0, c)
        token = model.forward_token(x, c, s, ring.get_active_slots(0, c), True)
        stream_tokens.append(token)
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = args.steps / e2e_s

    # ---- roofline of the dominant kernel: fused gate+up GeGLU over the layers' weights
    peak, peak_kind = load_peaks()
    I = cfgd["intermediate_size"] // world  # this rank's gate/up rows
    gu_bytes = 2 * (I * H // 32 * 20) + H * 4 + I * 4
    roof_layers = min(args.layers, 24)
    wbufs = []
    for l in range(roof_layers):
        g = eng.buffer(sx.packed_bytes(I, H, sx.QUANT_Q4))
        u = eng.buffer(sx.packed_bytes(I, H, sx.QUANT_Q4))
        wbufs.append((g, u))
    xin = torch.randn(H, device="cuda")
    yout = torch.empty(I, device="cuda")
    torch.cuda.synchronize()
    reps = 4
    with torch.cuda.stream(stream):
        for g, u in wbufs:
            eng.gate_up(g.ptr, u.ptr, xin, yout, I, H, 1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            for g, u in wbufs:
                eng.gate_up(g.ptr, u.ptr, xin, yout, I, H, 1)
        e1.record(stream)
    eng.sync()
    launch_ms = e0.elapsed_time(e1) / (reps * len(wbufs))
    achieved = gu_bytes / (launch_ms / 1e3) / 1e9
    traffic = profiled_traffic(f"gate_up_q4_{I}x{H}")
    kernels = None
    if world == 1 and args.layers == 48 and not args.no_kernel_lines:
        kernels = kernel_lines(torch, eng, peak)
    import hashlib
    tok_bytes = np.asarray(stream_tokens, np.uint32).tobytes()

    alg = algorithmic_bytes_per_token(cfgd)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32 accumulate (Q4_0/Q8_0 weights exact; x enters the MMA as a bf16 hi+lo pair, 16 significant bits)",
        "data": "synthetic (seeded random-init 12B-shaped weights, BASELINE distributions)",
        "config": {
            "workload": f"c4: 12B-shape Q4_0 greedy decode, batch 1, {args.layers} layers, H 3840, "
                        "16q/8kv x 256, I 15360, vocab 262144 (Q8_0 head), 640 live ring slots",
            "global_batch": 1, "seq_len": total_slots,
            "parallelism": f"tp{world} ({'NCCL' if args.allreduce == 'nccl' else 'one-shot peer'} "
                           f"all-reduce x2 per layer, vocab-parallel head)"
                           if world > 1 else "single",
            "graph": {2: "one persistent cooperative launch per token (grid barriers)",
                      3: "one streaming launch per token (producer warp per SM, weight ring)",
                      4: "3 kernels per layer (attention block, gate+up, down) + LM head, "
                         "programmatic dependent launch"}
                     .get(cfgd["reference_graph"],
                          "5 kernels per layer + LM head, programmatic dependent launch"),
            "l2": "inputs larger than L2 (8.1 GB of weights+KV read per step)",
            "algorithmic_bytes_per_token": alg["total"],
            "hbm_gbs_per_token_rate": alg["total"] * value / 1e9,
        },
        "e2e": {"value": e2e, "unit": UNIT,
                "h2d_bytes_per_step": 4 * H + 4 * total_slots + 16, "d2h_bytes_per_step": 4},
        # the e2e leg's greedy token stream (same inputs for every GPU count: a tensor-parallel
        # run must reproduce the one-GPU stream)
        "tokens_sha256": hashlib.sha256(tok_bytes).hexdigest(),
        "tokens_head": [int(t) for t in stream_tokens[:8]],
        "gpu_launches": kernels_per_token * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": f"gemv_kernel<4,2,1> fused gate+up GeGLU, 2 x {I}x{H} Q4_0",
                     "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": launch_ms,
                     "peak_kind": peak_kind + " (burst copy)"},
        "clocks": clk,
    }
    if kernels is not None:
        line["kernels"] = kernels
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.close()  # its graphs hold the collectives: released before the communicator
    if comm is not None:
        comm.close()
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
