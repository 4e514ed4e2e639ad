"""Benchmark of the B200 MXFP4 MoE layer (the reference's headline metric:
MoE layer tokens/s, decode HBM GB/s, prefill tensor throughput vs peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload at N = 1: BASELINE configs[3], the GPT-OSS-20B-shaped MoE layer
prefill (hidden 2880, intermediate 2880, 32 experts, top-4, 8192 tokens, bf16
activations, MXFP4 weights), seeded synthetic inputs (no dataset or
checkpoint exists here).  A step is one full layer forward (router, permute,
W1 + SwiGLU, W2, combine).  At N > 1 each rank runs its own 8192-token batch
with the experts sharded expert-parallel (E / N per GPU) and the routed pairs
exchanged over NVLink peer memory (weak scaling).  --workload gptoss120b_moe
runs BASELINE configs[4] instead: 128 experts, Zipf(1.1)-skewed routing,
4096 tokens per GPU, 128 / N experts per GPU.

--impl reference times the CPU restatement of the reference's path (the
reference's own Rust/wgpu code cannot be built or run on this box) on a
bounded token sample per step, on all host cores; rank 0 only.
"""
import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "burn-extended_b200"), os.path.join(ROOT, "oracle")]

import numpy as np  # noqa: E402

# DRAM bytes (read + write) of one launch, from the ncu captures summarised in
# profiles/tc_moe_gemm_prefill_gptoss20b.txt and profiles/tc_moe_gemm_decode_gptoss20b.txt.
W1_PREFILL_TRAFFIC = 500.8e6 + 174.2e6
W1_DECODE_TRAFFIC = 297.2e6 + 4.4e6  # ncu dram read + write of one FP4 W1 launch (profiles/tc_moe_gemm_decode_gptoss20b.txt)

METRIC = "MoE layer tokens/s (GPT-OSS-20B-shaped MXFP4 layer, prefill 8192 tokens/GPU)"
METRIC_120B = "MoE layer tokens/s (GPT-OSS-120B-shaped MXFP4 layer, 128 experts, Zipf routing, 4096 tokens/GPU)"


def metric_of(args):
    return METRIC_120B if args.workload == "gptoss120b_moe" else METRIC
UNIT = "tokens/s"
# kernels one mxmoe_forward launches: rms, router logits, top-k, permute,
# activation quantization, W1, W2, combine
LAUNCHES_PER_FORWARD = 8


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j["hbm_gbs"], j["bf16_tflops"], j["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """SM clock and throttle-reason sampling during the timed region, from
    NVML in a background thread (every ~2 ms, so that short timed regions
    still get samples).  Only reads: no clock or setting is changed."""
    # NVML clocks-event reason bits
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.thread = None
        self.stop = False
        self.err = None

    def _handle(self, nv):
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.gpu)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.gpu)

    def _run(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self.stop:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), smax, get_reasons(h)))
                time.sleep(0.002)
        except Exception as exc:  # noqa: BLE001
            self.err = f"nvml: {exc}"

    def __enter__(self):
        import threading
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        time.sleep(0.01)  # first samples precede the timed region's start
        return self

    def __exit__(self, *a):
        self.stop = True
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"]}
        sm = [s[0] for s in self.samples]
        reasons = sorted({name for s in self.samples for bit, name in self.REASONS.items() if s[2] & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def cpu_reference(inp, sample_tokens, nthreads=0):
    import oracle
    c = oracle.cfg(inp.d, inp.f, inp.E, inp.k)
    xs = inp.x[:sample_tokens]
    t0 = time.perf_counter()
    oracle.moe_forward(c, xs, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks, inp.host.w1_scales, inp.b1,
                       inp.host.w2_blocks, inp.host.w2_scales, inp.b2, nthreads)
    return time.perf_counter() - t0


def run_reference(args, world, rank):
    if rank != 0:
        return
    import oracle
    from mxmoe import synth
    cfg_name, data_desc = WORKLOADS[args.workload]
    inp = synth.make_config(cfg_name, seed=args.seed)
    sample = args.ref_sample
    for _ in range(args.warmup):
        cpu_reference(inp, sample)
    times = [cpu_reference(inp, sample) for _ in range(args.steps)]
    total = sum(times)
    value = sample * args.steps / total
    cores = oracle.num_threads()
    line = {
        "impl": "reference", "metric": metric_of(args), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": data_desc,
        "config": {"workload": args.workload, "tokens_per_step": sample, "d_model": inp.d,
                   "ffn_hidden": inp.f, "experts": inp.E, "top_k": inp.k},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{sample} tokens of the {inp.n}-token batch per step (C oracle, OpenMP)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "burn-extended's MoE path is Rust + wgpu (Metal); no Rust toolchain or graphics stack exists on "
                "this box, so the timed reference is the C restatement of its CPU semantics",
    }
    print(json.dumps(line), flush=True)


def measure_decode(args, local, dev, hbm_peak):
    """Decode-shaped layer (64 tokens, 32 experts, top-4):
    HBM-bound; GB/s = algorithmic bytes (weights of the experts touched, router,
    x and y) per forward time."""
    import torch
    import mxmoe
    from mxmoe import synth
    dec = synth.make_config("decode", seed=args.seed)
    d, f, E = dec.d, dec.f, dec.E
    dl = mxmoe.MoeConfig(dec.d, dec.f, dec.E, dec.k).init(local)
    dl.set_router(dec.gamma, dec.gate_w, dec.gate_b)
    dl.set_resident(dec.host, dec.b1, dec.b2)
    xd = torch.from_numpy(dec.x).to(torch.bfloat16).to(dev)
    for _ in range(3):
        dl.forward(xd)
    torch.cuda.synchronize()
    s2, e2_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(args.steps):
        dl.forward(xd)
    e2_.record()
    torch.cuda.synchronize()
    dec_ms = s2.elapsed_time(e2_) / args.steps
    # SM clock under this load (a longer loop so that the sampler sees it)
    with ClockSampler(local) as clk:
        for _ in range(400):
            dl.forward(xd)
        torch.cuda.synchronize()
    dec_clocks = clk.summary()
    rr = dl.routing_results(dec.n)
    used = int((np.diff(rr["offsets"].cpu().numpy()) > 0).sum())
    per_expert = 2 * f * d // 2 + 2 * f * d // 32 + d * f // 2 + d * f // 32 + 2 * (2 * f + d)
    dec_bytes = used * per_expert + 2 * E * d + E * 2 + 2 * dec.n * d * 2
    dl.set_profiling(True)
    dp = []
    for _ in range(args.steps):
        dl.forward(xd)
        dp.append(dl.last_profile())
    dstages = {s: statistics.mean(p[s] for p in dp) for s in dp[0]}
    dl.close()
    return {"config": "gptoss20b_moe_decode (64 tokens, 32 experts, top-4)",
            "tokens_per_s": dec.n / (dec_ms / 1e3), "ms_per_step": dec_ms,
            "algorithmic_bytes": dec_bytes, "hbm_gbs": dec_bytes / (dec_ms / 1e3) / 1e9,
            "hbm_frac": dec_bytes / (dec_ms / 1e3) / 1e9 / hbm_peak, "stages_ms": dstages,
            "roofline_w1": {"bound": "hbm", "kernel": "tc_moe_gemm_kernel (W1 + SwiGLU, stacked tiles)",
                            "achieved": used * (8294400 + 518400 + 23040) / (dstages["w1_gemm"] / 1e3) / 1e9,
                            "peak": hbm_peak, "unit": "GB/s",
                            "frac": used * (8294400 + 518400 + 23040) / (dstages["w1_gemm"] / 1e3) / 1e9 / hbm_peak,
                            "traffic": W1_DECODE_TRAFFIC},
            "clocks": dec_clocks,
            "l2": "weights of the 32 experts (423 MB) exceed the 126 MB L2; no flush"}


def measure_decode_batches(args, local, dev, hbm_peak):
    """Small-batch decode of the GPT-OSS-20B-shaped layer (32 experts, top-4)
    at 1, 2, 4, 8 and 16 tokens through the default dispatch (the fused
    dequant-GEMV kernel up to 8 routed pairs, the kind::mxf4 tensor-core tiles
    above).  GB/s = bytes of the experts the batch touches (codes, scales,
    biases) plus router weights and x / y, per layer forward.  The weights
    (423 MB) exceed the 126 MB L2, and consecutive forwards use different
    tokens and so different experts."""
    import torch
    import mxmoe
    from mxmoe import synth
    d = f = 2880
    per_expert = 2 * f * d // 2 + 2 * f * d // 32 + d * f // 2 + d * f // 32 + 2 * (2 * f + d)
    base = synth.make_config("decode", seed=args.seed + 3)
    L = mxmoe.MoeConfig(base.d, base.f, base.E, base.k).init(local)
    L.set_router(base.gamma, base.gate_w, base.gate_b)
    L.set_resident(base.host, base.b1, base.b2)
    L.reserve(16)
    out = {}
    for n in (1, 2, 4, 8, 16):
        # 32 different token batches in rotation: the touched experts change
        xs = [torch.from_numpy(synth.rank_tokens(base, r, args.seed).x[:n]).to(torch.bfloat16).to(dev)
              for r in range(32)]
        touched = []
        for xi in xs:
            L.forward(xi)
            rr = L.routing_results(n)
            touched.append(int((np.diff(rr["offsets"].cpu().numpy()) > 0).sum()))
        for _ in range(3):
            for xi in xs:
                L.forward(xi)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        calls = max(args.steps, 1) * len(xs)
        s.record()
        for i in range(calls):
            L.forward(xs[i % len(xs)])
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) / calls * 1e3
        nbytes = float(np.mean(touched)) * per_expert + 2 * base.E * d + base.E * 2 + 2 * n * d * 2
        out[f"n{n}"] = {"us_per_layer": us, "tokens_per_s": n / (us / 1e6), "experts_touched": float(np.mean(touched)),
                        "bytes": nbytes, "gbs": nbytes / (us / 1e6) / 1e9,
                        "hbm_frac": nbytes / (us / 1e6) / 1e9 / hbm_peak,
                        "x_touched_bytes_at_peak": us / (nbytes / (hbm_peak * 1e9) * 1e6),
                        "path": "dequant-GEMV (fused)" if n * base.k <= 8 else "kind::mxf4 tensor-core tiles"}
    L.close()
    return {"config": "gptoss20b_moe_decode at batch 1..16 (32 experts, top-4), bf16 x, default dispatch",
            "rotation": "32 token batches per n (different experts each)", **out}


def measure_attention(args, local, dev, hbm_peak):
    """Streaming multi-query attention decode step (mxmqa_forward_streaming)
    at the GPT-OSS shape: d_model 2880, 64 query heads over 8 KV heads of 64,
    learned sinks, bf16 weights, RoPE base 150000 with YaRN x32, a 128-token
    sliding window over a 160-slot ring cache (and a 4096-token full cache).
    A step is one new token per sequence after a 2048-token prompt.  GB/s =
    the q/k/v/o weights (53.1 MB bf16) plus the KV rows read (window x 8
    heads x 64 x 4 B x 2 per sequence) plus x / y, per step; the weights and a
    flushed L2 make every step stream from HBM."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "burn-extended_b200"))
    from mxmoe.attention import (AttnWindow, RopeConfig, StreamingMqaCache, StreamingMqaParams,
                                 StreamingMultiQueryAttentionConfig)
    d, nH, kvH, dk = 2880, 64, 8, 64
    rng = np.random.default_rng(args.seed + 11)

    def w(shape, sc):
        a = rng.standard_normal(shape).astype(np.float32) * np.float32(sc)
        u = a.view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    jq, jk = nH * dk, kvH * dk
    m = StreamingMultiQueryAttentionConfig(d, nH, kvH, dk).init(local)
    m.set_weights(w((d, jq), d ** -0.5), w((jq,), 0.02), w((d, jk), d ** -0.5), w((jk,), 0.02),
                  w((d, jk), d ** -0.5), w((jk,), 0.02), w((jq, d), jq ** -0.5), w((d,), 0.02), bf16=True)
    m.set_sinks(rng.standard_normal((kvH, nH // kvH)).astype(np.float32))
    m.set_rope(RopeConfig(131072, 150000.0, 32.0, 4096.0, 1.0, 32.0))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    wbytes = 2 * (d * (jq + 2 * jk) + jq * d)
    out = {}
    for B in (1, 8, 32):
        for name, cap, win in (("window128", 160, 128), ("full4096", 4096, None)):
            cache = StreamingMqaCache(m, B, cap, 0)
            prompt = torch.randn(B, 2048 if win is None else 128, d, device=dev).to(torch.bfloat16)
            pos = prompt.shape[1]
            m.forward_streaming(prompt, cache, StreamingMqaParams(0, AttnWindow(win)))
            x = torch.randn(B, 1, d, device=dev).to(torch.bfloat16)
            for _ in range(3):
                m.forward_streaming(x, cache, StreamingMqaParams(pos, AttnWindow(win)))
                pos += 1
            times = []
            for _ in range(max(args.steps, 5)):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                m.forward_streaming(x, cache, StreamingMqaParams(pos, AttnWindow(win)))
                e.record()
                torch.cuda.synchronize()
                times.append(s.elapsed_time(e) * 1e3)
                pos += 1
            us = float(np.median(times))
            keys = min(pos, cap) if win is None else win
            nbytes = wbytes + B * keys * kvH * dk * 4 * 2 + 2 * B * d * 2
            out[f"B{B}_{name}"] = {"us_per_step": us, "tokens_per_s": B / (us / 1e6), "bytes": nbytes,
                                   "gbs": nbytes / (us / 1e6) / 1e9, "hbm_frac": nbytes / (us / 1e6) / 1e9 / hbm_peak}
            cache.close()
    m.close()
    return {"config": "gptoss attention decode step (d 2880, 64 q / 8 kv heads x 64, sinks, bf16 weights, YaRN)",
            "l2": "256 MB buffer zeroed before every timed step", **out}


def measure_microbench(args, local, dev, hbm_peak):
    """Single-expert fused dequant + GEMV: W1 [5760, 2880]
    and W2 [2880, 2880] MXFP4, bf16 activations at T = 1, 2, 4, 8 tokens.
    Independent copies of the expert (one layer each) are used in rotation,
    together 4x the 126 MB L2, so every call streams its weights from HBM.
    GB/s = algorithmic bytes (the expert's codes, scales and biases plus the
    activations in and out) / time, for the whole layer call and for its two
    GEMM launches alone (CUDA events on the call's stream)."""
    import torch
    import mxmoe
    from mxmoe import synth
    d = f = 2880
    per_expert = 2 * f * d // 2 + 2 * f * d // 32 + d * f // 2 + d * f // 32
    copies = int(np.ceil(4 * 126e6 / per_expert)) + 1
    base = synth.make_inputs(d, f, 1, 1, 8, True, seed=args.seed + 7)
    layers = []
    for _ in range(copies):
        L = mxmoe.MoeConfig(d, f, 1, 1).init(local)
        L.set_router(base.gamma, base.gate_w, base.gate_b)
        L.set_resident(base.host, base.b1, base.b2)
        L.reserve(8)  # the rotation never resizes a workspace inside the timed loop
        layers.append(L)
    out = {}
    for T in (1, 2, 4, 8):
        x = torch.from_numpy(base.x[:T]).to(torch.bfloat16).to(dev)
        for _ in range(2):  # the second call per layer captures its CUDA graph
            for L in layers:
                L.forward(x)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        calls = max(args.steps, 1) * copies
        s.record()
        for i in range(calls):
            layers[i % copies].forward(x)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / calls
        gemm = []
        for i in range(copies):
            layers[i].set_profiling(True)
            layers[i].forward(x)
            pr = layers[i].last_profile()
            gemm.append(pr["w1_gemm"] + pr["w2_gemm"])
            layers[i].set_profiling(False)
        gemm_ms = statistics.median(gemm)
        nbytes = per_expert + 2 * (2 * f + d) + 2 * T * d * 2
        out[f"T{T}"] = {"us_per_call": ms * 1e3, "gbs": nbytes / (ms / 1e3) / 1e9,
                        "hbm_frac": nbytes / (ms / 1e3) / 1e9 / hbm_peak, "gemm_us": gemm_ms * 1e3,
                        "gemm_gbs": nbytes / (gemm_ms / 1e3) / 1e9,
                        "gemm_hbm_frac": nbytes / (gemm_ms / 1e3) / 1e9 / hbm_peak}
    for L in layers:
        L.close()
    return {"config": "single-expert MXFP4 dequant+GEMV, W1 [5760,2880] + W2 [2880,2880], bf16 x",
            "rotation": f"{copies} expert copies ({copies * per_expert / 1e6:.0f} MB, >= 4x L2)",
            "algorithmic_bytes_per_call": "codes + scales + biases + 2*T*d*2 activation bytes", **out}


def measure_120b(args, local, dev):
    """GPT-OSS-120B-shaped layer on one GPU: 4096 tokens,
    128 experts, top-4, router bias giving a Zipf(1.1)-like expert load."""
    import torch
    import mxmoe
    from mxmoe import synth
    inp = synth.make_config("gptoss120b", seed=args.seed)
    L = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k).init(local)
    L.set_router(inp.gamma, inp.gate_w, inp.gate_b)
    L.set_resident(inp.host, inp.b1, inp.b2)
    x = torch.from_numpy(inp.x).to(torch.bfloat16).to(dev)
    for _ in range(3):
        L.forward(x)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        L.forward(x)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    load = np.diff(L.routing_results(inp.n)["offsets"].cpu().numpy())
    flops = 2.0 * inp.n * inp.k * (2 * inp.f * inp.d + inp.f * inp.d) + 2.0 * inp.n * inp.d * inp.E
    L.close()
    return {"config": "gptoss120b_moe (4096 tokens, 128 experts, top-4, Zipf(1.1) router bias), 1 GPU",
            "tokens_per_s": inp.n / (ms / 1e3), "ms_per_step": ms, "useful_tflops": flops / (ms / 1e3) / 1e12,
            "expert_load_max": int(load.max()), "expert_load_mean": float(load.mean()),
            "expert_load_max_over_mean": float(load.max() / load.mean()), "experts_unused": int((load == 0).sum())}


# workload name -> (synth config, data description)
WORKLOADS = {
    "gptoss20b_moe_prefill": ("prefill", "synthetic (seeded, BASELINE configs[3] shapes)"),
    "gptoss120b_moe": ("gptoss120b", "synthetic (seeded, BASELINE configs[4] shapes, Zipf(1.1) router bias)"),
}


def run_ours(args, world, rank, local):
    import torch
    import mxmoe
    from mxmoe import synth

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    hbm_peak, tc_burst, tc_sust, peak_src = load_peaks()
    if args.only == "decode":
        print(json.dumps({"decode": measure_decode(args, local, dev, hbm_peak)}), flush=True)
        return
    if args.only == "microbench":
        print(json.dumps({"microbench": measure_microbench(args, local, dev, hbm_peak)}), flush=True)
        return
    if args.only == "decode_batches":
        print(json.dumps({"decode_batches": measure_decode_batches(args, local, dev, hbm_peak)}), flush=True)
        return
    if args.only == "gptoss120b":
        print(json.dumps({"gptoss120b": measure_120b(args, local, dev)}), flush=True)
        return
    if args.only == "attention":
        print(json.dumps({"attention": measure_attention(args, local, dev, hbm_peak)}), flush=True)
        return

    # one model on every rank (seeded once); each rank routes its own tokens
    cfg_name, data_desc = WORKLOADS[args.workload]
    inp = synth.make_config(cfg_name, seed=args.seed)
    if world > 1:
        inp = synth.rank_tokens(inp, rank, args.seed)
    n, d, f, E, k = inp.n, inp.d, inp.f, inp.E, inp.k
    if world > 1:
        from mxmoe import ep
        placement = replicas = None
        if args.workload == "gptoss120b_moe":
            # skewed routing: one extra expert slot per GPU for copies of the
            # hottest experts, then load-balanced placement of the slots, both
            # from the router loads of one seeded calibration batch (the same
            # on every rank)
            cal = synth.rank_tokens(inp, 0, args.seed + 1)
            loads = ep.expert_loads(cal.x, cal.gamma, cal.gate_w, cal.gate_b, k)
            if not args.no_replicas:
                replicas = ep.plan_replicas(loads, world)
                loads = np.array([loads[e] / np.count_nonzero(replicas == e) for e in replicas])
            placement = ep.balanced_placement(loads, world)
        runner = ep.build_quantized_peer_rank(inp, world, rank, dev, placement=placement, replicas=replicas)
        step = lambda x: runner.forward(x)  # noqa: E731
        x = torch.from_numpy(inp.x).to(torch.bfloat16).to(dev)
    else:
        layer = mxmoe.MoeConfig(d, f, E, k).init(local)
        layer.set_router(inp.gamma, inp.gate_w, inp.gate_b)
        layer.set_resident(inp.host, inp.b1, inp.b2)
        layer.reserve(n)
        x = torch.from_numpy(inp.x).to(torch.bfloat16).to(dev)
        y = torch.empty_like(x)
        stream = torch.cuda.current_stream()

        def step(xx):
            mxmoe.lib()
            mxmoe.check(mxmoe.lib().mxmoe_forward(layer._h, xx.data_ptr(), mxmoe.BF16, y.data_ptr(), mxmoe.BF16, n,
                                                   stream.cuda_stream))
            return y

    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        start.record()
        for _ in range(args.steps):
            step(x)
        stop.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = n * world * args.steps / (ms / 1e3)
    clocks = clk.summary()

    if world > 1:
        stages = runner.profile(x, args.steps)
        # end to end through the layer's Python API: each step copies its
        # tokens from pinned host memory, runs the expert-parallel forward and
        # reads the output back to pinned host memory; wall clock, max over ranks
        xh = x.cpu().pin_memory()
        yh = torch.empty_like(xh).pin_memory()
        xd = torch.empty_like(x)

        def e2e_step():
            xd.copy_(xh, non_blocking=True)
            yh.copy_(runner.forward(xd), non_blocking=True)
            torch.cuda.current_stream().synchronize()

        e2e_step()
        torch.distributed.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        e2e_s = torch.tensor([(time.perf_counter() - t0) / args.steps], device=dev)
        torch.distributed.all_reduce(e2e_s, op=torch.distributed.ReduceOp.MAX)
        e2e = {"value": n * world / float(e2e_s.item()), "unit": UNIT,
               "h2d_bytes_per_step": xh.numel() * xh.element_size(),
               "d2h_bytes_per_step": yh.numel() * yh.element_size(), "per": "rank"}
        if rank == 0:
            line = {"metric": metric_of(args), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "e2m1 x e4m3(2 terms), f32 accum",
                    "data": data_desc,
                    "config": {"workload": args.workload, "tokens_per_gpu": n, "experts": E,
                               "experts_per_gpu": runner.E // world, "top_k": k, "parallelism": f"ep{world}",
                               "placement": "contiguous" if placement is None else
                               "load-balanced (greedy on the router loads of a seeded calibration batch)",
                               "expert_slots": runner.E,
                               "replicas": None if replicas is None else
                               f"{len(replicas) - E} copies of the hottest experts, pairs split by token",
                               "l2": "working set > 126 MB L2 (expert weights alone 423 MB per 32 experts)"},
                    "e2e": e2e, "clocks": clocks, "stages_ms": stages,
                    "gpu_launches": runner.launches_per_step * args.steps}
            print(json.dumps(line), flush=True)
        torch.distributed.destroy_process_group()
        return

    # per-stage device times (CUDA events on the forward's stream), separate pass
    layer.set_profiling(True)
    prof = []
    for _ in range(args.steps):
        step(x)
        prof.append(layer.last_profile())
    layer.set_profiling(False)
    stages = {s: statistics.mean(p[s] for p in prof) for s in prof[0]}
    P = n * k
    w1_flops = 2.0 * P * (2 * f) * d
    w2_flops = 2.0 * P * d * f
    t_w1 = stages["w1_gemm"] / 1e3
    achieved = w1_flops / t_w1 / 1e12
    # W1 is timed alone (CUDA events around its launch inside a 1.5 ms step),
    # so the denominator is the burst bf16 peak; the two-term E4M3 x E2M1 MMA
    # pair issues at the bf16-equivalent rate.  North star's MXF4 target is
    # also reported: MXF4 dense is 4x bf16 dense (9 vs 2.25 PFLOP/s nominal),
    # applied to the measured bf16 burst.
    roofline = {"bound": "tensor", "kernel": "tc_moe_gemm_kernel (W1 + SwiGLU)", "achieved": achieved,
                "peak": tc_burst, "unit": "TFLOP/s", "frac": achieved / tc_burst,
                "peak_source": f"{peak_src} bf16 burst (kernel timed alone)",
                "frac_of_mxf4_peak": achieved / (4.0 * tc_burst),
                "mxf4_peak_source": f"4 x {peak_src} bf16 burst (nominal MXF4 : bf16 dense = 9 : 2.25)",
                "traffic": W1_PREFILL_TRAFFIC if args.workload == "gptoss20b_moe_prefill" else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum "
                "of one W1 launch (profiles/tc_moe_gemm_prefill_gptoss20b.txt)",
                "flops_per_launch": w1_flops}
    layer_flops = w1_flops + w2_flops
    extra = {"layer_tflops": layer_flops / (ms_per_step / 1e3) / 1e12,
             "w2_tflops": w2_flops / (stages["w2_gemm"] / 1e3) / 1e12}

    if args.only == "prefill":
        print(json.dumps({"metric": metric_of(args), "value": value, "unit": UNIT, "ms_per_step": ms_per_step,
                          "stages_ms": stages, "roofline": roofline, "clocks": clocks}), flush=True)
        layer.close()
        return
    # end to end through the public host-buffer entry point (pinned memory)
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    layer.forward_host(xh, yh)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer.forward_host(xh, yh)
    e2e_s = (time.perf_counter() - t0) / args.steps
    e2e = {"value": n / e2e_s, "unit": UNIT, "h2d_bytes_per_step": xh.numel() * xh.element_size(),
           "d2h_bytes_per_step": yh.numel() * yh.element_size()}

    if args.workload == "gptoss20b_moe_prefill":
        extra["decode"] = measure_decode(args, local, dev, hbm_peak)
    if args.only == "all" and args.workload == "gptoss20b_moe_prefill":
        extra["decode_batches"] = measure_decode_batches(args, local, dev, hbm_peak)
        extra["microbench"] = measure_microbench(args, local, dev, hbm_peak)
        extra["gptoss120b"] = measure_120b(args, local, dev)

    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        sample = args.cpu_sample
        cpu_reference(inp, 2)
        dt = cpu_reference(inp, sample)
        cpu = {"value": sample / dt, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
               "sample": f"{sample} tokens of the {n}-token batch (C oracle, OpenMP, all host threads)"}

    line = {
        "metric": metric_of(args), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 x e4m3(2 terms), f32 accum",
        "data": data_desc,
        "config": {"workload": args.workload, "tokens": n, "d_model": d, "ffn_hidden": f, "experts": E,
                   "top_k": k, "parallelism": "ep1",
                   "l2": "inputs+weights > 126 MB L2 (expert weights alone 423 MB); no flush"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks, "stages_ms": stages,
        "gpu_launches": LAUNCHES_PER_FORWARD * args.steps, "extra": extra,
    }
    print(json.dumps(line), flush=True)
    layer.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample", type=int, default=24)
    ap.add_argument("--ref-sample", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-replicas", action="store_true",
                    help="gptoss120b_moe at N > 1: placement only, no copies of hot experts")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="gptoss20b_moe_prefill",
                    help="gptoss20b_moe_prefill (configs[3], the headline) or gptoss120b_moe (configs[4]: 128 "
                         "experts, Zipf-skewed routing, 4096 tokens per GPU; expert-parallel at N > 1)")
    ap.add_argument("--only", choices=["all", "prefill", "decode", "decode_batches", "microbench", "gptoss120b", "attention"],
                    default="all",
                    help="run only that leg (profiling runs); 'all' adds decode, microbench and gptoss120b as extras")
    args = ap.parse_args()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
