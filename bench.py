"""Benchmark of the ds-ocr MoE-decoder hot path on B200.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                [--workload decode|moe_layer|prefill] [--engine 0|1]

Prints ONE JSON line (rank 0). Under torchrun (N > 1) every rank runs its own
independent replica of the workload (weak scaling: decode streams / tokens
are independent), timing is on the device with CUDA events, max over ranks.

Workloads (synthetic random-init weights):
  decode    config 3: greedy decode of the 12-layer DeepSeek3B-MoE decoder,
            batch 1, 662-token BF16 KV prefix        (headline)
  moe_layer config 0: one MoE layer, one token; steps rotate over 11 layers'
            weights (5.0 GB) so no step finds its experts in L2
  prefill   config 4: batched MoE prefill, 3328 tokens through the 11 MoE
            layers (router logits overridden, skewed routing)
  lm_head   config 1: argmax LM head 129280 x 1280 at batch 64 (and batch 1)
  decode64  config 3 at 64 independent streams, sharded by stream over the
            GPUs (one tensor-core step for all of a GPU's streams)
--impl reference times the reference's own CPU code (compiled unmodified
into oracle/_ref/libdsref.so) on the same workload, on this host's cores.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    d = dict(PEAKS_FALLBACK)
    d["source"] = "fallback"
    return d


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        pg = dist
    return rank, world, local, pg


def max_over_ranks(v, pg):
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v, pg):
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return float(t.item())


def barrier(pg):
    if pg is not None:
        pg.barrier()


def cpu_threads():
    return max(1, min(16, os.cpu_count() or 1))


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------
MOE_BYTES_PER_TOKEN = 163840 + 6 * 6881280 + 13762560   # config 0 algorithmic bytes
# DRAM bytes per launch of the dominant kernels (dram__bytes_read.sum +
# dram__bytes_write.sum of one ncu capture of each: the batch-1 and batch-64
# LM heads and the prefill gate/up GEMM at 3328 tokens)
TRAFFIC_ARGMAX_TMA = 331042048 + 4175872
TRAFFIC_LT_ARGMAX = 331387648 + 6157568
TRAFFIC_PF_GATE_UP = 423503616 + 78080000
LM_BYTES = 129280 * 1280 * 2                                 # config 1 per call


class MoeLayerWorkload:
    """Config 0. 11 distinct MoE layers (as in the decoder) registered in HBM;
    step s runs layer s % 11 on token input s."""

    name = "moe_layer"
    metric = "MoE layer decode tokens/s (1 token, 64 experts top-6 + 2 shared, BF16)"
    unit = "tokens/s"

    def __init__(self, n_layers=11, n_inputs=64):
        from ds_ocr_b200 import synth
        self.d = synth.Dims()
        self.layers = [synth.MoeWeights(self.d, l + 1) for l in range(n_layers)]
        self.X = synth.normal_f32((n_inputs, self.d.hidden), synth.seed_of("bench", "moe_x"))

    def config(self):
        return {"workload": "config0_moe_layer", "hidden": 1280, "experts": 64, "top_k": 6, "shared": 2,
                "moe_inter": 896, "layers_rotated": len(self.layers), "batch": 1,
                "l2": "weights rotate over 11 layers (5.0 GB) > L2"}


# Config 2: the INT8 (--int4) expert path. Per token: the BF16 router plus,
# for each of the 6 routed experts, gate/up int8 [1792 x 1280] + 2 x 1792
# F32 scale/offset and down int8 [1280 x 896] + 2 x 1280 F32, and the shared
# expert's int8 gate/up [3584 x 1280] + 2 x 3584 F32 and down [1280 x 1792]
# + 2 x 1280 F32 = 27,875,328 B.
INT8_BYTES_PER_TOKEN = (163840 + 6 * (2293760 + 14336 + 1146880 + 10240)
                        + (4587520 + 28672 + 2293760 + 10240))


class MoeLayerInt8Workload(MoeLayerWorkload):
    """Config 2: config 0's layers with per-row INT8 expert copies,
    quantised by the GPU quantiser (bit-identical to ds_int4_quantize_bf16)."""

    name = "moe_layer_int8"
    metric = "INT8 MoE layer decode tokens/s (1 token, 64 experts top-6 + 2 shared, per-row INT8 experts)"

    def __init__(self, ctx=None, n_layers=11, n_inputs=64):
        super().__init__(n_layers, n_inputs)
        if ctx is not None:
            self.quantize(ctx)

    def quantize(self, ctx):
        from ds_ocr_b200 import synth
        from ds_ocr_b200.decoder import quantize_int8
        carrier = synth.Model.__new__(synth.Model)
        carrier.d = self.d
        carrier.layers = [type("L", (), {"moe": m})() for m in self.layers]
        quantize_int8(carrier, ctx)

    def config(self):
        c = super().config()
        c.update(workload="config2_moe_layer_int8", experts_dtype="int8 per-row asymmetric",
                 l2="int8 weights rotate over 11 layers (2.5 GB) > L2")
        return c


def run_ours_moe(args, rank, world, pg, int8=False):
    import torch
    from ds_ocr_b200 import cuda
    ctx = cuda.Context(0 if world == 1 else int(os.environ.get("LOCAL_RANK", "0")))
    wl = MoeLayerInt8Workload(ctx) if int8 else MoeLayerWorkload()
    d = wl.d
    lib = ctx.lib
    Q8 = ("gu_q", "gu_s", "gu_o", "dn_q", "dn_s", "dn_o", "sgu_q", "sgu_s", "sgu_o", "sdn_q", "sdn_s", "sdn_o")
    for mw in wl.layers:
        for a in (mw.router, mw.block, mw.down, mw.shared_down):
            ctx.register(a)
        if int8:
            for n in Q8:
                ctx.register(getattr(mw.int8, n))
    dev = [(ctx.device_ptr(m.router), ctx.device_ptr(m.block), ctx.device_ptr(m.down), ctx.device_ptr(m.shared_down))
           for m in wl.layers]
    dev8 = [[ctx.device_ptr(getattr(m.int8, n)) for n in Q8] for m in wl.layers] if int8 else None
    dX = torch.from_numpy(wl.X).cuda()
    dout = torch.empty((wl.X.shape[0], d.hidden), device="cuda")
    didx = torch.empty((wl.X.shape[0], 8), dtype=torch.int32, device="cuda")
    dw = torch.empty((wl.X.shape[0], 8), device="cuda")
    torch.cuda.synchronize()
    st = torch.cuda.ExternalStream(ctx.stream)
    nL, nX = len(dev), wl.X.shape[0]

    def step(s):
        r, b, dn, sd = dev[s % nL]
        i = s % nX
        if int8:
            rc = lib.ds_cuda_moe_layer_int8_dev(ctx.h, dX[i].data_ptr(), dout[i].data_ptr(), r, *dev8[s % nL],
                                                d.hidden, d.moe_inter, d.shared_inter, d.n_experts, d.top_k,
                                                didx[i].data_ptr(), dw[i].data_ptr(), None)
        else:
            rc = lib.ds_cuda_moe_layer_dev(ctx.h, dX[i].data_ptr(), dout[i].data_ptr(), r, b, dn, sd, d.hidden,
                                           d.moe_inter, d.shared_inter, d.n_experts, d.top_k, didx[i].data_ptr(),
                                           dw[i].data_ptr(), None)
        assert rc == 0, lib.ds_cuda_last_error(ctx.h)

    for s in range(args.warmup):
        step(s)
    ctx.synchronize()
    barrier(pg)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        ctx.synchronize()
        ev0.record(st)
        for s in range(args.steps):
            step(s)
        ev1.record(st)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, pg)
    value = world * args.steps / (ms_max / 1e3)

    # e2e: host pointers through the Metal-shaped public API, host copies inside
    e2e_steps = max(args.steps // 4, 8)
    ctx.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(st)
    for s in range(e2e_steps):
        mw = wl.layers[s % nL]
        if int8:
            ctx.moe_layer_int8(wl.X[s % nX], mw)
        else:
            ctx.moe_layer(wl.X[s % nX], mw)
    t1.record(st)
    t1.synchronize()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), pg)
    e2e = world * e2e_steps / (e2e_ms / 1e3)
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clk.summary(),
        "e2e": {"value": e2e, "unit": wl.unit, "h2d_bytes_per_step": d.hidden * 4,
                "d2h_bytes_per_step": d.hidden * 4 + 2 * d.top_k * 4},
        "gpu_launches": 3 * args.steps, "config": wl.config(), "metric": wl.metric, "unit": wl.unit,
        "dtype": "bf16 weights, f32 math",
    }
    bpt = INT8_BYTES_PER_TOKEN if int8 else MOE_BYTES_PER_TOKEN
    achieved = bpt / (ms_max / args.steps / 1e3) / 1e9
    pk = peaks()
    res["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                       "frac": achieved / pk["hbm_gbs"], "traffic": None,
                       "kernel": f"moe layer (router + gate_up + down{', INT8 experts' if int8 else ''}), "
                                 f"{bpt:,} B/token",
                       "peak_source": pk["source"]}
    if int8:
        res["dtype"] = "int8 expert weights (per-row scale/offset), bf16 router, f32 math"
    ctx.close()
    return res


def ref_moe_time(wl, threads, budget_s, int8=False):
    """Times the reference's own moe_forward (compiled unmodified into
    oracle/_ref/libdsref.so) on the same layers and inputs, `threads` host
    threads, for about budget_s seconds of work. Returns (tokens/s, calls).
    int8: the reference's --int4 path (its own ds_int4_quantize_bf16, then
    moe_forward's INT8 branch, ds_moe_decoder.c:237-243, 269-278) on the
    first 3 layers (quantised outside the timed calls; 0.7 GB of INT8
    weights, far above the host caches)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from ds_ocr_b200 import synth
    nl = 3 if int8 else 1
    carrier = synth.Model.__new__(synth.Model)
    carrier.d = synth.Dims(n_layers=1 + nl, vocab=16)
    carrier.layers = []
    carrier.final_norm = np.ones(1280, np.float32)
    carrier.lm_head = np.zeros((16, 1280), np.uint16)
    R = O.RefDecoder(carrier, kv_max=8, threads=threads)
    if int8:
        for l in range(nl):
            R.set_layer(1 + l, wl.layers[l])
        R.r.ref_ctx_quantize(R.ctx)
    n, t_total = 0, 0.0
    while t_total < budget_s:
        if int8:
            layer = 1 + n % nl
        else:
            layer = 1
            R.set_layer(1, wl.layers[n % len(wl.layers)])
        x = wl.X[n % wl.X.shape[0]]
        t = time.perf_counter()
        R.moe_forward(layer, x)
        t_total += time.perf_counter() - t
        n += 1
    R.close()
    return n / t_total, n


# ---------------------------------------------------------------------------
# Decode (config 3), the headline workload
# ---------------------------------------------------------------------------
DEC_WEIGHT_BYTES = 1148318720        # per token: attention + dense L0 + 11 MoE + LM head + norms
KV_BYTES_PER_KEY = 61440             # 12 layers x (K + V) x 1280 x BF16
PREFIX = 662


def decode_bytes(first_pos, n_steps):
    keys = sum(first_pos + s + 1 for s in range(n_steps))
    return DEC_WEIGHT_BYTES * n_steps + KV_BYTES_PER_KEY * keys


def sampling_of(args):
    """(repeat_penalty, no_repeat_ngram_size, temperature) of the decode
    workloads; all defaults = greedy argmax (the reference's defaults,
    ds_ocr.c:949-951)."""
    return (getattr(args, "repeat_penalty", 1.0), getattr(args, "no_repeat_ngram", 0),
            getattr(args, "temperature", 0.0))


def decode_mode(args):
    rp, ng, t = sampling_of(args)
    if rp <= 1.0 and ng <= 0 and t <= 0.0:
        return "greedy"
    return f"repeat_penalty={rp:g}, no_repeat_ngram_size={ng}, temperature={t:g}"


def decode_config(kv_max):
    return {"workload": "config3_decode_b1", "model": "DeepSeek3B-MoE decoder (12 layers, random init)",
            "global_batch": 1, "streams_per_gpu": 1, "kv_prefix": PREFIX, "kv_max": kv_max,
            "hidden": 1280, "experts": 64, "top_k": 6, "vocab": 129280,
            "l2": "each step streams 1.2 GB of weights (> 126 MB L2)"}


def build_decode_model():
    from ds_ocr_b200 import synth
    model = synth.Model()
    ks, vs = synth.kv_prefix(model.d, PREFIX)
    return model, ks, vs


def run_ours_decode(args, rank, world, pg, model, ks, vs):
    import torch
    from ds_ocr_b200 import cuda
    from ds_ocr_b200.decoder import Decoder
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = cuda.Context(local if world > 1 else 0)
    kv_max = 1024
    dec = Decoder(model, ctx, kv_max=kv_max, engine=args.engine)
    dec.load_kv(ks, vs)
    rp, ng, temp = sampling_of(args)
    sampled = decode_mode(args) != "greedy"
    if sampled:
        dec.set_sampling(rp, ng, temp)
    unif = np.random.default_rng(17).random(max(args.steps, args.warmup) + 1).astype(np.float32)

    def fresh_history():
        # each phase starts a generation: empty history, its own uniforms
        if sampled:
            dec.set_history([])
            if temp > 0:
                dec.set_uniforms(unif)

    st = torch.cuda.ExternalStream(ctx.stream)
    e0 = model.embed(1)
    # warm-up (graph capture happens here), then reset to the prefix
    fresh_history()
    dec.generate(args.warmup, first_embed=e0)
    dec.set_len(PREFIX)
    fresh_history()
    dec.forward(e0)
    first = PREFIX + 1
    ctx.synchronize()
    barrier(pg)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(st)
        dec.generate_dev(args.steps)
        ev1.record(st)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, pg)
    value = world * args.steps / (ms_max / 1e3)
    step_bytes = decode_bytes(first, args.steps)
    launches = dec.launches_per_step

    # e2e: the public host-pointer API, one call per token: H2D of the
    # token's embedding, D2H of the token (+ its logit), host picks the next
    # embedding (the reference's decode loop, ds_ocr.c:2157-2282)
    n_e2e = args.steps
    dec.set_len(PREFIX)
    fresh_history()
    e = e0
    ctx.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(st)
    for _ in range(n_e2e):
        tok = dec.forward(e)
        e = model.embed(tok)
    t1.record(st)
    t1.synchronize()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), pg)
    e2e = world * n_e2e / (e2e_ms / 1e3)

    # LM-head argmax kernel launched alone on the same stream (same kernel,
    # same grid): its own roofline, reported beside the step's
    lib = ctx.lib
    d_lm = ctx.device_ptr(model.lm_head)
    X = torch.randn(64, 1280, device="cuda")
    tok_t = torch.zeros(64, dtype=torch.int32, device="cuda")
    val_t = torch.zeros(64, device="cuda")
    torch.cuda.synchronize()
    for i in range(5):
        lib.ds_cuda_argmax_matvec_bf16_dev(ctx.h, X[i].data_ptr(), d_lm, 1280, 129280, tok_t[i].data_ptr(),
                                           val_t[i].data_ptr(), None)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nk = 50
    k0.record(st)
    for i in range(nk):
        lib.ds_cuda_argmax_matvec_bf16_dev(ctx.h, X[i % 64].data_ptr(), d_lm, 1280, 129280,
                                           tok_t[i % 64].data_ptr(), val_t[i % 64].data_ptr(), None)
    k1.record(st)
    k1.synchronize()
    lm_us = k0.elapsed_time(k1) / nk * 1e3
    pk = peaks()
    lm_ach = LM_BYTES / (lm_us * 1e-6) / 1e9
    step_ach = step_bytes / (ms_max / 1e3) / 1e9
    # the step's dominant kernel, timed live inside the graph (per-CTA
    # globaltimer trace over 3 steps): its critical-path time per launch
    dominant = None
    if args.engine == 0 and not sampled:
        from ds_ocr_b200 import trace as dtrace
        dec.set_len(PREFIX + 1)
        launches_t = dtrace.capture(lambda: dec.generate_dev(3))
        summ = dtrace.summary(launches_t, 3)
        name, d = max(summ.items(), key=lambda kv: kv[1]["share"])
        kb = {"moe_step_kernel": MOE_BYTES_PER_TOKEN}.get(name)
        dominant = {"kernel": name, "us_per_launch": d["us_per_launch"], "share_of_step": d["share"],
                    "launches_per_step": d["launches_per_step"], "kernels": summ,
                    "timing": "per-CTA globaltimer trace inside the CUDA graph (last exit minus the previous "
                              "launch's last exit), 3 steps"}
        if kb:
            ach = kb / (d["us_per_launch"] * 1e-6) / 1e9
            dominant.update({"bytes_per_launch": kb, "achieved": ach, "unit": "GB/s", "peak": pk["hbm_gbs"],
                             "frac": ach / pk["hbm_gbs"]})
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clk.summary(),
        "metric": f"decode tokens/s ({decode_mode(args)}, batch 1 per GPU, 12-layer DeepSeek3B-MoE, "
                  "662-token KV prefix)",
        "unit": "tokens/s", "dtype": "bf16 weights + bf16 KV, f32 math",
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 1280 * 4, "d2h_bytes_per_step": 8},
        # persistent engine: the timed region is ONE kernel launch for all steps
        "gpu_launches": launches * args.steps if launches else 1,
        "config": dict(decode_config(kv_max), engine=["kernel graph", "persistent kernel"][args.engine],
                       **({"sampling": decode_mode(args)} if sampled else {})),
        # the roofline of the whole step: one CUDA graph whose kernels all
        # stream weights (1.196 GB per token at the mean context)
        "roofline": {"bound": "hbm", "achieved": step_ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": step_ach / pk["hbm_gbs"], "frac_of_8tbs": step_ach / 8000.0, "traffic": None,
                     "kernel": "decode step (CUDA graph of all kernels)",
                     "bytes_per_token": step_bytes / args.steps, "peak_source": pk["source"]},
        "dominant_kernel": dominant,
        "lm_head_roofline": {"bound": "hbm", "achieved": lm_ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": lm_ach / pk["hbm_gbs"], "traffic": TRAFFIC_ARGMAX_TMA,
                             "kernel": "argmax_tma_kernel (LM head 129280x1280, 330,956,800 B/launch)",
                             "kernel_us": lm_us},
    }
    dec.close()
    ctx.close()
    return res


MS_STREAMS = 64
MS_ATTN_BYTES = 157286400 + 52592640    # attention (12 layers) + dense layer 0 weights
MS_MOE_LAYER_BYTES = 64 * 6881280 + 13762560 + 163840   # every expert touched (64 streams x top-6)


def run_ours_decode_streams(args, rank, world, pg, model, prefixes):
    """Config 3 at 64 streams, sharded by stream: this rank decodes streams
    [rank*64/G, (rank+1)*64/G) in lockstep (one tensor-core step for all of
    them), weights replicated per GPU, no collective."""
    import torch
    from ds_ocr_b200 import cuda
    from ds_ocr_b200.decoder import BatchDecoder
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = cuda.Context(local if world > 1 else 0)
    a, b = MS_STREAMS * rank // world, MS_STREAMS * (rank + 1) // world
    S = b - a
    kv_max = 1024
    bd = BatchDecoder(model, S, ctx, kv_max=kv_max)
    for i in range(S):
        ks, vs = prefixes[a + i]
        bd.load_kv(i, ks, vs)
    st = torch.cuda.Stream()
    sp = st.cuda_stream
    E = np.stack([model.embed((1 + 7 * (a + i)) % model.d.vocab) for i in range(S)])
    rp, ng, temp = sampling_of(args)
    sampled = decode_mode(args) != "greedy"
    n_e2e = max(3, args.steps // 4)
    if sampled:
        # the LM head's sampling settings for every stream (each with its own
        # history); uniforms for every step the run takes
        bd.set_sampling(rp, ng, temp)
        if temp > 0:
            bd.set_uniforms(np.random.default_rng(11).random((S, 1 + args.warmup + args.steps + n_e2e))
                            .astype(np.float32))
    bd.forward(E)  # first step from the given embeddings (and scratch set-up)
    bd.generate_dev(max(1, args.warmup - 1), sp)
    st.synchronize()
    barrier(pg)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(st)
        bd.generate_dev(args.steps, sp)
        ev1.record(st)
        ev1.synchronize()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), pg)
    value = MS_STREAMS * args.steps / (ms_max / 1e3)
    # e2e: the host API, one call per step (previous tokens' embeddings on
    # the device, the S tokens copied back every step)
    for i in range(S):
        bd.set_len(i, PREFIX)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(st)
    bd.forward(E)
    for _ in range(n_e2e - 1):
        bd.forward()
    t1.record(st)
    t1.synchronize()
    e2e = MS_STREAMS * n_e2e / (max_over_ranks(t0.elapsed_time(t1), pg) / 1e3)
    first = PREFIX + args.warmup
    keys = sum(first + s + 1 for s in range(args.steps))
    step_bytes = MS_ATTN_BYTES + 11 * MS_MOE_LAYER_BYTES + LM_BYTES + 128000 + KV_BYTES_PER_KEY * S * keys / args.steps
    pk = peaks()
    ach = step_bytes / (ms_max / args.steps / 1e3) / 1e9
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clk.summary(),
        "metric": (f"decode tokens/s ({decode_mode(args)}, 64 independent streams, 12-layer DeepSeek3B-MoE, "
                   "662-token KV prefixes)"),
        "unit": "tokens/s", "dtype": "bf16 weights + bf16 KV, f32 activations as two bf16 planes, f32 accumulate",
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": S * 4},
        # per step: 7 per layer (3 norm/split passes, QKV, RoPE/KV, attention,
        # O-proj), 2 per dense FFN, 8 per MoE layer (router, top-k, count,
        # plan, scatter, gate/up, down, combine), 3 for the final norm, LM
        # head and advance (177 per step, as in the ncu launch list); with
        # sampling settings the selection kernels (history dots with a
        # penalty and no temperature, fast, full-logits, full selection)
        "gpu_launches": (7 * model.d.n_layers + 2 * model.d.first_dense
                         + 8 * (model.d.n_layers - model.d.first_dense) + 3
                         + ((4 if rp > 1.0 and temp <= 0.0 else 3) if sampled else 0)) * args.steps,
        "config": dict(decode_config(kv_max), workload="config3_decode_64_streams", global_batch=MS_STREAMS,
                       streams_per_gpu=S, parallelism=f"sharded by stream over {world} GPU(s)",
                       **({"sampling": decode_mode(args)} if sampled else {})),
        "roofline": {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / pk["hbm_gbs"], "traffic": None,
                     "kernel": "whole step: weights once per step (all 64 experts of each MoE layer assumed "
                               "touched) + every stream's KV",
                     "peak_source": pk["source"]},
        "scaling": "strong" if world > 1 else "weak",
    }
    bd.close()
    del st
    torch.cuda.synchronize()
    ctx.close()
    return res


def ref_decode_time(model, ks, vs, threads, budget_s, max_steps, sampling=(1.0, 0, 0.0)):
    """The reference's own ds_decoder_forward (compiled unmodified) on the
    same weights and KV prefix, `threads` host threads, with the sampling
    settings and the generation loop's history (ds_ocr.c:2245-2248)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    R = O.RefDecoder(model, kv_max=1024, threads=threads)
    R.load_kv(ks, vs)
    R.set_sampling(*sampling)
    R.set_history([])
    e = model.embed(1)
    tok = R.step_gen(e)             # warm (page-in, thread pool)
    e = model.embed(tok)
    n, t_total = 0, 0.0
    while t_total < budget_s and n < max_steps:
        t = time.perf_counter()
        tok = R.step_gen(e)
        t_total += time.perf_counter() - t
        e = model.embed(tok)
        n += 1
    R.close()
    return n / t_total, n


_STREAM_MODEL = None  # shared with forked reference processes (copy-on-write)


def _ref_stream(args):
    threads, budget_s, max_steps, stream, sampling = args
    from ds_ocr_b200 import synth
    ks, vs = synth.kv_prefix(_STREAM_MODEL.d, PREFIX, stream=stream)
    return ref_decode_time(_STREAM_MODEL, ks, vs, threads, budget_s, max_steps, sampling=sampling)


def ref_decode_streams_time(model, threads, budget_s, max_steps, sampling=(1.0, 0, 0.0)):
    """The reference decodes streams one at a time per context; its
    multi-stream aggregate is floor(nproc / threads) concurrent processes,
    one stream each (stream s's own KV prefix). Returns (aggregate tokens/s,
    steps per process, processes). Forks: call only from a process without
    a CUDA context."""
    import multiprocessing as mp
    global _STREAM_MODEL
    n_proc = max(1, (os.cpu_count() or 1) // threads)
    _STREAM_MODEL = model
    jobs = [(threads, budget_s, max_steps, s, sampling) for s in range(n_proc)]
    if n_proc == 1:
        v, n = _ref_stream(jobs[0])
        return v, n, 1
    with mp.get_context("fork").Pool(n_proc) as pool:
        res = pool.map(_ref_stream, jobs)
    return sum(v for v, _ in res), min(n for _, n in res), n_proc


# ---------------------------------------------------------------------------
# Argmax LM head (config 1), batch 64 and batch 1
# ---------------------------------------------------------------------------
LM_BATCH = 64


def lm_inputs():
    from ds_ocr_b200 import synth
    W = synth.normal_bf16((129280, 1280), 300)
    X = synth.normal_f32((LM_BATCH, 1280), 2)
    return W, X


def lm_config():
    return {"workload": "config1_lm_head_b64", "vocab": 129280, "hidden": 1280, "batch": LM_BATCH,
            "kernel": "tcgen05 argmax (split-BF16 inputs, one pass over W)",
            "l2": "each call streams 331 MB of weights (> 126 MB L2)"}


def run_ours_lmhead(args, rank, world, pg):
    import torch
    from ds_ocr_b200 import cuda
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = cuda.Context(local if world > 1 else 0)
    lib = ctx.lib
    W, X = lm_inputs()
    ctx.register(W)
    dW = ctx.device_ptr(W)
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    dX = torch.from_numpy(X).cuda()
    tok = torch.zeros(LM_BATCH, dtype=torch.int32, device="cuda")
    val = torch.zeros(LM_BATCH, device="cuda")
    sp = st.cuda_stream

    def call(B):
        if B == 1:
            rc = lib.ds_cuda_argmax_matvec_bf16_dev(ctx.h, dX.data_ptr(), dW, 1280, 129280, tok.data_ptr(),
                                                    val.data_ptr(), sp)
        else:
            rc = lib.ds_cuda_argmax_matvec_bf16_batch_dev(ctx.h, dX.data_ptr(), dW, 1280, 129280, B, tok.data_ptr(),
                                                          val.data_ptr(), sp)
        assert rc == 0, lib.ds_cuda_last_error(ctx.h)

    def timed(B, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(n):
            call(B)
        e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1)

    for _ in range(args.warmup):
        call(LM_BATCH)
        call(1)
    st.synchronize()
    barrier(pg)
    with ClockSampler(local) as clk:
        ms = timed(LM_BATCH, args.steps)
    ms_max = max_over_ranks(ms, pg)
    value = world * LM_BATCH * args.steps / (ms_max / 1e3)
    ms1 = timed(1, args.steps)
    # e2e: host inputs in, tokens and logits out, through the host API
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(3, args.steps // 4)
    t0.record(st)
    for _ in range(n_e2e):
        ctx.argmax_batch(X, W, 1280, 129280)
    t1.record(st)
    t1.synchronize()
    e2e = world * LM_BATCH * n_e2e / (max_over_ranks(t0.elapsed_time(t1), pg) / 1e3)
    pk = peaks()
    us = ms_max / args.steps * 1e3
    ach = LM_BYTES / (us * 1e-6) / 1e9
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clk.summary(),
        "metric": "argmax LM head tokens/s (batch 64, vocab 129280 x 1280 BF16)", "unit": "tokens/s",
        "dtype": "bf16 weights, f32 inputs as two bf16 planes, f32 accumulate",
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": LM_BATCH * 1280 * 4,
                "d2h_bytes_per_step": LM_BATCH * 8},
        "gpu_launches": 2 * args.steps, "config": lm_config(),
        "roofline": {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / pk["hbm_gbs"], "traffic": TRAFFIC_LT_ARGMAX,
                     "kernel": "lt_argmax_kernel (330,956,800 B per call)", "kernel_us": us,
                     "peak_source": pk["source"]},
        "batch1": {"us_per_call": ms1 / args.steps * 1e3, "tokens_per_s": args.steps / (ms1 / 1e3),
                   "kernel": "argmax_tma_kernel"},
    }
    del dX, tok, val
    torch.cuda.synchronize()
    ctx.close()
    return res


def ref_lmhead_time(threads, budget_s):
    """The reference's ds_argmax_matvec_bf16 (compiled unmodified), one call
    per input as the reference does, on `threads` host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    W, X = lm_inputs()
    r = O.ref()
    r.ref_set_threads(threads)
    n, t_total = 0, 0.0
    while t_total < budget_s and n < 4 * LM_BATCH:
        t = time.perf_counter()
        r.ref_argmax(X[n % LM_BATCH].ctypes.data, W.ctypes.data, 1280, 129280, None)
        t_total += time.perf_counter() - t
        n += 1
    return n / t_total, n


# ---------------------------------------------------------------------------
# Batched MoE prefill (config 4)
# ---------------------------------------------------------------------------
PF_TOKENS = 3328
PF_LAYERS = 11
PF_FLOPS_LAYER = PF_TOKENS * (6 * 6881280 + 13762560)        # routed + shared, per MoE layer
PF_FLOPS_GU_LAYER = PF_TOKENS * (6 * 2 * 1792 * 1280 + 2 * 3584 * 1280)


def prefill_inputs(d, n=PF_TOKENS):
    """x [n x 1280] N(0,1) (seed 5); per layer l = 1..11 the router logits
    N(0,1) (seed 600+l) plus a per-expert bias N(0,0.5) (seed 700+l), which
    replace xn W_r^T and give the skewed routing of config 4. The generator
    is counter-based, so the first 3328 rows are config 4's at any n."""
    from ds_ocr_b200 import synth
    x = synth.normal_f32((n, d.hidden), 5)
    logits = []
    for l in range(1, PF_LAYERS + 1):
        lg = synth.normal_f32((n, d.n_experts), 600 + l)
        lg += 0.5 * synth.normal_f32(d.n_experts, 700 + l)[None, :]
        logits.append(lg)
    return x, logits


def prefill_config(n_layers=PF_LAYERS):
    return {"workload": "config4_prefill_moe" if n_layers == PF_LAYERS else f"prefill_moe_{n_layers}_layers",
            "model": "DeepSeek3B-MoE MoE layers 1-11 (random init)",
            "tokens": PF_TOKENS, "layers": n_layers, "hidden": 1280, "experts": 64, "top_k": 6,
            "routing": "logits N(0,1) + per-expert bias N(0,0.5) (attention not included)",
            "gemm": "tcgen05 split-BF16 activations x BF16 weights, F32 accumulate",
            "l2": "each step streams 5.0 GB of expert weights and 0.5 GB of activations (> 126 MB L2)"}


def run_ours_prefill(args, rank, world, pg, model):
    import torch
    from ds_ocr_b200 import cuda
    from ds_ocr_b200.prefill import Prefill
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = cuda.Context(local if world > 1 else 0)
    d = model.d
    pf = Prefill(d, ctx)
    # strong scaling: config 4's 3328 tokens split over the ranks; weak:
    # 3328 tokens per rank (a batch of 3328 x N)
    weak = getattr(args, "ep_scaling", "strong") == "weak" and world > 1
    ntot = PF_TOKENS * world if weak else PF_TOKENS
    x, logits = prefill_inputs(d, ntot)
    n_layers = args.prefill_layers
    layers = model.layers[1:1 + n_layers]
    logits = logits[:n_layers]
    ep = None
    native = getattr(args, "ep_impl", "native") == "native"
    a, b = 0, PF_TOKENS
    if world > 1:
        # expert-parallel: this rank's token slice, experts [rank*E/G, ...)
        from ds_ocr_b200.ep import CudaStages, ExpertParallelPrefill, NativeExpertParallelPrefill, token_range
        a, b = token_range(ntot, rank, world)
        if native:
            # the library's own layer: NCCL from C, the id shared over the
            # process group
            uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(NativeExpertParallelPrefill.unique_id(ctx)),
                                           dtype=torch.uint8))
            pg.broadcast(uid, 0)  # pg: the torch.distributed module (default group)
            ep = NativeExpertParallelPrefill(d, ctx, rank, world, bytes(uid.cpu().numpy().tobytes()))
            st = torch.cuda.Stream()
        else:
            stages = CudaStages(d, ctx)
            ep = ExpertParallelPrefill(d, stages, pg, rank, world, stages.device)
            st = stages.stream
    else:
        st = torch.cuda.Stream()
    # every kernel, copy and collective of a step runs on stream st (the C
    # ABI takes its handle per call)
    sp = st.cuda_stream
    torch.cuda.set_stream(st)
    dx0 = torch.from_numpy(x[a:b].copy()).cuda()
    dx = dx0.clone()
    dlg = [torch.from_numpy(l[a:b].copy()).cuda() for l in logits]
    st.synchronize()

    def run_layers(xbuf, lgs):
        for lw, lg in zip(layers, lgs):
            if ep is None:
                pf.moe_layer_dev(lw, xbuf.data_ptr(), PF_TOKENS, lg.data_ptr(), stream=sp)
            elif native:
                ep.moe_layer(lw, xbuf, lg, stream=sp)
            else:
                ep.moe_layer(lw, xbuf, lg)

    def step():
        dx.copy_(dx0)
        run_layers(dx, dlg)

    for _ in range(args.warmup):
        step()
    st.synchronize()
    pf.check()
    barrier(pg)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(st)
        for _ in range(args.steps):
            step()
        ev1.record(st)
        ev1.synchronize()
    pf.check()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), pg)
    # expert-parallel: (row, expert) pairs each rank computed, max / mean
    ep_load = None
    if ep is not None:
        if native:
            # (token, expert) pairs each rank's experts take per step, from
            # the routing the logits fix (top-6 of each row)
            e_per = d.n_experts // world
            pairs = [0] * world
            for lg in logits:
                top = np.argpartition(-lg, d.top_k - 1, axis=1)[:, :d.top_k]
                cnt = np.bincount((top // e_per).ravel(), minlength=world)
                pairs = [p + int(c) for p, c in zip(pairs, cnt)]
        else:
            pairs = ep.load()[0]
        mean = sum(pairs) / len(pairs)
        ep_load = {"pairs_per_rank_per_step": pairs, "imbalance_max_over_mean": max(pairs) / mean,
                   "impl": "ds_cuda_prefill_moe_ep (NCCL from the library)" if native
                           else "torch.distributed all_to_all_single between the stage kernels"}
    # one GPU: 3328 tokens per step; expert-parallel: the same 3328 tokens
    # split over the ranks (strong scaling)
    value = ntot * args.steps / (ms_max / 1e3)

    # per-stage device times (one extra, untimed pass): the gate/up GEMM is
    # the dominant kernel
    pf.timing(True)
    stages = np.zeros(6)
    dx.copy_(dx0)
    for lw, lg in zip(layers, dlg):
        if ep is None:
            pf.moe_layer_dev(lw, dx.data_ptr(), PF_TOKENS, lg.data_ptr(), stream=sp)
        elif native:
            ep.moe_layer(lw, dx, lg, stream=sp)
        else:
            ep.moe_layer(lw, dx, lg)
        stages += pf.stage_ms()
    pf.timing(False)
    stages /= len(layers)

    # e2e through the public API with host buffers: one GPU, the host-pointer
    # ds_cuda_prefill_moe per layer (x and logits in, x and routing out);
    # expert-parallel, the rank's x slice and logits copied in from pinned
    # host memory before the layers and x copied out after them
    n_e2e = max(1, min(args.steps, 3))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.synchronize()
    barrier(pg)
    if ep is None:
        xs = x.copy()
        t0.record(st)
        for _ in range(n_e2e):
            xs[:] = x
            for lw, lg in zip(layers, logits):
                pf.moe_layer(lw, xs, lg)
        t1.record(st)
        h2d = n_layers * PF_TOKENS * (d.hidden + d.n_experts) * 4
        d2h = n_layers * PF_TOKENS * (d.hidden + 2 * d.top_k) * 4
    else:
        hx = torch.from_numpy(x[a:b].copy()).pin_memory()
        hl = [torch.from_numpy(l[a:b].copy()).pin_memory() for l in logits]
        out = torch.empty_like(hx).pin_memory()
        t0.record(st)
        for _ in range(n_e2e):
            dx.copy_(hx, non_blocking=True)
            for dl, hlg in zip(dlg, hl):
                dl.copy_(hlg, non_blocking=True)
            run_layers(dx, dlg)
            out.copy_(dx, non_blocking=True)
        t1.record(st)
        h2d = (b - a) * (d.hidden + n_layers * d.n_experts) * 4
        d2h = (b - a) * d.hidden * 4
    t1.synchronize()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), pg)
    e2e = ntot * n_e2e / (e2e_ms / 1e3)
    pk = peaks()
    peak_t = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    # expert-parallel: rank 0's GEMM does about 1/G of the layer's work
    gu_ach = PF_FLOPS_GU_LAYER * (ntot / PF_TOKENS) / world / (stages[3] / 1e3) / 1e12
    step_ach = PF_FLOPS_LAYER * (ntot / PF_TOKENS) * n_layers * args.steps / (ms_max / 1e3) / 1e12 / world
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clk.summary(),
        "metric": "MoE prefill tokens/s (3328 tokens x 11 MoE layers, 64 experts top-6 + 2 shared)",
        "unit": "tokens/s", "dtype": "bf16 weights, f32 activations as two bf16 planes, f32 accumulate",
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        # per layer: norm/route, count, plan, scatter, gate/up, down, combine
        # (7); expert-parallel adds the dispatch plan, row packing and pair
        # compaction (10)
        "gpu_launches": (7 if world == 1 else 10) * n_layers * args.steps,
        "config": dict(prefill_config(n_layers), parallelism=f"ep{world}" if world > 1 else "single GPU",
                       tokens_per_rank=b - a, global_batch=ntot),
        "scaling": "strong" if world > 1 and not weak else "weak",
        "roofline": {"bound": "tensor", "achieved": gu_ach, "peak": peak_t, "unit": "TFLOP/s",
                     "frac": gu_ach / peak_t, "traffic": TRAFFIC_PF_GATE_UP if world == 1 else None,
                     "kernel": "pf_gemm_kernel<0> (gate/up + SwiGLU), 122.1 GFLOP algorithmic per layer; "
                               "the split-BF16 A operand doubles the tensor work (not counted)",
                     "kernel_us": stages[3] * 1e3, "peak_source": pk["source"] + " (sustained bf16)"},
        "step_roofline": {"bound": "tensor", "achieved": step_ach, "peak": peak_t, "unit": "TFLOP/s",
                          "frac": step_ach / peak_t, "flops_per_step": PF_FLOPS_LAYER * n_layers,
                          "stage_us": dict(zip(["norm_route", "plan", "scatter", "gemm_gate_up", "gemm_down",
                                                "combine"], [round(float(s) * 1e3, 1) for s in stages]))},
    }
    if ep_load is not None:
        res["ep_load"] = ep_load
    if native and ep is not None:
        torch.cuda.synchronize()
        ep.close()
    # torch tensors used on the context's stream go before the stream does
    del dx, dx0, dlg, ep
    import gc
    gc.collect()
    torch.cuda.synchronize()
    ctx.close()
    return res


# ---------------------------------------------------------------------------
# Whole-decoder prefill (the widened config 4: ds_decoder_prefill)
# ---------------------------------------------------------------------------
PFF_REF_TOKENS = 128   # the reference's bounded CPU sample


def prefill_full_flops(T, d):
    """Algorithmic FLOPs of ds_decoder_prefill on T tokens from an empty
    cache: QKV + O projections, causal attention (QK and PV), dense layer 0,
    11 MoE layers (6 routed + shared experts + router), the first token's
    LM-head row."""
    H, QD = d.hidden, d.n_heads * d.head_dim
    proj = 2 * T * (H * 3 * QD + QD * H)
    attn = 4 * QD * T * (T + 1) // 2
    dense = 2 * T * 3 * d.dense_inter * H
    moe = 2 * T * (d.top_k * 3 * d.moe_inter * H + 3 * d.n_shared * d.moe_inter * H + d.n_experts * H)
    n_moe = d.n_layers - d.first_dense
    return d.n_layers * (proj + attn) + d.first_dense * dense + n_moe * moe + 2 * d.vocab * H


def prefill_full_embeds(model, T):
    """Input embeddings: the embedding rows of a seeded token sequence."""
    ids = (np.arange(T, dtype=np.int64) * 7919 + 13) % model.d.vocab
    return np.stack([model.embed(int(t)) for t in ids])


def prefill_full_config(T):
    return {"workload": "config4_full_prefill", "model": "DeepSeek3B-MoE decoder (12 layers, random init)",
            "tokens": T, "layers": 12, "hidden": 1280, "experts": 64, "top_k": 6,
            "routing": "the model's own router", "kv": "written to the decoder's cache (kv_max 4096)",
            "gemm": "tcgen05 split-BF16 activations x BF16 weights, F32 accumulate; attention on tcgen05 (split-BF16 Q K^T and W V) with the reference's sequential fast-exp rule per query row",
            "l2": "each step streams 5.9 GB of weights (> 126 MB L2)"}


def run_ours_prefill_full(args, rank, world, pg, model):
    """ds_decoder_prefill of 3328 tokens through all 12 layers on one GPU per
    rank (replicas only: a prefill does not shard here; every rank runs its
    own)."""
    import torch
    from ds_ocr_b200 import cuda
    from ds_ocr_b200.decoder import Decoder
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = cuda.Context(local if world > 1 else 0)
    d = model.d
    T = PF_TOKENS
    dec = Decoder(model, ctx, kv_max=4096)
    emb = prefill_full_embeds(model, T).astype(np.float32)
    st = torch.cuda.ExternalStream(ctx.stream)
    d_emb = torch.from_numpy(emb).cuda()
    torch.cuda.synchronize()

    def step():
        dec.set_len(0)
        dec.prefill_dev(d_emb.data_ptr(), T)

    for _ in range(args.warmup):
        step()
    ctx.synchronize()
    barrier(pg)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(st)
        for _ in range(args.steps):
            step()
        ev1.record(st)
        ev1.synchronize()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), pg)
    value = world * T * args.steps / (ms_max / 1e3)
    # e2e: the host-pointer API, embeddings in, first token out
    n_e2e = max(1, min(args.steps, 3))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.synchronize()
    t0.record(st)
    for _ in range(n_e2e):
        dec.set_len(0)
        dec.prefill(emb)
    t1.record(st)
    t1.synchronize()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), pg)
    pk = peaks()
    peak_t = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    flops = prefill_full_flops(T, d)
    ach = flops * args.steps / (ms_max / 1e3) / 1e12
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clk.summary(),
        "metric": "whole-decoder prefill tokens/s (3328 tokens x 12 layers: attention, dense layer 0, 11 MoE layers)",
        "unit": "tokens/s", "dtype": "bf16 weights, f32 activations as two bf16 planes, f32 accumulate",
        "e2e": {"value": world * T * n_e2e / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * d.hidden * 4,
                "d2h_bytes_per_step": 8},
        # per prefill: every layer norm/split, QKV GEMM, RoPE/KV, attention,
        # split, O-proj GEMM, residual (7); a dense layer + norm/split, gate/up,
        # down, residual (4); a MoE layer + router norm/split, router GEMM and
        # route, count, plan, scatter, gate/up, down, combine (9); then the
        # LM-head argmax, final norm, finish (3): 190 for 1 dense + 11 MoE
        "gpu_launches": (7 * d.n_layers + 4 * d.first_dense + 9 * (d.n_layers - d.first_dense) + 3) * args.steps,
        "config": dict(prefill_full_config(T), parallelism=f"replicas on {world} GPU(s)"),
        "roofline": {"bound": "tensor", "achieved": ach, "peak": peak_t, "unit": "TFLOP/s", "frac": ach / peak_t,
                     "traffic": None, "kernel": "whole prefill step (algorithmic FLOPs of every GEMM and the "
                                                "attention / step time)",
                     "flops_per_step": flops, "peak_source": pk["source"]},
    }
    if world > 1:
        res["scaling"] = "weak"
    dec.close()
    ctx.close()
    return res


def ref_prefill_full_time(model, threads, T=PFF_REF_TOKENS):
    """The reference's own ds_decoder_prefill (compiled unmodified) on the
    first T tokens of the same embeddings, from an empty cache."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    emb = prefill_full_embeds(model, T).astype(np.float32)
    R = O.RefDecoder(model, kv_max=4096, threads=threads)
    R.prefill(emb[:8])  # warm (weight conversion, thread pool)
    R.r.ref_ctx_set_len(R.ctx, 0)
    t = time.perf_counter()
    R.prefill(emb)
    dt = time.perf_counter() - t
    R.close()
    return T / dt, T


def ref_prefill_time(model, threads, budget_s):
    """The reference's prefill MoE block (its own kernels and OpenBLAS sgemm,
    compiled unmodified) on the config-4 inputs, one layer per call, until
    about budget_s seconds have passed. Returns (tokens/s through 11 layers,
    layers run)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    x, logits = prefill_inputs(model.d)
    R = O.RefDecoder(model, kv_max=8, threads=threads)
    n, t_total = 0, 0.0
    xs = x.copy()
    while t_total < budget_s and n < PF_LAYERS:
        t = time.perf_counter()
        R.prefill_moe(1 + n, xs, logits[n])
        t_total += time.perf_counter() - t
        n += 1
    R.close()
    return PF_TOKENS * n / (t_total * PF_LAYERS), n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=224)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "decode64", "moe_layer", "moe_layer_int8", "prefill", "prefill_full",
                             "lm_head"])
    ap.add_argument("--engine", type=int, default=0, choices=[0, 1],
                    help="decode engine: 0 CUDA graph of per-phase kernels, 1 persistent kernel")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of reference CPU work to time")
    ap.add_argument("--prefill-layers", type=int, default=PF_LAYERS,
                    help="prefill: MoE layers per step (11 = config 4; fewer only for small profiling runs)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep-impl", default="native", choices=["native", "torch"],
                    help="expert-parallel prefill: the library's NCCL layer or torch.distributed between stages")
    ap.add_argument("--ep-scaling", default="strong", choices=["strong", "weak"],
                    help="prefill on N GPUs: 3328 tokens split over the ranks (strong) or 3328 per rank (weak)")
    ap.add_argument("--no-ep-prefill", action="store_true",
                    help="decode: skip the expert-parallel prefill block reported beside the decode line")
    ap.add_argument("--repeat-penalty", type=float, default=1.0,
                    help="decode: the reference's --repeat-penalty (> 1 enables)")
    ap.add_argument("--no-repeat-ngram", type=int, default=0,
                    help="decode: the reference's --no-repeat-ngram (V3 CLI default 35)")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="decode: sampling temperature (> 0 enables; uniforms supplied per step)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local, pg = dist_setup(args.gpus)
    T = cpu_threads()
    common = {"higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "data": "synthetic (seeded random-init weights of the DeepSeek3B-MoE shapes; BF16 N(0,1) KV prefix)"}

    if args.impl == "reference":
        if rank != 0:
            return
        # the reference arm draws the same synthetic weights through the numpy
        # restatement of the generator: this process maps no library of ours
        from ds_ocr_b200 import synth
        synth.use_numpy_backend(True)
        if args.workload == "decode":
            model, ks, vs = build_decode_model()
            v, n = ref_decode_time(model, ks, vs, T, max(args.cpu_budget, 1.0), max_steps=args.steps,
                                   sampling=sampling_of(args))
            metric = (f"decode tokens/s ({decode_mode(args)}, batch 1 per GPU, 12-layer DeepSeek3B-MoE, "
                      "662-token KV prefix)")
            cfg, sample = decode_config(1024), f"{n} {decode_mode(args)} ds_decoder_forward steps from position 663"
            if decode_mode(args) != "greedy":
                cfg["sampling"] = decode_mode(args)
        elif args.workload == "decode64":
            model, _, _ = build_decode_model()
            v, n, n_proc = ref_decode_streams_time(model, T, max(args.cpu_budget, 1.0), args.steps,
                                                   sampling=sampling_of(args))
            metric = (f"decode tokens/s ({decode_mode(args)}, 64 independent streams, 12-layer DeepSeek3B-MoE, "
                      "662-token KV prefixes)")
            cfg = dict(decode_config(1024), workload="config3_decode_64_streams", global_batch=MS_STREAMS)
            if decode_mode(args) != "greedy":
                cfg["sampling"] = decode_mode(args)
            sample = (f"{n_proc} concurrent reference processes of {T} threads, one stream each "
                      f"(the reference decodes one stream per context), {n} ds_decoder_forward steps each")
        elif args.workload == "lm_head":
            v, n = ref_lmhead_time(T, max(args.cpu_budget, 1.0))
            metric = "argmax LM head tokens/s (batch 64, vocab 129280 x 1280 BF16)"
            cfg, sample = lm_config(), f"{n} ds_argmax_matvec_bf16 calls (one per input)"
        elif args.workload == "prefill":
            from ds_ocr_b200 import synth
            v, n = ref_prefill_time(synth.Model(), T, max(args.cpu_budget, 1.0))
            metric = "MoE prefill tokens/s (3328 tokens x 11 MoE layers, 64 experts top-6 + 2 shared)"
            cfg, sample = prefill_config(), f"{n} of 11 MoE layers of the prefill block at 3328 tokens"
        elif args.workload == "prefill_full":
            from ds_ocr_b200 import synth
            v, n = ref_prefill_full_time(synth.Model(), T)
            metric = ("whole-decoder prefill tokens/s (3328 tokens x 12 layers: attention, dense layer 0, "
                      "11 MoE layers)")
            cfg = prefill_full_config(PF_TOKENS)
            sample = f"one ds_decoder_prefill of the first {n} tokens (12 layers)"
        elif args.workload == "moe_layer_int8":
            wl = MoeLayerInt8Workload(n_layers=3)
            v, n = ref_moe_time(wl, T, max(args.cpu_budget, 1.0), int8=True)
            metric, cfg = wl.metric, dict(wl.config(), layers_rotated=11)
            sample = f"{n} single-token INT8 moe_forward calls over 3 layers quantised by the reference"
        else:
            wl = MoeLayerWorkload()
            v, n = ref_moe_time(wl, T, max(args.cpu_budget, 1.0))
            metric, cfg, sample = wl.metric, wl.config(), f"{n} single-token moe_forward calls over 11 layers"
        line = {"impl": "reference", "metric": metric, "value": v, "unit": "tokens/s", "n_gpus": 0, "steps": n,
                "warmup": 1, "ms_per_step": 1e3 / v,
                "dtype": ("int8 expert weights (per-row scale/offset), bf16 router, f32 math"
                          if args.workload == "moe_layer_int8" else "bf16 weights, f32 math"), "config": cfg,
                "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": T, "kind": "reference", "sample": sample},
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        line.update(common)
        print(json.dumps(line), flush=True)
        return

    if args.workload == "decode":
        model, ks, vs = build_decode_model()
        res = run_ours_decode(args, rank, world, pg, model, ks, vs)
        if not args.no_ep_prefill:
            # the path that shards with a collective, measured at every N
            # beside the decode replicas: config 4's expert-parallel prefill
            # (3328 tokens over the ranks, experts in blocks of 64 / N)
            import copy
            pa = copy.copy(args)
            pa.steps, pa.warmup = min(args.steps, 10), 3
            pa.ep_scaling = "weak"
            pr = run_ours_prefill(pa, rank, world, pg, model)
            res["ep_prefill"] = {"metric": pr["metric"].replace("3328 tokens", "3328 tokens per GPU"),
                                 "value": pr["value"], "unit": pr["unit"],
                                 "ms_per_step": pr["ms_per_step"], "steps": pa.steps, "n_ranks": world,
                                 "parallelism": pr["config"]["parallelism"], "scaling": "weak",
                                 "global_batch": pr["config"]["global_batch"],
                                 "ep_load": pr.get("ep_load"), "roofline": pr["roofline"],
                                 "collective": "NCCL send/recv all-to-all(v) per direction per layer" if world > 1
                                               else None}
    elif args.workload == "prefill":
        from ds_ocr_b200 import synth
        model = synth.Model()
        res = run_ours_prefill(args, rank, world, pg, model)
    elif args.workload == "prefill_full":
        from ds_ocr_b200 import synth
        model = synth.Model()
        res = run_ours_prefill_full(args, rank, world, pg, model)
    elif args.workload == "lm_head":
        res = run_ours_lmhead(args, rank, world, pg)
    elif args.workload == "decode64":
        from ds_ocr_b200 import synth
        model = synth.Model()
        prefixes = [synth.kv_prefix(model.d, PREFIX, stream=s) for s in range(MS_STREAMS)]
        ks, vs = prefixes[0]
        res = run_ours_decode_streams(args, rank, world, pg, model, prefixes)
    elif args.workload == "moe_layer_int8":
        res = run_ours_moe(args, rank, world, pg, int8=True)
    else:
        res = run_ours_moe(args, rank, world, pg)
    if rank != 0:
        return
    line = {"metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "dtype": res["dtype"],
            "config": res["config"], "e2e": res["e2e"], "roofline": res["roofline"], "clocks": res["clocks"],
            "gpu_launches": res["gpu_launches"]}
    for k in ("step_roofline", "dominant_kernel", "lm_head_roofline", "batch1", "ep_load", "ep_prefill"):
        if k in res:
            line[k] = res[k]
    line.update(common)
    if "scaling" in res:
        line["scaling"] = res["scaling"]
    if not args.no_cpu_baseline and world == 1:
        try:
            if args.workload in ("decode", "decode64"):
                v, n = ref_decode_time(model, ks, vs, T, args.cpu_budget, max_steps=64, sampling=sampling_of(args))
                sample = f"{n} {decode_mode(args)} ds_decoder_forward steps from position 663 (one stream; " \
                         "the reference decodes streams one at a time)"
            elif args.workload == "lm_head":
                v, n = ref_lmhead_time(T, args.cpu_budget)
                sample = f"{n} ds_argmax_matvec_bf16 calls (one per input)"
            elif args.workload == "prefill":
                v, n = ref_prefill_time(model, T, args.cpu_budget)
                sample = f"{n} of 11 MoE layers of the prefill block at 3328 tokens"
            elif args.workload == "prefill_full":
                v, n = ref_prefill_full_time(model, T)
                sample = f"one ds_decoder_prefill of the first {n} tokens (12 layers; the attention share grows " \
                         "with the length, so 3328 tokens run slower per token)"
            elif args.workload == "moe_layer_int8":
                wl = MoeLayerInt8Workload(n_layers=3)
                v, n = ref_moe_time(wl, T, args.cpu_budget, int8=True)
                sample = f"{n} single-token INT8 moe_forward calls over 3 layers quantised by the reference"
            else:
                wl = MoeLayerWorkload()
                v, n = ref_moe_time(wl, T, args.cpu_budget)
                sample = f"{n} single-token moe_forward calls over 11 layers"
            line["cpu_baseline"] = {"value": v, "unit": res["unit"], "cores": T, "kind": "reference",
                                    "sample": sample}
        except Exception as e:  # reported, never silently substituted
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
    if os.environ.get("WORLD_SIZE", "1") != "1":
        import torch.distributed as _dist
        if _dist.is_initialized():
            _dist.destroy_process_group()
