"""Benchmark of the ds-ocr MoE-decoder hot path on B200.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                [--workload decode|moe_layer|lm_head]

Prints ONE JSON line (rank 0). Under torchrun (N > 1) every rank runs its own
independent replica of the workload (weak scaling: decode streams / tokens
are independent), timing is on the device with CUDA events, max over ranks.

Workloads (synthetic random-init weights):
  decode    config 3: greedy decode of the 12-layer DeepSeek3B-MoE decoder,
            batch 1, 662-token BF16 KV prefix        (headline)
  moe_layer config 0: one MoE layer, one token; steps rotate over 11 layers'
            weights (5.0 GB) so no step finds its experts in L2
  lm_head   config 1: argmax LM head 129280 x 1280, batch 1
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


def run_ours_moe(args, rank, world, pg):
    import torch
    from ds_ocr_b200 import cuda
    wl = MoeLayerWorkload()
    d = wl.d
    ctx = cuda.Context(0 if world == 1 else int(os.environ.get("LOCAL_RANK", "0")))
    lib = ctx.lib
    for mw in wl.layers:
        for a in (mw.router, mw.block, mw.down, mw.shared_down):
            ctx.register(a)
    dev = [(ctx.device_ptr(m.router), ctx.device_ptr(m.block), ctx.device_ptr(m.down), ctx.device_ptr(m.shared_down))
           for m in wl.layers]
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
    achieved = MOE_BYTES_PER_TOKEN / (ms_max / args.steps / 1e3) / 1e9
    pk = peaks()
    res["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                       "frac": achieved / pk["hbm_gbs"], "traffic": None,
                       "kernel": "moe layer (router + gate_up + down), 55,214,080 B/token",
                       "peak_source": pk["source"]}
    ctx.close()
    return res


def ref_moe_time(wl, threads, budget_s):
    """Times the reference's own moe_forward (compiled unmodified into
    oracle/_ref/libdsref.so) on the same layers and inputs, `threads` host
    threads, for about budget_s seconds of work. Returns (tokens/s, calls)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from ds_ocr_b200 import synth
    carrier = synth.Model.__new__(synth.Model)
    carrier.d = synth.Dims(n_layers=2, vocab=16)
    carrier.layers = []
    carrier.final_norm = np.ones(1280, np.float32)
    carrier.lm_head = np.zeros((16, 1280), np.uint16)
    R = O.RefDecoder(carrier, kv_max=8, threads=threads)
    n, t_total = 0, 0.0
    while t_total < budget_s:
        mw = wl.layers[n % len(wl.layers)]
        R.set_layer(1, mw)
        x = wl.X[n % wl.X.shape[0]]
        t = time.perf_counter()
        R.moe_forward(1, x)
        t_total += time.perf_counter() - t
        n += 1
    R.close()
    return n / t_total, n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="moe_layer", choices=["moe_layer"])
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of reference CPU work to time")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local, pg = dist_setup(args.gpus)

    if args.impl == "reference":
        if rank != 0:
            return
        wl = MoeLayerWorkload()
        T = cpu_threads()
        v, n = ref_moe_time(wl, T, max(args.cpu_budget, 1.0))
        line = {"impl": "reference", "metric": wl.metric, "value": v, "unit": wl.unit, "n_gpus": 0,
                "steps": n, "warmup": 1, "ms_per_step": 1e3 / v, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16 weights, f32 math", "data": "synthetic",
                "config": wl.config(),
                "cpu_baseline": {"value": v, "unit": wl.unit, "cores": T, "kind": "reference",
                                 "sample": f"{n} single-token moe_forward calls over 11 layers"},
                "e2e": {"value": v, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    res = run_ours_moe(args, rank, world, pg)
    if rank != 0:
        return
    line = {"metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": res["dtype"],
            "data": "synthetic (seeded random-init weights of the DeepSeek3B-MoE shapes)",
            "config": res["config"], "e2e": res["e2e"], "roofline": res["roofline"],
            "clocks": res["clocks"], "gpu_launches": res["gpu_launches"]}
    if not args.no_cpu_baseline:
        try:
            wl = MoeLayerWorkload()
            T = cpu_threads()
            v, n = ref_moe_time(wl, T, args.cpu_budget)
            line["cpu_baseline"] = {"value": v, "unit": res["unit"], "cores": T, "kind": "reference",
                                    "sample": f"{n} single-token moe_forward calls over 11 layers"}
        except Exception as e:  # reported, never silently substituted
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
