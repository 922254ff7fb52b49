"""Per-kernel live timeline of the decode step, from the library's optional
launch trace (globaltimer ns written by every CTA of the instrumented
kernels: entry, past the dependency wait, exit). A kernel launch's share of
the step is its critical-path time: its last CTA's exit minus the previous
launch's last exit, so overlapped prologues are not counted twice."""
import ctypes

import numpy as np

from . import _lib

KINDS = {1: "qkv_rope_kernel", 2: "attention", 3: "matvec_res_kernel (O-proj)", 4: "router tail",
         5: "matvec_long_kernel", 6: "moe_gate_up_kernel", 7: "moe_down_kernel", 8: "argmax_tma_kernel (LM head)",
         9: "decode_advance_kernel", 10: "moe_step_kernel", 11: "dense_step_kernel"}
TAGS = ("decode", "moe", "stream", "step", "attn2")
WORDS = 12


def _setters(lib):
    out = []
    for t in TAGS:
        f = getattr(lib, f"ds_trace_set_{t}", None)
        if f is not None:
            f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint]
            f.restype = ctypes.c_int
            out.append(f)
    return out


def capture(run, cap=1 << 18):
    """Runs run() with the trace on; returns launches in start order:
    dicts with kind, start, wait (last CTA past the wait), end, crit (ns)."""
    import torch
    lib = _lib.load()
    rec = torch.zeros(cap * WORDS, dtype=torch.int64, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    sets = _setters(lib)
    torch.cuda.synchronize()
    for f in sets:
        if f(rec.data_ptr(), cnt.data_ptr(), cap) != 0:
            raise RuntimeError("trace buffer could not be set")
    try:
        run()
        torch.cuda.synchronize()
    finally:
        for f in sets:
            f(None, None, 0)
    n = min(int(cnt.item()), cap)
    r = rec[: WORDS * n].view(n, WORDS).cpu().numpy().astype(np.int64)
    r = r[np.argsort(r[:, 1])]
    launches, cur = [], {}
    for k, a, w, b in zip(r[:, 0] & 0xffff, r[:, 1], r[:, 2], r[:, 3]):
        L = cur.get(k)
        if L is None or a > L["end"]:
            L = {"kind": int(k), "start": a, "wait": 0, "end": b}
            launches.append(L)
            cur[k] = L
        L["end"] = max(L["end"], b)
        L["wait"] = max(L["wait"], w)
    launches.sort(key=lambda L: L["start"])
    prev = launches[0]["start"] if launches else 0
    for L in launches:
        L["crit"] = L["end"] - prev
        prev = max(prev, L["end"])
    return launches


def summary(launches, steps):
    """Per kind: launches per step, mean critical-path us per launch, share."""
    tot = sum(L["crit"] for L in launches)
    out = {}
    for k in sorted({L["kind"] for L in launches}):
        c = [L["crit"] for L in launches if L["kind"] == k]
        out[KINDS.get(k, str(k))] = {"launches_per_step": len(c) / steps, "us_per_launch": float(np.mean(c)) / 1e3,
                                     "share": float(sum(c)) / tot if tot else 0.0}
    return out
