"""Generates tests/golden/golden.npz and golden_widened.npz from the REFERENCE ITSELF (its own C
sources compiled unmodified into oracle/_ref/libdsref.so; run `make -C
oracle ref` first, which needs the reference tree).

Inputs are not stored: they are regenerated from their seeds by
ds_ocr_b200.synth (counter-based, machine-independent), so the fixture holds
only the reference's outputs. Usage: python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402
from ds_ocr_b200 import synth  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
OUT_WIDENED = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_widened.npz")

# selection cases of golden_widened.npz: (repeat_penalty, n-gram size,
# temperature, history builder from the first step's top-4 tokens)
SELECT_CASES = {
    "penalty": (1.5, 0, 0.0, lambda t: [t[0], t[1], t[0], t[2], t[3]]),
    "ngram_ban": (1.0, 3, 0.0, lambda t: [11, 12, t[0], 13, 14, 11, 12]),
    "temperature": (1.2, 0, 0.8, lambda t: [t[0], t[2]]),
}
SWA = (8, 20, 20, 14)     # window, prefill length, KV prefix, steps
PREFILL_T = 37
PREFILL_ROWS = (0, 5, 36)  # K/V rows kept of every layer


def main():
    r = O.ref()
    r.ref_set_threads(4)
    g = {}
    # 1. fast exp (Schraudolph, FMA-contracted) on a fixed grid
    xs = synth.normal_f32(4096, synth.seed_of("golden", "fexp"), std=30.0)
    g["fexp_out"] = np.array([r.ref_fast_expf(float(x)) for x in xs], np.float32)
    # 2. LM-head argmax: W [4099 x 1280], 16 inputs
    W = synth.normal_bf16((4099, 1280), synth.seed_of("golden", "lm"))
    X = synth.normal_f32((16, 1280), synth.seed_of("golden", "lm_x"))
    toks, vals, logits = [], [], []
    for x in X:
        v = np.empty(1, np.float32)
        toks.append(r.ref_argmax(x.ctypes.data, W.ctypes.data, 1280, 4099, v.ctypes.data))
        vals.append(v[0])
        y = np.empty(4099, np.float32)
        r.ref_matvec(y.ctypes.data, x.ctypes.data, W.ctypes.data, 1280, 4099)
        logits.append(y)
    top2 = np.sort(np.stack(logits), axis=1)[:, -2:]
    g["lm_tok"], g["lm_val"], g["lm_gap"] = np.array(toks, np.int32), np.array(vals, np.float32), top2[:, 1] - top2[:, 0]
    # 3. full MoE layer (64 experts + shared), BF16, both truncation modes, then INT8
    model = synth.Model(n_layers=2, vocab=4096)
    R = O.RefDecoder(model, kv_max=128, threads=4)
    Xm = synth.normal_f32((8, 1280), synth.seed_of("golden", "moe_x"))
    for sim in (0, 1):
        r.ref_set_simulate(sim)
        g[f"moe_out_sim{sim}"] = np.stack([R.moe_forward(1, x) for x in Xm])
    r.ref_set_simulate(0)
    # 4. decode: 2-layer model (dense + MoE), 50-token KV prefix, 5 greedy steps
    ks, vs = synth.kv_prefix(model.d, 50)
    R.load_kv(ks, vs)
    e = model.embed(11)
    toks, fxs = [], []
    for _ in range(5):
        t, fx, _ = R.step(e)
        toks.append(t)
        fxs.append(fx)
        e = model.embed(t)
    g["dec_tok"], g["dec_x"] = np.array(toks, np.int32), np.stack(fxs)
    # 5. prefill MoE block, 32 tokens, router logits overridden, then real router
    xp = synth.normal_f32((16, 1280), synth.seed_of("golden", "prefill_x"))
    lg = synth.normal_f32((16, 64), synth.seed_of("golden", "prefill_logits"))
    for name, logits in (("ovr", lg), ("router", None)):
        x = xp.copy()
        idx, w = R.prefill_moe(1, x, logits)
        g[f"prefill_{name}_x"], g[f"prefill_{name}_idx"], g[f"prefill_{name}_w"] = x, idx, w
    # 6. INT8 (--int4): quantisation checksums and the INT8 MoE layer
    R.quantize()
    q = model.layers[1].moe.int8
    for name in ("gu_q", "gu_s", "gu_o", "dn_q", "dn_s", "dn_o", "sgu_q", "sgu_s", "sgu_o", "sdn_q", "sdn_s", "sdn_o"):
        g["int8_sha_" + name] = np.array(hashlib.sha256(getattr(q, name).tobytes()).hexdigest())
    g["int8_gu_s_e0"], g["int8_gu_o_e0"] = q.gu_s[:1792].copy(), q.gu_o[:1792].copy()
    g["int8_moe_out"] = np.stack([R.moe_forward(1, x) for x in Xm])
    np.savez_compressed(OUT, **g)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


def _top4(model, fx):
    lg = synth.bf16_to_f32(model.lm_head) @ fx
    return [int(t) for t in np.argsort(-lg, kind="stable")[:4]]


def widened():
    """The rows added to the decode step: LM-head selection with sampling
    settings (ds_moe_decoder.c:1021-1263), the V3 sliding window
    (:409-436) and the whole prefill (:480-905), from the reference."""
    import ctypes
    r = O.ref()
    g = {}
    model = synth.Model(n_layers=2, vocab=4096)
    ks, vs = synth.kv_prefix(model.d, 30)
    probe = O.OracleDecoder(model, kv_max=64)
    probe.load_kv(ks, vs)
    _, fx0, _ = probe.step(model.embed(7))
    top = _top4(model, fx0)
    libc = ctypes.CDLL(None)
    for name, (rp, ng, temp, hist_of) in SELECT_CASES.items():
        R = O.RefDecoder(model, kv_max=64, threads=4)
        R.load_kv(ks, vs)
        R.set_sampling(rp, ng, temp)
        R.set_history(hist_of(top))
        libc.srand(4321)
        us = np.array([libc.rand() / 2147483647.0 for _ in range(6)], np.float32)
        r.ref_srand(4321)
        e, toks = model.embed(7), []
        for _ in range(6):
            t = R.step_gen(e)
            toks.append(t)
            e = model.embed(t)
        g[f"sel_{name}_tok"], g[f"sel_{name}_u"] = np.array(toks, np.int32), us
        g[f"sel_{name}_hist0"] = np.array(hist_of(top), np.int32)
        R.close()
    W, P, prefix, steps = SWA
    ks2, vs2 = synth.kv_prefix(model.d, prefix)
    R = O.RefDecoder(model, kv_max=64, threads=4)
    R.load_kv(ks2, vs2)
    R.set_window(W, P)
    e, toks, xs = model.embed(5), [], []
    for _ in range(steps):
        t, fx, _ = R.step(e)
        toks.append(t)
        xs.append(fx)
        e = model.embed(t)
    g["swa_tok"], g["swa_x_last"] = np.array(toks, np.int32), xs[-1]
    R.close()
    m3 = synth.Model(n_layers=3, vocab=4096)
    R = O.RefDecoder(m3, kv_max=64, threads=4)
    emb = np.stack([m3.embed(t) for t in (np.arange(PREFILL_T) * 37 + 11) % m3.d.vocab])
    t, lg = R.prefill(emb)
    g["pf_tok"], g["pf_logit"] = np.array(t, np.int32), np.array(lg, np.float32)
    rows = list(PREFILL_ROWS)
    g["pf_k"] = np.stack([R.kv(l, 0, PREFILL_T)[0][rows] for l in range(m3.d.n_layers)])
    g["pf_v"] = np.stack([R.kv(l, 0, PREFILL_T)[1][rows] for l in range(m3.d.n_layers)])
    R.close()
    np.savez_compressed(OUT_WIDENED, **g)
    print("wrote", OUT_WIDENED, os.path.getsize(OUT_WIDENED), "bytes")


if __name__ == "__main__":
    if "--widened" in sys.argv:
        widened()
    else:
        main()
        widened()
