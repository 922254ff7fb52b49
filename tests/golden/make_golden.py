"""Generates tests/golden/golden.npz from the REFERENCE ITSELF (its own C
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


if __name__ == "__main__":
    main()
