"""How much the parity bar's gap rule leaves out of exact comparison. Router
indices are compared exactly where the 6th and 7th routing probabilities
differ by more than 1e-4, tokens where the top two logits differ by more
than 1e-4; everything else is compared within tolerance only. This measures
the excluded fraction on the benchmark input distributions (seeded as in
bench.py), from the oracle's values, and checks that it stays small.
Run with -s to see the fractions."""
import numpy as np
import pytest

import oracle as O
from ds_ocr_b200 import synth

GAP = 1e-4


def _probs(logits):
    z = logits - logits.max(axis=-1, keepdims=True)
    e = np.exp(z.astype(np.float64))
    return e / e.sum(axis=-1, keepdims=True)


def _router_gap_fraction(probs, k=6):
    p = np.sort(probs, axis=-1)[:, ::-1]
    return float(np.mean(p[:, k - 1] - p[:, k] <= GAP))


def test_router_gap_config0():
    # single-token MoE layer inputs: x N(0,1), RMSNorm with unit weights,
    # logits = xn . W_r^T (BF16 router N(0, 0.02))
    d = synth.Dims()
    W = synth.bf16_to_f32(synth.MoeWeights(d, 1).router)
    x = synth.normal_f32((2000, d.hidden), 11)
    xn = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + 1e-6)
    frac = _router_gap_fraction(_probs(xn @ W.T))
    print(f"\nrouter (config 0): {100 * frac:.2f}% of tokens within {GAP} at the 6th/7th probability")
    # the small random router (logits of std ~0.7) packs the probabilities
    # near 1/64, so about one token in twenty has a 6th/7th gap below 1e-4
    assert frac < 0.1


def test_router_gap_config4():
    # the prefill benchmark's overridden logits: N(0,1) + a per-expert bias
    d = synth.Dims()
    fr = []
    for l in range(1, 12):
        lg = synth.normal_f32((3328, d.n_experts), 600 + l)
        lg += 0.5 * synth.normal_f32(d.n_experts, 700 + l)[None, :]
        fr.append(_router_gap_fraction(_probs(lg)))
    frac = float(np.mean(fr))
    print(f"\nrouter (config 4, 11 layers x 3328 tokens): {100 * frac:.2f}% within {GAP}")
    assert frac < 0.05


def test_token_gap_lm_head_and_decode():
    o = O.oracle()
    # LM head inputs of the batch-64 benchmark
    W = synth.normal_bf16((129280, 1280), 300)
    X = synth.normal_f32((64, 1280), 2)
    y = np.empty(129280, np.float32)
    small = 0
    for x in X:
        o.orc_matvec_bf16(y.ctypes.data, x.ctypes.data, W.ctypes.data, 1280, 129280)
        t = np.partition(y, -2)[-2:]
        small += abs(t[1] - t[0]) <= GAP
    frac_lm = small / len(X)
    # greedy decode steps of a 3-layer model from a 40-token prefix
    m = synth.Model(n_layers=3, vocab=8192)
    dec = O.OracleDecoder(m, kv_max=128)
    ks, vs = synth.kv_prefix(m.d, 40)
    dec.load_kv(ks, vs)
    e = m.embed(7)
    yv = np.empty(m.d.vocab, np.float32)
    small_d, steps = 0, 24
    for _ in range(steps):
        tok, fx, _ = dec.step(e)
        o.orc_matvec_bf16(yv.ctypes.data, fx.ctypes.data, m.lm_head.ctypes.data, m.d.hidden, m.d.vocab)
        t = np.partition(yv, -2)[-2:]
        small_d += abs(t[1] - t[0]) <= GAP
        e = m.embed(tok)
    frac_d = small_d / steps
    print(f"\nLM head (config 1, 64 inputs): {100 * frac_lm:.2f}% within {GAP}; "
          f"decode steps: {100 * frac_d:.2f}% of {steps}")
    assert frac_lm < 0.05 and frac_d < 0.1
