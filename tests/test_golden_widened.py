"""The oracle's widened rows against fixtures generated from the compiled
reference (tests/golden/make_golden.py, golden_widened.npz): LM-head
selection with sampling settings, the V3 sliding window, the whole prefill.
Runs without the reference tree."""
import os
import sys

import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden import PREFILL_ROWS, PREFILL_T, SELECT_CASES, SWA  # noqa: E402

G = np.load(os.path.join(HERE, "golden", "golden_widened.npz"))


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=2, vocab=4096)


@pytest.mark.parametrize("name", list(SELECT_CASES))
def test_selection(model, name):
    rp, ng, temp, _ = SELECT_CASES[name]
    ks, vs = synth.kv_prefix(model.d, 30)
    D = O.OracleDecoder(model, kv_max=64)
    D.load_kv(ks, vs)
    h = list(G[f"sel_{name}_hist0"])
    u = G[f"sel_{name}_u"]
    e = model.embed(7)
    for s, want in enumerate(G[f"sel_{name}_tok"]):
        _, fx, _ = D.step(e)
        tok, _, _ = D.select(fx, h, rp, ng, temp, float(u[s]) if temp > 0 else 0.0)
        assert tok == want, (name, s)
        h.append(tok)
        e = model.embed(tok)


def test_sliding_window(model):
    W, P, prefix, steps = SWA
    ks, vs = synth.kv_prefix(model.d, prefix)
    D = O.OracleDecoder(model, kv_max=64)
    D.load_kv(ks, vs)
    D.window, D.ref_len = W, P
    e = model.embed(5)
    for s, want in enumerate(G["swa_tok"]):
        tok, fx, _ = D.step(e)
        assert tok == want, s
        e = model.embed(tok)
    assert rel_l2(fx, G["swa_x_last"]) < 1e-4


def test_whole_prefill():
    m = synth.Model(n_layers=3, vocab=4096)
    D = O.OracleDecoder(m, kv_max=64)
    emb = np.stack([m.embed(t) for t in (np.arange(PREFILL_T) * 37 + 11) % m.d.vocab])
    tok, _, lg = D.prefill(emb)
    assert tok == int(G["pf_tok"])
    assert abs(lg - float(G["pf_logit"])) <= 1e-4 * max(1.0, abs(lg))
    rows = list(PREFILL_ROWS)
    for l in range(m.d.n_layers):
        assert rel_l2(D.k[l, rows], G["pf_k"][l]) < 1e-5, l
        assert rel_l2(D.v[l, rows], G["pf_v"][l]) < 1e-5, l
