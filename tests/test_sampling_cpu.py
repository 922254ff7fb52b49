"""LM-head selection with the sampling settings (repetition penalty, n-gram
blocking, temperature): the oracle restatement against the compiled
reference's own ds_decoder_forward (ds_moe_decoder.c:1021-1263) driven
through its generation-loop history (ds_ocr.c:2245-2248)."""
import ctypes

import numpy as np
import pytest

from ds_ocr_b200 import synth
import oracle as O

pytestmark = pytest.mark.ref


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=2, vocab=4096)


def _top(model, fx, k):
    W = synth.bf16_to_f32(model.lm_head)
    lg = W @ fx
    return [int(t) for t in np.argsort(-lg, kind="stable")[:k]], lg


def _uniforms(seed, n):
    libc = ctypes.CDLL(None)
    libc.rand.restype = ctypes.c_int
    libc.srand(seed)
    rand_max = 2147483647
    return [np.float32(libc.rand()) / np.float32(rand_max) for _ in range(n)]


CASES = {
    # name: (repeat_penalty, ngram, temperature, history builder)
    "penalty": (1.5, 0, 0.0, lambda t: [t[0], t[1], t[0], t[2], t[3]]),
    "ngram_ban": (1.0, 3, 0.0, lambda t: [11, 12, t[0], 13, 14, 11, 12]),
    "penalty_and_ngram": (1.3, 3, 0.0, lambda t: [t[1], 12, t[0], 13, t[1], 12]),
    "temperature": (1.2, 0, 0.8, lambda t: [t[0], t[2]]),
    "temperature_ngram": (1.0, 2, 0.6, lambda t: [t[0], 5, t[0]]),
    # n-gram size 1: every history token is banned (empty prefix matches all)
    "ngram1": (1.0, 1, 0.0, lambda t: [t[0], t[1]]),
    # size 2 with the winner right after the last token's earlier occurrence
    "ngram2": (1.0, 2, 0.0, lambda t: [9, t[0], 4, 9]),
    # a strong penalty on all top tokens: penalised positives and negatives
    "penalty_strong": (4.0, 0, 0.0, lambda t: [t[0], t[1], t[2], t[3], 17, 18]),
}


@pytest.mark.parametrize("name", list(CASES))
def test_select_matches_reference(model, name):
    rp, ngram, temp, hist_of = CASES[name]
    d = model.d
    ks, vs = synth.kv_prefix(d, 30)
    # the first step's top tokens shape the history so that every rule bites
    probe = O.OracleDecoder(model, kv_max=64)
    probe.load_kv(ks, vs)
    _, fx0, _ = probe.step(model.embed(7))
    top, _ = _top(model, fx0, 4)
    hist = hist_of(top)

    R = O.RefDecoder(model, kv_max=64, threads=4)
    D = O.OracleDecoder(model, kv_max=64)
    R.load_kv(ks, vs)
    D.load_kv(ks, vs)
    R.set_sampling(rp, ngram, temp)
    R.set_history(hist)
    steps = 6
    us = _uniforms(4321, steps)
    O.ref().ref_srand(4321)
    h = list(hist)
    e = model.embed(7)
    fulls = 0
    for s in range(steps):
        rt = R.step_gen(e)
        _, fx, _ = D.step(e)
        ot, _, full = D.select(fx, h, rp, ngram, temp, us[s] if temp > 0 else 0.0)
        fulls += full
        assert rt == ot, (name, s, rt, ot)
        h.append(ot)
        e = model.embed(rt)
    assert list(R.history()) == h
    if name == "ngram_ban":
        assert fulls >= 1  # the banned greedy winner forced the full-logits path


def test_select_rules_by_hand(model):
    # direct checks of the rules on one hidden state
    D = O.OracleDecoder(model, kv_max=8)
    fx = synth.normal_f32(model.d.hidden, 99)
    top, lg = _top(model, fx, 3)
    t0, t1 = top[0], top[1]
    # no settings: plain argmax
    assert D.select(fx, [])[0] == t0
    # the fast path re-scores history tokens only: a penalised winner stays
    # the winner even when a token outside the history now scores higher
    # (ds_moe_decoder.c:1044-1066)
    assert lg[t0] > 0 and lg[t1] > 0
    rp = float(lg[t0] / lg[t1]) * 1.05
    tok, val, full = D.select(fx, [t0], rp)
    assert tok == t0 and not full and abs(val - lg[t0] / rp) < 1e-4
    # bans on other tokens keep the fast path: after (t0) came 9 and 8
    tok, _, full = D.select(fx, [t0, 9, t0, 8, t0], rp, 2, 0.0)
    assert not full and tok == t0
    # penalty applied once per history occurrence on the full path only
    tok, val, full = D.select(fx, [3, 4, 3], 1.0, 2, 0.0)  # prefix (3) seen before 4: 4 banned
    assert not full or tok != 4
    # the winner completes a seen bigram: full path, winner excluded
    tok, _, full = D.select(fx, [t0, t0 if t0 != 5 else 6, 9, t0], 1.0, 0, 0.0)
    assert tok == t0 and not full
    tok, _, full = D.select(fx, [9, t0, 2, 9], 1.0, 2, 0.0)
    assert full and tok == t1
