"""LM-head selection with the sampling settings on the GPU (select.cu,
through the C ABI) against the oracle restatement (pinned to the reference's
ds_decoder_forward in test_sampling_cpu.py): repetition penalty, n-gram
blocking (fast path and the full-logits fallback), temperature sampling
with supplied uniforms, the device-kept history, and the host checks."""
import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth
from ds_ocr_b200.cuda import DsCudaError
from ds_ocr_b200.decoder import Decoder

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=3, vocab=8192)


def _top(model, fx, k):
    lg = synth.bf16_to_f32(model.lm_head) @ fx
    return [int(t) for t in np.argsort(-lg, kind="stable")[:k]]


CASES = {
    # name: (repeat_penalty, ngram, temperature, history builder from the first step's top tokens)
    "greedy_history_only": (1.0, 0, 0.0, lambda t: [t[0], t[1]]),
    "penalty": (1.5, 0, 0.0, lambda t: [t[0], t[1], t[0], t[2], t[3]]),
    "penalty_strong": (3.0, 0, 0.0, lambda t: [t[1], t[0], t[2]]),
    "ngram_ban": (1.0, 3, 0.0, lambda t: [11, 12, t[0], 13, 14, 11, 12]),
    "penalty_and_ngram": (1.3, 3, 0.0, lambda t: [t[1], 12, t[0], 13, t[1], 12]),
    "temperature": (1.2, 0, 0.8, lambda t: [t[0], t[2]]),
    "temperature_ngram": (1.0, 2, 0.6, lambda t: [t[0], 5, t[0]]),
}


@pytest.mark.parametrize("name", list(CASES))
def test_selection_matches_oracle(cuda_ctx, model, name):
    rp, ngram, temp, hist_of = CASES[name]
    ks, vs = synth.kv_prefix(model.d, 40)
    ora = O.OracleDecoder(model, kv_max=128)
    ora.load_kv(ks, vs)
    dec = Decoder(model, cuda_ctx, kv_max=128)
    try:
        dec.load_kv(ks, vs)
        probe = O.OracleDecoder(model, kv_max=128)
        probe.load_kv(ks, vs)
        _, fx0, _ = probe.step(model.embed(7))
        hist = hist_of(_top(model, fx0, 4))
        steps = 8
        u = np.random.default_rng(5).random(steps).astype(np.float32)
        dec.set_sampling(rp, ngram, temp)
        dec.set_history(hist)
        if temp > 0:
            dec.set_uniforms(u)
        h = list(hist)
        e = model.embed(7)
        for s in range(steps):
            tok, fx, val = dec.forward(e, want_x=True)
            _, ofx, _ = ora.step(e)
            assert rel_l2(fx, ofx) < 1e-3, (name, s)
            # the selection rules on the GPU's own hidden state
            otok, oval, _ = ora.select(fx, h, rp, ngram, temp, float(u[s]) if temp > 0 else 0.0)
            assert tok == otok, (name, s, tok, otok)
            if temp <= 0:
                assert abs(val - oval) <= 1e-4 * max(1.0, abs(oval)), (name, s, val, oval)
            h.append(otok)
            e = model.embed(tok)
        assert list(dec.history()) == h
    finally:
        dec.close()


def test_generate_matches_forward_with_sampling(cuda_ctx, model):
    # the device-looped generate follows the same history as host-driven steps
    ks, vs = synth.kv_prefix(model.d, 30)
    a = Decoder(model, cuda_ctx, kv_max=128)
    b = Decoder(model, cuda_ctx, kv_max=128)
    try:
        u = np.random.default_rng(9).random(12).astype(np.float32)
        for d in (a, b):
            d.load_kv(ks, vs)
            d.set_sampling(1.3, 2, 0.7)
            d.set_history([3, 4])
            d.set_uniforms(u)
        host = []
        e = model.embed(7)
        for _ in range(12):
            t = a.forward(e)
            host.append(t)
            e = model.embed(t)
        dev = b.generate(12, first_embed=model.embed(7))
        assert list(dev) == host
        assert list(a.history()) == [3, 4] + host == list(b.history())
    finally:
        a.close()
        b.close()


def test_uniforms_and_engine_checks(cuda_ctx, model):
    ks, vs = synth.kv_prefix(model.d, 10)
    dec = Decoder(model, cuda_ctx, kv_max=64)
    try:
        dec.load_kv(ks, vs)
        dec.set_sampling(1.0, 0, 0.5)
        dec.set_uniforms(np.array([0.25, 0.75], np.float32))
        dec.generate(2, first_embed=model.embed(1))
        with pytest.raises(DsCudaError):
            dec.forward(model.embed(1))  # no uniform left
        # back to greedy: the history keeps growing, the token is the argmax
        dec.set_sampling(1.0, 0, 0.0)
        n0 = len(dec.history())
        tok, fx, _ = dec.forward(model.embed(2), want_x=True)
        assert tok == O.OracleDecoder(model, kv_max=8).select(fx, [])[0]
        assert len(dec.history()) == n0 + 1
    finally:
        dec.close()
    per = Decoder(model, cuda_ctx, kv_max=64, engine=1)
    try:
        with pytest.raises(DsCudaError):
            per.set_sampling(1.2, 0, 0.0)
        per.set_sampling(1.0, 0, 0.0)  # greedy stays allowed
    finally:
        per.close()
