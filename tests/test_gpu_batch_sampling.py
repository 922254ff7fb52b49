"""The multi-stream decoder with the LM head's sampling settings and V3's
sliding-window attention (select.cu with a stream grid dimension, the SWA
attention kernel over streams; through the C ABI), each stream against its
own oracle decoder (pinned to the reference's decoder step in
test_sampling_cpu.py and test_swa_cpu.py): the final hidden state within
1e-3 relative L2 and the selected token equal."""
import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth
from ds_ocr_b200.cuda import DsCudaError
from ds_ocr_b200.decoder import BatchDecoder

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=3, vocab=8192)


def _top(model, fx, k):
    lg = synth.bf16_to_f32(model.lm_head) @ fx
    return [int(t) for t in np.argsort(-lg, kind="stable")[:k]]


def _gap(model, fx):
    t = np.sort(synth.bf16_to_f32(model.lm_head) @ fx)[-2:]
    return t[1] - t[0]


# (repeat_penalty, ngram, temperature): the settings are shared by the
# streams, each stream has its own history
SETTINGS = {
    "penalty": (1.5, 0, 0.0),
    "ngram_ban": (1.0, 3, 0.0),
    "penalty_and_ngram": (1.3, 3, 0.0),
    "temperature": (1.2, 0, 0.8),
    "temperature_ngram": (1.0, 2, 0.6),
}


def _history(s, top):
    # a different history shape per stream: penalised winners, an n-gram
    # that the first step's winner would complete, or nothing
    kind = s % 4
    if kind == 0:
        return [top[0], top[1], top[0], top[2]]
    if kind == 1:
        return [11, 12, top[0], 13, 14, 11, 12]
    if kind == 2:
        return [top[1], 12, top[0], 13, top[1], 12]
    return []


@pytest.mark.parametrize("S", [4, 64])
@pytest.mark.parametrize("name", list(SETTINGS))
def test_batch_selection_matches_oracle(cuda_ctx, model, name, S):
    rp, ngram, temp = SETTINGS[name]
    if S == 64 and name not in ("penalty_and_ngram", "temperature"):
        pytest.skip("64 streams: two settings cover the many-stream launch shapes")
    kv_max, steps = 256, 6
    check = range(S) if S <= 4 else (0, 1, 2, 3, 37, 63)
    prefixes = [synth.kv_prefix(model.d, 20 + 9 * s % 50, stream=s + 1) for s in range(S)]
    first = [(7 + 13 * s) % model.d.vocab for s in range(S)]
    bd = BatchDecoder(model, S, cuda_ctx, kv_max=kv_max)
    try:
        oras, hists = {}, {}
        for s in range(S):
            bd.load_kv(s, *prefixes[s])
        for s in check:
            probe = O.OracleDecoder(model, kv_max=kv_max)
            probe.load_kv(*prefixes[s])
            _, fx0, _ = probe.step(model.embed(first[s]))
            hists[s] = _history(s, _top(model, fx0, 4))
            o = O.OracleDecoder(model, kv_max=kv_max)
            o.load_kv(*prefixes[s])
            oras[s] = o
        u = np.random.default_rng(S).random((S, steps)).astype(np.float32)
        bd.set_sampling(rp, ngram, temp)
        for s in range(S):
            bd.set_history(s, hists.get(s, []))
        if temp > 0:
            bd.set_uniforms(u)
        h = {s: list(hists[s]) for s in check}
        E = np.stack([model.embed(t) for t in first])
        for step in range(steps):
            toks, fx = bd.forward(E, want_x=True)
            for s in check:
                _, ofx, _ = oras[s].step(E[s])
                assert rel_l2(fx[s], ofx) < 1e-3, (name, step, s)
                otok, _, _ = oras[s].select(fx[s], h[s], rp, ngram, temp, float(u[s, step]) if temp > 0 else 0.0)
                assert toks[s] == otok, (name, step, s, toks[s], otok)
                h[s].append(otok)
            E = np.stack([model.embed(int(t)) for t in toks])
        for s in check:
            assert list(bd.history(s)) == h[s], s
    finally:
        bd.close()


def test_batch_generate_dev_matches_forward_with_sampling(cuda_ctx, model):
    # the captured step graph runs the same selection as host-driven steps
    S, n = 8, 6
    u = np.random.default_rng(3).random((S, n + 1)).astype(np.float32)
    runs = []
    for mode in ("forward", "dev"):
        bd = BatchDecoder(model, S, cuda_ctx, kv_max=128)
        try:
            for s in range(S):
                bd.load_kv(s, *synth.kv_prefix(model.d, 20 + s, stream=s + 1))
                bd.set_history(s, [3 + s, 4])
            bd.set_sampling(1.3, 2, 0.7)
            bd.set_uniforms(u)
            E = np.stack([model.embed(3 + s) for s in range(S)])
            if mode == "forward":
                seq = [bd.forward(E)] + [bd.forward() for _ in range(n)]
                last = seq[-1]
            else:
                bd.forward(E)
                bd.generate_dev(n - 1)
                cuda_ctx.synchronize()
                last = bd.forward()
            runs.append((last, [list(bd.history(s)) for s in range(S)]))
        finally:
            bd.close()
    assert np.array_equal(runs[0][0], runs[1][0])
    assert runs[0][1] == runs[1][1]


def test_batch_uniform_and_setting_checks(cuda_ctx, model):
    S = 2
    bd = BatchDecoder(model, S, cuda_ctx, kv_max=64)
    try:
        for s in range(S):
            bd.load_kv(s, *synth.kv_prefix(model.d, 10, stream=s + 1))
        bd.set_sampling(1.0, 0, 0.5)
        bd.set_uniforms(np.full((S, 1), 0.5, np.float32))
        bd.forward(np.stack([model.embed(1)] * S))
        with pytest.raises(DsCudaError):
            bd.forward()  # no uniform left
        bd.set_sampling(1.0, 0, 0.0)  # greedy again: the history keeps growing
        toks, fx = bd.forward(want_x=True)
        for s in range(S):
            assert toks[s] == O.OracleDecoder(model, kv_max=8).select(fx[s], [])[0]
            assert len(bd.history(s)) == 2
        with pytest.raises(DsCudaError):
            bd.set_sampling(0.0, 0, 0.0)
    finally:
        bd.close()


@pytest.mark.parametrize("window,refs,prefixes,steps", [
    (8, [40, 30, 12], [40, 30, 12], 14),        # the window leaves the reference rows
    (16, [100, 250, 5], [300, 260, 200], 10),   # gaps of different lengths per stream
    (600, [40, 40, 40], [40, 50, 60], 4),       # the window never leaves: full causal
])
def test_batch_swa_matches_oracle(cuda_ctx, model, window, refs, prefixes, steps):
    S = len(refs)
    kv = [synth.kv_prefix(model.d, p, stream=s + 1) for s, p in enumerate(prefixes)]
    bd = BatchDecoder(model, S, cuda_ctx, kv_max=1024)
    try:
        oras = []
        for s in range(S):
            bd.load_kv(s, *kv[s])
            o = O.OracleDecoder(model, kv_max=1024)
            o.load_kv(*kv[s])
            o.window, o.ref_len = window, refs[s]
            oras.append(o)
        bd.set_window(window, refs)
        E = np.stack([model.embed(9 + s) for s in range(S)])
        compared = 0
        for step in range(steps):
            toks, fx = bd.forward(E, want_x=True)
            nxt = []
            for s in range(S):
                otok, ofx, _ = oras[s].step(E[s])
                assert rel_l2(fx[s], ofx) < 1e-3, (step, s)
                if _gap(model, ofx) > 1e-4:
                    assert toks[s] == otok, (step, s)
                    compared += 1
                nxt.append(model.embed(otok))
            E = np.stack(nxt)
        assert compared >= S * steps // 2
    finally:
        bd.close()
