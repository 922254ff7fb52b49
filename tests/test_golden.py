"""The CPU oracle against the golden vectors the reference itself produced
(tests/golden/make_golden.py). Runs without the reference tree or a GPU."""
import hashlib
import os

import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def test_fast_expf(orc):
    xs = synth.normal_f32(4096, synth.seed_of("golden", "fexp"), std=30.0)
    a = np.array([orc.orc_fast_expf(float(x)) for x in xs], np.float32)
    assert np.array_equal(a.view(np.uint32), G["fexp_out"].view(np.uint32))


def test_lm_head_argmax(orc):
    W = synth.normal_bf16((4099, 1280), synth.seed_of("golden", "lm"))
    X = synth.normal_f32((16, 1280), synth.seed_of("golden", "lm_x"))
    for i, x in enumerate(X):
        v = np.empty(1, np.float32)
        t = orc.orc_argmax_bf16(x.ctypes.data, W.ctypes.data, 1280, 4099, v.ctypes.data)
        if G["lm_gap"][i] > 1e-4:
            assert t == G["lm_tok"][i]
        assert abs(v[0] - G["lm_val"][i]) < 1e-4


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=2, vocab=4096)


def test_moe_layer(model):
    Xm = synth.normal_f32((8, 1280), synth.seed_of("golden", "moe_x"))
    for sim, tol in ((0, 1e-5), (1, 1e-3)):
        D = O.OracleDecoder(model, kv_max=64, simulate=sim)
        out = np.stack([D.moe_forward(1, x)[0] for x in Xm])
        assert rel_l2(out, G[f"moe_out_sim{sim}"]) < tol


def test_decode_steps(model):
    D = O.OracleDecoder(model, kv_max=128)
    ks, vs = synth.kv_prefix(model.d, 50)
    D.load_kv(ks, vs)
    e = model.embed(11)
    for i in range(5):
        t, fx, _ = D.step(e)
        assert t == G["dec_tok"][i]
        assert rel_l2(fx, G["dec_x"][i]) < 1e-4
        e = model.embed(t)


def test_prefill_moe(model):
    D = O.OracleDecoder(model, kv_max=64)
    xp = synth.normal_f32((16, 1280), synth.seed_of("golden", "prefill_x"))
    lg = synth.normal_f32((16, 64), synth.seed_of("golden", "prefill_logits"))
    for name, logits in (("ovr", lg), ("router", None)):
        x = xp.copy()
        idx, w = D.prefill_moe(1, x, logits)
        assert np.array_equal(idx, G[f"prefill_{name}_idx"])
        assert rel_l2(w, G[f"prefill_{name}_w"]) < 1e-5
        assert rel_l2(x - xp, G[f"prefill_{name}_x"] - xp) < 1e-5


def test_int8(model, orc):
    d = model.d
    mw = model.layers[1].moe
    q = synth.Int8Moe(d)
    H, I, S, E = d.hidden, d.moe_inter, d.shared_inter, d.n_experts
    for e in range(E):
        orc.orc_int8_quantize(mw.expert_gate_up(e).ctypes.data, 2 * I, H, q.gu_q[e * 2 * I * H:].ctypes.data,
                              q.gu_s[e * 2 * I:].ctypes.data, q.gu_o[e * 2 * I:].ctypes.data)
        orc.orc_int8_quantize(mw.expert_down(e).ctypes.data, H, I, q.dn_q[e * H * I:].ctypes.data,
                              q.dn_s[e * H:].ctypes.data, q.dn_o[e * H:].ctypes.data)
    orc.orc_int8_quantize(mw.shared_gate_up().ctypes.data, 2 * S, H, q.sgu_q.ctypes.data, q.sgu_s.ctypes.data,
                          q.sgu_o.ctypes.data)
    orc.orc_int8_quantize(mw.shared_down.ctypes.data, H, S, q.sdn_q.ctypes.data, q.sdn_s.ctypes.data,
                          q.sdn_o.ctypes.data)
    for name in ("gu_q", "gu_s", "gu_o", "dn_q", "dn_s", "dn_o", "sgu_q", "sgu_s", "sgu_o", "sdn_q", "sdn_s", "sdn_o"):
        assert hashlib.sha256(getattr(q, name).tobytes()).hexdigest() == str(G["int8_sha_" + name]), name
    mw.int8 = q
    try:
        D = O.OracleDecoder(model, kv_max=64)
        Xm = synth.normal_f32((8, 1280), synth.seed_of("golden", "moe_x"))
        out = np.stack([D.moe_forward(1, x, use_int8=True)[0] for x in Xm])
        assert rel_l2(out, G["int8_moe_out"]) < 1e-5
    finally:
        mw.int8 = None
