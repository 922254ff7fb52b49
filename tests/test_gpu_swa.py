"""V3's reference sliding-window decode attention on the GPU (the SWA
instantiation of attn_decode_kernel, through the C ABI) against the oracle,
which is pinned to the reference's decoder step in test_swa_cpu.py."""
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


def logit_gap(model, fx):
    t = np.sort(synth.bf16_to_f32(model.lm_head) @ fx)[-2:]
    return t[1] - t[0]


@pytest.mark.parametrize("window,ref_len,prefix,steps", [
    (8, 40, 40, 16),      # the window leaves the reference rows after 8 steps
    (16, 100, 300, 12),   # a gap of ~190 rows from the first step, across cluster CTAs
    (600, 40, 40, 6),     # window never leaves: full causal
    (5, 700, 700, 10),    # long reference range, short window
])
def test_swa_decode_matches_oracle(cuda_ctx, model, window, ref_len, prefix, steps):
    ks, vs = synth.kv_prefix(model.d, prefix)
    dec = Decoder(model, cuda_ctx, kv_max=1024)
    ora = O.OracleDecoder(model, kv_max=1024)
    try:
        dec.load_kv(ks, vs)
        ora.load_kv(ks, vs)
        dec.set_window(window, ref_len)
        ora.window, ora.ref_len = window, ref_len
        e = model.embed(9)
        compared = 0
        for s in range(steps):
            tok, fx, _ = dec.forward(e, want_x=True)
            otok, ofx, _ = ora.step(e)
            assert rel_l2(fx, ofx) < 1e-3, s
            if logit_gap(model, ofx) > 1e-4:
                assert tok == otok, s
                compared += 1
            e = model.embed(otok)
        assert compared >= steps // 2
        # device-looped steps take the same path
        dev = Decoder(model, cuda_ctx, kv_max=1024)
        try:
            dev.load_kv(ks, vs)
            dev.set_window(window, ref_len)
            toks = dev.generate(4, first_embed=model.embed(9))
            host = Decoder(model, cuda_ctx, kv_max=1024)
            host.load_kv(ks, vs)
            host.set_window(window, ref_len)
            e = model.embed(9)
            for t in toks:
                h = host.forward(e)
                assert h == t
                e = model.embed(h)
            host.close()
        finally:
            dev.close()
    finally:
        dec.close()


def test_swa_persistent_engine_rejected(cuda_ctx, model):
    per = Decoder(model, cuda_ctx, kv_max=64, engine=1)
    try:
        with pytest.raises(DsCudaError):
            per.set_window(8, 10)
        per.set_window(0, 0)
    finally:
        per.close()
