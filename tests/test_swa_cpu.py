"""V3's reference sliding-window decode attention (R-SWA): the oracle
restatement against the compiled reference's own ds_decoder_forward with
cfg->sliding_window_size and ctx->prefill_token_count set
(ds_moe_decoder.c:409-436, ds_kernels.c:2255-2314)."""
import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth

pytestmark = pytest.mark.ref


@pytest.mark.parametrize("window,ref_len,prefix", [
    (8, 20, 20),    # the window slides away from the reference rows after 8 steps
    (4, 12, 30),    # query already past the window: gap from the first step
    (64, 20, 20),   # window never leaves the reference rows: full causal
])
def test_rswa_decode_matches_reference(window, ref_len, prefix):
    model = synth.Model(n_layers=2, vocab=4096)
    ks, vs = synth.kv_prefix(model.d, prefix)
    R = O.RefDecoder(model, kv_max=64, threads=4)
    D = O.OracleDecoder(model, kv_max=64)
    R.load_kv(ks, vs)
    D.load_kv(ks, vs)
    R.set_window(window, ref_len)
    D.window, D.ref_len = window, ref_len
    e = model.embed(5)
    for s in range(14):
        rt, rx, _ = R.step(e)
        ot, ox, _ = D.step(e)
        assert rel_l2(ox, rx) < 1e-4, s
        assert rt == ot, s
        e = model.embed(rt)


def test_rswa_changes_the_result():
    # the window really drops rows: same inputs, full causal attention differs
    model = synth.Model(n_layers=2, vocab=4096)
    ks, vs = synth.kv_prefix(model.d, 30)
    a = O.OracleDecoder(model, kv_max=64)
    b = O.OracleDecoder(model, kv_max=64)
    a.load_kv(ks, vs)
    b.load_kv(ks, vs)
    b.window, b.ref_len = 4, 10
    _, xa, _ = a.step(model.embed(5))
    _, xb, _ = b.step(model.embed(5))
    assert rel_l2(xa, xb) > 1e-3
