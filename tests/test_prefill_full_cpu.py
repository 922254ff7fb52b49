"""The whole decoder prefill (ds_decoder_prefill, ds_moe_decoder.c:480-905):
the oracle restatement against the compiled reference on the same weights
and embeddings: every layer's K/V rows, the first generated token and its
logit, from an empty cache and after a prefix."""
import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth

pytestmark = pytest.mark.ref


@pytest.mark.parametrize("T,prefix", [(37, 0), (20, 15), (1, 9)])
def test_prefill_matches_reference(T, prefix):
    model = synth.Model(n_layers=3, vocab=4096)
    R = O.RefDecoder(model, kv_max=128, threads=4)
    D = O.OracleDecoder(model, kv_max=128)
    if prefix:
        ks, vs = synth.kv_prefix(model.d, prefix)
        R.load_kv(ks, vs)
        D.load_kv(ks, vs)
    emb = np.stack([model.embed(t) for t in (np.arange(T) * 37 + 11) % model.d.vocab])
    rt, rl = R.prefill(emb)
    ot, ox, ol = D.prefill(emb)
    for l in range(model.d.n_layers):
        rk, rv = R.kv(l, prefix, T)
        assert rel_l2(D.k[l, prefix:prefix + T], rk) < 1e-5, l
        assert rel_l2(D.v[l, prefix:prefix + T], rv) < 1e-5, l
    assert rt == ot
    assert abs(rl - ol) <= 1e-4 * max(1.0, abs(rl))
    # decoding continues from the prefilled cache identically
    e = model.embed(rt)
    for _ in range(3):
        a, _, _ = R.step(e)
        b, _, _ = D.step(e)
        assert a == b
        e = model.embed(a)
