"""The whole-decoder prefill on the GPU (ds_cuda_decoder_prefill, through
the C ABI) against the oracle (pinned to the reference's ds_decoder_prefill
in test_prefill_full_cpu.py): every layer's K/V rows within 1e-3 relative
L2, the first token bit-exact where the top-2 logit gap exceeds 1e-4, and
decoding that continues from the prefilled cache."""
import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth
from ds_ocr_b200.decoder import Decoder

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=3, vocab=8192)


def gap(model, fx):
    t = np.sort(synth.bf16_to_f32(model.lm_head) @ fx)[-2:]
    return t[1] - t[0]


@pytest.mark.parametrize("T,prefix", [(37, 0), (20, 15), (1, 9), (300, 0), (129, 64)])
def test_prefill_matches_oracle(cuda_ctx, model, T, prefix):
    dec = Decoder(model, cuda_ctx, kv_max=1024)
    ora = O.OracleDecoder(model, kv_max=1024)
    try:
        if prefix:
            ks, vs = synth.kv_prefix(model.d, prefix)
            dec.load_kv(ks, vs)
            ora.load_kv(ks, vs)
        emb = np.stack([model.embed(t) for t in (np.arange(T) * 37 + 11) % model.d.vocab])
        tok, fx, lg = dec.prefill(emb, want_x=True)
        otok, ofx, olg = ora.prefill(emb)
        assert dec.length == prefix + T
        for l in range(model.d.n_layers):
            k, v = dec.kv(l, prefix, T)
            assert rel_l2(k, ora.k[l, prefix:prefix + T]) < 1e-3, l
            assert rel_l2(v, ora.v[l, prefix:prefix + T]) < 1e-3, l
        assert rel_l2(fx, ofx) < 1e-3
        if gap(model, ofx) > 1e-4:
            assert tok == otok
        # decoding continues: the device loop consumes the staged embedding
        toks = dec.generate(4)
        e = model.embed(otok)
        for s in range(4):
            ot, ox, _ = ora.step(e)
            if gap(model, ox) > 1e-4:
                assert toks[s] == ot, s
            e = model.embed(ot)
        assert list(dec.history())[:1] == [tok]
    finally:
        dec.close()


def test_long_prefill_takes_the_large_query_blocks(cuda_ctx, model):
    # 2000 tokens x 10 heads: enough 128-query blocks to fill the SMs, so the
    # large-tile attention kernel runs (shorter prefills use 32-query blocks)
    T = 2000
    dec = Decoder(model, cuda_ctx, kv_max=2048)
    ora = O.OracleDecoder(model, kv_max=2048)
    try:
        emb = np.stack([model.embed(t) for t in (np.arange(T) * 53 + 5) % model.d.vocab])
        tok, fx, _ = dec.prefill(emb, want_x=True)
        otok, ofx, _ = ora.prefill(emb)
        assert rel_l2(fx, ofx) < 1e-3
        for l in range(model.d.n_layers):
            k, v = dec.kv(l, 0, T)
            assert rel_l2(k, ora.k[l, :T]) < 1e-3 and rel_l2(v, ora.v[l, :T]) < 1e-3, l
        if gap(model, ofx) > 1e-4:
            assert tok == otok
    finally:
        dec.close()


def test_prefill_dense_and_moe_layers_full_size(cuda_ctx):
    # the full 12-layer model (dense layer 0 + 11 MoE layers), 200 tokens
    m = synth.Model()
    dec = Decoder(m, cuda_ctx, kv_max=512)
    ora = O.OracleDecoder(m, kv_max=512)
    try:
        emb = np.stack([m.embed(t) for t in (np.arange(200) * 101 + 3) % m.d.vocab])
        tok, fx, _ = dec.prefill(emb, want_x=True)
        otok, ofx, _ = ora.prefill(emb)
        assert rel_l2(fx, ofx) < 1e-3
        for l in (0, 1, 11):
            k, v = dec.kv(l, 0, 200)
            assert rel_l2(k, ora.k[l, :200]) < 1e-3 and rel_l2(v, ora.v[l, :200]) < 1e-3, l
        if gap(m, ofx) > 1e-4:
            assert tok == otok
    finally:
        dec.close()
