"""Decoder weights from a safetensors checkpoint (csrc/ingest.cu, through
the C ABI): the checkpoint-built decoder against the decoder built from the
same arrays (bit-identical results), one file and shards, BF16 and F32
norms, separate token embeddings in the device decode loop, tied LM head,
INT8 quantised on the device, and the loader's errors."""
import numpy as np
import pytest

from ds_ocr_b200 import synth
from ds_ocr_b200.cuda import DsCudaError
from ds_ocr_b200.decoder import Decoder, quantize_int8
from st_checkpoint import decoder_tensors, write_checkpoint, write_safetensors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    return synth.Model(n_layers=3, vocab=8192)


def _steps(dec, model, n, first=7, embed_of=None):
    embed_of = embed_of or model.embed
    out, e = [], embed_of(first)
    for _ in range(n):
        tok, fx, lg = dec.forward(e, want_x=True)
        out.append((tok, fx.copy(), lg))
        e = embed_of(tok)
    return out


@pytest.mark.parametrize("shards,norm", [(1, "BF16"), (2, "F32")])
def test_checkpoint_matches_arrays(cuda_ctx, tmp_path, model, shards, norm):
    write_checkpoint(model, str(tmp_path), shards=shards, norm_dtype=norm)
    ks, vs = synth.kv_prefix(model.d, 30)
    a = Decoder(model, cuda_ctx, kv_max=256)
    b = Decoder.from_safetensors(tmp_path, model.d, cuda_ctx, kv_max=256)
    try:
        for d in (a, b):
            d.load_kv(ks, vs)
        ra, rb = _steps(a, model, 5), _steps(b, model, 5)
        for (ta, xa, la), (tb, xb, lb) in zip(ra, rb):
            assert ta == tb and la == lb
            assert np.array_equal(xa, xb)
    finally:
        a.close()
        b.close()


def test_separate_embeddings_feed_the_device_loop(cuda_ctx, tmp_path, model):
    # embed_tokens differs from lm_head: generate() must take the next input
    # from embed_tokens (the reference's tok_embeddings_bf16)
    emb = synth.normal_bf16((model.d.vocab, model.d.hidden), 4242)
    write_checkpoint(model, str(tmp_path), embed=emb)
    ks, vs = synth.kv_prefix(model.d, 20)
    embed_of = lambda t: synth.bf16_to_f32(emb[t]).copy()
    host = Decoder.from_safetensors(tmp_path, model.d, cuda_ctx, kv_max=128)
    dev = Decoder.from_safetensors(tmp_path, model.d, cuda_ctx, kv_max=128)
    try:
        host.load_kv(ks, vs)
        dev.load_kv(ks, vs)
        want = [t for t, _, _ in _steps(host, model, 6, embed_of=embed_of)]
        got = list(dev.generate(6, first_embed=embed_of(7)))
        assert got == want
        # the array-built decoder takes the same table through set_embeddings
        arr = Decoder(model, cuda_ctx, kv_max=128)
        arr.load_kv(ks, vs)
        arr.set_embeddings(emb)
        assert list(arr.generate(6, first_embed=embed_of(7))) == want
        arr.close()
    finally:
        host.close()
        dev.close()


def test_tied_checkpoint(cuda_ctx, tmp_path, model):
    write_checkpoint(model, str(tmp_path), tied=True)  # no lm_head.weight: the embeddings serve
    ks, vs = synth.kv_prefix(model.d, 20)
    a = Decoder(model, cuda_ctx, kv_max=128)
    b = Decoder.from_safetensors(tmp_path, model.d, cuda_ctx, kv_max=128)
    try:
        a.load_kv(ks, vs)
        b.load_kv(ks, vs)
        assert list(a.generate(5, first_embed=model.embed(3))) == list(b.generate(5, first_embed=model.embed(3)))
    finally:
        a.close()
        b.close()


def test_int8_quantised_on_device(cuda_ctx, tmp_path):
    m = synth.Model(n_layers=3, vocab=8192)
    write_checkpoint(m, str(tmp_path))
    quantize_int8(m, cuda_ctx)
    ks, vs = synth.kv_prefix(m.d, 20)
    a = Decoder(m, cuda_ctx, kv_max=128, use_int8=True)
    b = Decoder.from_safetensors(tmp_path, m.d, cuda_ctx, kv_max=128, use_int8=True)
    try:
        a.load_kv(ks, vs)
        b.load_kv(ks, vs)
        ra, rb = _steps(a, m, 4), _steps(b, m, 4)
        for (ta, xa, _), (tb, xb, _) in zip(ra, rb):
            assert ta == tb
            assert np.array_equal(xa, xb)
    finally:
        a.close()
        b.close()


def test_loader_errors_name_the_tensor(cuda_ctx, tmp_path, model):
    t = decoder_tensors(model)
    del t["model.layers.1.mlp.experts.3.up_proj.weight"]
    write_safetensors(str(tmp_path / "model.safetensors"), t)
    with pytest.raises(DsCudaError, match="experts.3.up_proj"):
        Decoder.from_safetensors(tmp_path, model.d, cuda_ctx, kv_max=64)
    t = decoder_tensors(model)
    t["model.layers.0.self_attn.q_proj.weight"] = ("BF16", model.layers[0].wq[:-1])
    write_safetensors(str(tmp_path / "model.safetensors"), t)
    with pytest.raises(DsCudaError, match="unexpected shape"):
        Decoder.from_safetensors(tmp_path, model.d, cuda_ctx, kv_max=64)
    with pytest.raises(DsCudaError, match="no safetensors|cannot open"):
        Decoder.from_safetensors(tmp_path / "nothing", model.d, cuda_ctx, kv_max=64)
