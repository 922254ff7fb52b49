"""Multi-stream decode on the tensor cores: the skinny GEMM (<= 64 token
rows against BF16 weights, inputs split into two BF16 planes) against an
F32 reference of the same product."""
import numpy as np
import pytest

from conftest import rel_l2
from ds_ocr_b200 import synth

pytestmark = pytest.mark.gpu


def _bf16_f32(W):
    return (W.view(np.uint16).astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("n,K,N", [(1, 1280, 1280), (7, 1280, 200), (64, 1280, 3840), (64, 896, 1280),
                                   (33, 6848, 1280), (64, 1280, 64)])
def test_skinny_matmul(cuda_ctx, n, K, N):
    import torch
    W = synth.normal_bf16((N, K), synth.seed_of("skinny", n, K, N))
    X = synth.normal_f32((n, K), synth.seed_of("skinny_x", n, K, N))
    R = synth.normal_f32((n, N), synth.seed_of("skinny_r", n, K, N))
    cuda_ctx.register(W)
    dW = cuda_ctx.device_ptr(W)
    tx, tr = torch.from_numpy(X).cuda(), torch.from_numpy(R).cuda()
    ty = torch.full((n, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    lib = cuda_ctx.lib
    assert lib.ds_cuda_skinny_matmul_dev(cuda_ctx.h, tx.data_ptr(), n, K, dW, N, None, ty.data_ptr(), None) == 0
    cuda_ctx.synchronize()
    ref = X.astype(np.float64) @ _bf16_f32(W).astype(np.float64).T
    y = ty.cpu().numpy()
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) < 1e-5
    ty2 = torch.empty_like(ty)
    assert lib.ds_cuda_skinny_matmul_dev(cuda_ctx.h, tx.data_ptr(), n, K, dW, N, tr.data_ptr(), ty2.data_ptr(),
                                         None) == 0
    cuda_ctx.synchronize()
    assert rel_l2(ty2.cpu().numpy() - R, ref) < 1e-5


def _gap(orc, model, fx):
    y = np.empty(model.d.vocab, np.float32)
    orc.orc_matvec_bf16(y.ctypes.data, fx.ctypes.data, model.lm_head.ctypes.data, model.d.hidden, model.d.vocab)
    t = np.sort(y)[-2:]
    return t[1] - t[0]


@pytest.fixture(scope="module")
def small_model():
    return synth.Model(n_layers=3, vocab=8192)


@pytest.mark.parametrize("S", [1, 4, 64])
def test_batch_decoder_matches_single_stream(cuda_ctx, orc, small_model, S):
    # S streams with their own KV prefixes (different lengths) against the
    # single-stream decoder run on each stream: final hidden states within
    # 1e-3 relative L2, tokens equal where the top-2 logit gap > 1e-4
    from ds_ocr_b200.decoder import BatchDecoder, Decoder
    model = small_model
    bd = BatchDecoder(model, S, cuda_ctx, kv_max=256)
    prefixes = [synth.kv_prefix(model.d, 5 + 11 * s % 97, stream=s + 1) for s in range(S)]
    for s, (ks, vs) in enumerate(prefixes):
        bd.load_kv(s, ks, vs)
    check = range(S) if S <= 4 else (0, 17, 63)
    singles = {}
    for s in check:
        dec = Decoder(model, cuda_ctx, kv_max=256)
        dec.load_kv(*prefixes[s])
        singles[s] = dec
    E = np.stack([model.embed((7 + 13 * s) % model.d.vocab) for s in range(S)])
    compared = 0
    try:
        for step in range(3):
            toks, fx = bd.forward(E, want_x=True)
            for s in check:
                t1, fx1, _ = singles[s].forward(E[s], want_x=True)
                assert rel_l2(fx[s], fx1) < 1e-3, (step, s)
                if _gap(orc, model, fx1) > 1e-4:
                    assert toks[s] == t1, (step, s)
                    compared += 1
            E = np.stack([model.embed(int(t)) for t in toks])
    finally:
        bd.close()
        for d in singles.values():
            d.close()
    assert compared >= len(check)


def test_batch_decoder_generate_dev_matches_forward(cuda_ctx, small_model):
    from ds_ocr_b200.decoder import BatchDecoder
    model = small_model
    S = 8
    outs = []
    for mode in ("forward", "dev"):
        bd = BatchDecoder(model, S, cuda_ctx, kv_max=128)
        for s in range(S):
            bd.load_kv(s, *synth.kv_prefix(model.d, 20 + s, stream=s + 1))
        E = np.stack([model.embed(3 + s) for s in range(S)])
        first = bd.forward(E)
        if mode == "forward":
            seq = [first] + [bd.forward() for _ in range(5)]
        else:
            bd.generate_dev(5)
            cuda_ctx.synchronize()
            seq = [first] + [None] * 5
            seq[-1] = bd.forward()  # one more step reads the device state
            seq = [first, seq[-1]]
        outs.append(seq)
        bd.close()
    # the step after 5 device-looped steps equals the 7th host-driven step
    fwd = outs[0]
    bd2 = BatchDecoder(model, S, cuda_ctx, kv_max=128)
    for s in range(S):
        bd2.load_kv(s, *synth.kv_prefix(model.d, 20 + s, stream=s + 1))
    E = np.stack([model.embed(3 + s) for s in range(S)])
    host = [bd2.forward(E)] + [bd2.forward() for _ in range(6)]
    bd2.close()
    assert np.array_equal(outs[1][1], host[6])


def test_batch_decoder_vs_oracle_full_config(cuda_ctx, orc):
    """The benchmark's configuration: 12 layers, vocabulary 129280, 64
    streams with their own 662-token KV prefixes, compared directly with the
    CPU oracle's decoder step (not with another CUDA path) on four streams
    over 3 steps: final hidden state within 1e-3 relative L2 (the north-star
    activation bar), token equal where the top-2 logit gap exceeds 1e-4."""
    import oracle as O
    from ds_ocr_b200.decoder import BatchDecoder
    model = synth.Model()
    S, P = 64, 662
    bd = BatchDecoder(model, S, cuda_ctx, kv_max=1024)
    check = (0, 21, 42, 63)
    oracles = {}
    try:
        for s in range(S):
            ks, vs = synth.kv_prefix(model.d, P, stream=s + 1)
            bd.load_kv(s, ks, vs)
            if s in check:
                o = O.OracleDecoder(model, kv_max=1024)
                o.load_kv(ks, vs)
                oracles[s] = o
            del ks, vs
        E = np.stack([model.embed((1 + 7 * s) % model.d.vocab) for s in range(S)])
        compared = 0
        for step in range(3):
            toks, fx = bd.forward(E, want_x=True)
            # both sides take the same input embedding every step
            for s in check:
                otok, ofx, _ = oracles[s].step(E[s])
                err = rel_l2(fx[s], ofx)
                assert err < 1e-3, (step, s, err)
                if _gap(orc, model, ofx) > 1e-4:
                    assert toks[s] == otok, (step, s)
                    compared += 1
            E = np.stack([model.embed(int(t)) for t in toks])
        assert compared >= 8
    finally:
        bd.close()
