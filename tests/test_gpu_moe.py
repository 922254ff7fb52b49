"""Parity of the CUDA decode kernels (through the C ABI) with the CPU oracle:
argmax LM head, plain matvec, the MoE layer (BF16, both truncation modes, and
INT8), the Metal-shaped expert calls, and the bit-exact INT8 quantiser."""
import ctypes

import numpy as np
import pytest

import oracle as O
from conftest import rel_l2
from ds_ocr_b200 import synth
from ds_ocr_b200.cuda import Int8Block

pytestmark = pytest.mark.gpu
H, I, S, E, K, V = 1280, 896, 1792, 64, 6, 129280


def oracle_logits(orc, x, W, n, rows):
    y = np.empty(rows, np.float32)
    orc.orc_matvec_bf16(y.ctypes.data, x.ctypes.data, W.ctypes.data, n, rows)
    return y


@pytest.fixture(scope="module")
def lm_head():
    return synth.normal_bf16((V, H), synth.seed_of("test", "lm_head"))


def test_lm_head_argmax_full_vocab(cuda_ctx, orc, lm_head):
    checked = 0
    for s in range(12):
        x = synth.normal_f32(H, 1000 + s)
        tok, val = cuda_ctx.argmax_matvec_bf16(x, lm_head, H, V)
        y = oracle_logits(orc, x, lm_head, H, V)
        top = np.argsort(y)[-2:]
        assert abs(val - y[tok]) < 1e-4
        if y[top[1]] - y[top[0]] > 1e-4:
            assert tok == top[1]
            checked += 1
        assert cuda_ctx.lm_head_argmax(x, lm_head, H, V) == tok
    assert checked >= 10


@pytest.mark.parametrize("rows,n", [(1, 1280), (3, 1280), (4097, 8), (1001, 2048), (64, 896)])
def test_argmax_shapes(cuda_ctx, orc, rows, n):
    W = synth.normal_bf16((rows, n), synth.seed_of("argmax_shape", rows, n))
    x = synth.normal_f32(n, rows + n)
    tok, val = cuda_ctx.argmax_matvec_bf16(x, W, n, rows)
    y = oracle_logits(orc, x, W, n, rows)
    srt = np.sort(y)
    if rows == 1 or srt[-1] - srt[-2] > 1e-4:
        assert tok == int(np.argmax(y))
    assert abs(val - y[tok]) < 1e-4


def test_argmax_ties_take_lowest_index(cuda_ctx):
    W = synth.normal_bf16((5000, 256), 5)
    for r in (4000, 333, 4999):
        W[r] = W[1234]
    x = synth.bf16_to_f32(W[1234]).copy()
    tok, _ = cuda_ctx.argmax_matvec_bf16(x, W, 256, 5000)
    assert tok == 333


def _torch_logits(X, W):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    w = torch.from_numpy(W.view(np.int16).astype(np.int32) << 16).view(torch.float32).cuda()
    return (torch.from_numpy(X).cuda() @ w.t()).cpu().numpy()


@pytest.mark.parametrize("B", [2, 5, 33, 64])
def test_argmax_batch_tensor_core(cuda_ctx, orc, lm_head, B):
    # batches of 2..64 run as one tcgen05 pass (split-BF16 inputs): tokens
    # equal the F32 reference wherever the top-2 gap exceeds 1e-4, logits
    # within 1e-4; the oracle pins four of them
    X = synth.normal_f32((B, H), 77 + B)
    toks, vals = cuda_ctx.argmax_batch(X, lm_head, H, V)
    Y = _torch_logits(X, lm_head)
    for b in range(B):
        srt = np.sort(Y[b])
        if srt[-1] - srt[-2] > 1e-4:
            assert toks[b] == int(np.argmax(Y[b])), b
        assert abs(vals[b] - Y[b][toks[b]]) < 1e-4
    for b in range(min(B, 4)):
        y = oracle_logits(orc, X[b], lm_head, H, V)
        t2 = np.sort(y)[-2:]
        if t2[1] - t2[0] > 1e-4:
            assert toks[b] == int(np.argmax(y))


@pytest.mark.parametrize("rows,n,B", [(1001, 256, 7), (129, 64, 64), (300, 1280, 3)])
def test_argmax_batch_shapes(cuda_ctx, rows, n, B):
    W = synth.normal_bf16((rows, n), synth.seed_of("argmax_batch_shape", rows, n))
    X = synth.normal_f32((B, n), rows + B)
    toks, vals = cuda_ctx.argmax_batch(X, W, n, rows)
    Y = _torch_logits(X, W)
    for b in range(B):
        srt = np.sort(Y[b])
        if rows == 1 or srt[-1] - srt[-2] > 1e-4:
            assert toks[b] == int(np.argmax(Y[b]))
        assert abs(vals[b] - Y[b][toks[b]]) < 1e-4


def test_argmax_batch_ties_take_lowest_index(cuda_ctx):
    W = synth.normal_bf16((5000, 256), 5)
    for r in (4000, 333, 4999):
        W[r] = W[1234]
    x = synth.bf16_to_f32(W[1234]).copy()
    X = np.stack([x, x, -x]).astype(np.float32)
    toks, _ = cuda_ctx.argmax_batch(X, W, 256, 5000)
    assert toks[0] == 333 and toks[1] == 333


def test_matvec(cuda_ctx, orc):
    W = synth.normal_bf16((3840, H), 31)
    bias = synth.normal_f32(3840, 32)
    x = synth.normal_f32(H, 33)
    y = cuda_ctx.matvec_bf16(x, W, H, 3840)
    assert rel_l2(y, oracle_logits(orc, x, W, H, 3840)) < 1e-6
    yb = cuda_ctx.matvec_bf16(x, W, H, 3840, bias)
    assert rel_l2(yb - bias, y) < 1e-6


def routing_gap(orc, mw, x):
    scores = oracle_logits(orc, x, mw.router, H, E)
    p = np.exp(scores - scores.max())
    p = np.sort(p / p.sum())
    return p[-K] - p[-K - 1]


def oracle_layer(mw, simulate=0):
    d = mw.d
    dims = O.make_dims(d, simulate)

    class _LW:
        pass
    lw = _LW()
    for n in ("wq", "wk", "wv", "wo", "input_norm", "post_norm", "dense_gate", "dense_up", "dense_down"):
        setattr(lw, n, None)
    lw.moe = mw
    return dims, O.make_layer(lw)


def oracle_moe(orc, mw, x, simulate=0, int8=False):
    dims, L = oracle_layer(mw, simulate)
    out = np.empty(H, np.float32)
    idx = np.empty(K, np.int32)
    w = np.empty(K, np.float32)
    orc.orc_moe_forward(out.ctypes.data, x.ctypes.data, ctypes.byref(L), ctypes.byref(dims), int(int8),
                        idx.ctypes.data, w.ctypes.data)
    return out, idx, w


@pytest.mark.parametrize("simulate", [0, 1])
def test_moe_layer(cuda_ctx, orc, moe_weights, simulate):
    cuda_ctx.set_numerics(simulate_bf16=simulate)
    try:
        for s in range(12):
            x = synth.normal_f32(H, 2000 + s)
            out, idx, w = cuda_ctx.moe_layer(x, moe_weights, return_routing=True)
            ro, ridx, rw = oracle_moe(orc, moe_weights, x, simulate)
            if routing_gap(orc, moe_weights, x) > 1e-4:
                assert np.array_equal(idx, ridx)
                assert rel_l2(w, rw) < 1e-5
                assert rel_l2(out, ro) < (1e-5 if simulate == 0 else 1e-3)
    finally:
        cuda_ctx.set_numerics(0, 0)


def test_moe_layer_repeatable(cuda_ctx, moe_weights):
    x = synth.normal_f32(H, 31337)
    a = cuda_ctx.moe_layer(x, moe_weights)
    b = cuda_ctx.moe_layer(x, moe_weights)
    assert np.array_equal(a, b)


def test_metal_shaped_calls(cuda_ctx, orc, moe_weights):
    mw = moe_weights
    x = synth.normal_f32(H, 4242)
    ro, ridx, rw = oracle_moe(orc, mw, x)
    out = cuda_ctx.moe_experts(x, [mw.expert_gate_up(e) for e in ridx], [mw.expert_down(e) for e in ridx], rw, H, I)
    cuda_ctx.shared_experts(x, mw.shared_gate_up(), mw.shared_down, H, S, out)
    assert rel_l2(out, ro) < 1e-5
    # ds_expert_forward_fused signature
    y = cuda_ctx.expert_forward_fused(x, mw.expert_gate_up(3), mw.expert_down(3), H, I)
    yo = np.empty(H, np.float32)
    orc.orc_expert_fused(yo.ctypes.data, x.ctypes.data, mw.expert_gate_up(3).ctypes.data,
                         mw.expert_down(3).ctypes.data, H, I, 0)
    assert rel_l2(y, yo) < 1e-5


def quantize_all(orc, mw):
    d = mw.d
    q = synth.Int8Moe(d)
    for e in range(E):
        orc.orc_int8_quantize(mw.expert_gate_up(e).ctypes.data, 2 * I, H, q.gu_q[e * 2 * I * H:].ctypes.data,
                              q.gu_s[e * 2 * I:].ctypes.data, q.gu_o[e * 2 * I:].ctypes.data)
        orc.orc_int8_quantize(mw.expert_down(e).ctypes.data, H, I, q.dn_q[e * H * I:].ctypes.data,
                              q.dn_s[e * H:].ctypes.data, q.dn_o[e * H:].ctypes.data)
    orc.orc_int8_quantize(mw.shared_gate_up().ctypes.data, 2 * S, H, q.sgu_q.ctypes.data, q.sgu_s.ctypes.data,
                          q.sgu_o.ctypes.data)
    orc.orc_int8_quantize(mw.shared_down.ctypes.data, H, S, q.sdn_q.ctypes.data, q.sdn_s.ctypes.data,
                          q.sdn_o.ctypes.data)
    return q


def test_int8_quantize_bit_exact(cuda_ctx, orc, moe_weights):
    for W, r, c in ((moe_weights.expert_gate_up(5), 2 * I, H), (moe_weights.expert_down(9), H, I),
                    (synth.normal_bf16((7, 48), 3), 7, 48), (np.full(64, 0x3f80, np.uint16), 2, 32)):
        q, s, o = cuda_ctx.int8_quantize_bf16(W, r, c)
        qa, sa, oa = np.empty(r * c, np.int8), np.empty(r, np.float32), np.empty(r, np.float32)
        orc.orc_int8_quantize(W.ctypes.data, r, c, qa.ctypes.data, sa.ctypes.data, oa.ctypes.data)
        assert np.array_equal(q, qa) and np.array_equal(s, sa) and np.array_equal(o, oa)


def test_moe_layer_int8(cuda_ctx, orc, moe_weights):
    mw = moe_weights
    mw.int8 = quantize_all(orc, mw)
    try:
        for s in range(8):
            x = synth.normal_f32(H, 3000 + s)
            out, idx, w = cuda_ctx.moe_layer_int8(x, mw, return_routing=True)
            ro, ridx, _ = oracle_moe(orc, mw, x, int8=True)
            bf = oracle_moe(orc, mw, x)[0]
            if routing_gap(orc, mw, x) > 1e-4:
                assert np.array_equal(idx, ridx)
                assert rel_l2(out, ro) < 1e-5
            # INT8 against the BF16 layer: the reference's INT8 matvec bar
            # (test_int4.c:84, relative error < 0.02); ~0.013 measured
            assert rel_l2(out, bf) < 0.02
        q = mw.int8
        # config 2's RMS < 0.01, as the reference measures quantisation error
        # (ds_int4_quant_error_rms, ds_quantize.c:127-144: relative RMS of the
        # dequantised weights against the BF16 originals)
        for e in (0, 31, 63):
            Wf = synth.bf16_to_f32(mw.expert_gate_up(e)).reshape(2 * I, H).astype(np.float64)
            qq = q.gu_q[e * 2 * I * H:(e + 1) * 2 * I * H].reshape(2 * I, H).astype(np.float64)
            deq = (q.gu_s[e * 2 * I:(e + 1) * 2 * I, None].astype(np.float32) * (qq + 128).astype(np.float32)
                   + q.gu_o[e * 2 * I:(e + 1) * 2 * I, None])
            rms = np.sqrt(((Wf - deq) ** 2).sum() / (Wf ** 2).sum())
            print(f"expert {e} gate_up quantisation RMS {rms:.5f}")
            assert rms < 0.01
        gub = Int8Block.of(q.gu_q[:2 * I * H], q.gu_s[:2 * I], q.gu_o[:2 * I], 2 * I, H)
        dnb = Int8Block.of(q.dn_q[:H * I], q.dn_s[:H], q.dn_o[:H], H, I)
        x = synth.normal_f32(H, 99)
        y = cuda_ctx.expert_forward_fused_int4(x, gub, dnb, H, I)
        yo = np.empty(H, np.float32)
        orc.orc_expert_fused_int8(yo.ctypes.data, x.ctypes.data, q.gu_q.ctypes.data, q.gu_s.ctypes.data,
                                  q.gu_o.ctypes.data, q.dn_q.ctypes.data, q.dn_s.ctypes.data, q.dn_o.ctypes.data,
                                  H, I, 0)
        assert rel_l2(y, yo) < 1e-5
    finally:
        mw.int8 = None


def test_dev_entry_points_with_torch_buffers(cuda_ctx, moe_weights):
    import torch
    mw = moe_weights
    lib = cuda_ctx.lib
    dr = cuda_ctx.device_ptr(mw.router)
    if not dr:
        cuda_ctx.moe_layer(synth.normal_f32(H, 1), mw)  # registers on first use
        dr = cuda_ctx.device_ptr(mw.router)
    db, dd, ds_ = cuda_ctx.device_ptr(mw.block), cuda_ctx.device_ptr(mw.down), cuda_ctx.device_ptr(mw.shared_down)
    x = synth.normal_f32(H, 555)
    tx = torch.from_numpy(x).cuda()
    tout = torch.empty(H, device="cuda")
    tidx = torch.empty(K, dtype=torch.int32, device="cuda")
    tw = torch.empty(K, device="cuda")
    torch.cuda.synchronize()
    rc = lib.ds_cuda_moe_layer_dev(cuda_ctx.h, tx.data_ptr(), tout.data_ptr(), dr, db, dd, ds_, H, I, S, E, K,
                                   tidx.data_ptr(), tw.data_ptr(), None)
    assert rc == 0
    cuda_ctx.synchronize()
    ref = cuda_ctx.moe_layer(x, mw)
    assert np.array_equal(tout.cpu().numpy(), ref)


@pytest.mark.ref
def test_moe_layer_int8_vs_compiled_reference(cuda_ctx, orc):
    """The GPU INT8 layer against the reference itself: oracle/_ref quantises
    with ds_int4_quantize_bf16 and runs moe_forward with int4_enabled
    (ds_moe_decoder.c:237-243, 269-278); the GPU runs the same INT8 blocks."""
    model = synth.Model(n_layers=2, vocab=4096)
    R = O.RefDecoder(model, kv_max=64, threads=8)
    R.quantize()
    mw = model.layers[1].moe
    try:
        for s in range(6):
            x = synth.normal_f32(H, 4100 + s)
            ro = R.moe_forward(1, x)
            out = cuda_ctx.moe_layer_int8(x, mw)
            if routing_gap(orc, mw, x) > 1e-4:
                assert rel_l2(out, ro) < 1e-5, s
    finally:
        mw.int8 = None
