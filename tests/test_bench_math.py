"""The algorithmic byte and FLOP counts bench.py divides by (roofline
`achieved`), re-derived here from the model's shapes."""
import os
import sys

from ds_ocr_b200 import synth

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


D = synth.Dims()
H, I, E, K, V = D.hidden, D.moe_inter, D.n_experts, D.top_k, D.vocab
S = D.n_shared * D.moe_inter
QD = D.n_heads * D.head_dim


def test_moe_layer_bytes():
    expert = (2 * I * H + H * I) * 2          # fused gate/up + down, BF16
    shared = (2 * S * H + H * S) * 2
    router = E * H * 2
    assert expert == 6_881_280 and shared == 13_762_560 and router == 163_840
    assert bench.MS_MOE_LAYER_BYTES == E * expert + shared + router


def test_decode_step_bytes():
    attn = 4 * QD * H * 2                      # wq, wk, wv, wo
    dense = 3 * D.dense_inter * H * 2
    moe = K * 6_881_280 + 13_762_560 + 163_840
    norms = (2 * D.n_layers + 1) * H * 4
    lm = V * H * 2
    weights = D.n_layers * attn + D.first_dense * dense + (D.n_layers - D.first_dense) * moe + lm + norms
    assert lm == bench.LM_BYTES == 330_956_800
    assert abs(bench.DEC_WEIGHT_BYTES - weights) <= 128_000  # up to the norm vectors' accounting
    assert bench.KV_BYTES_PER_KEY == D.n_layers * 2 * QD * 2  # K and V rows, BF16 hi plane
    assert bench.decode_bytes(10, 2) == 2 * bench.DEC_WEIGHT_BYTES + bench.KV_BYTES_PER_KEY * (11 + 12)


def test_prefill_flops():
    T = bench.PF_TOKENS
    per_token_moe = 2 * (K * (2 * I * H + H * I) + (2 * S * H + H * S))
    # 2 FLOPs per BF16 weight (2 bytes): the per-token FLOPs equal the bytes
    assert bench.PF_FLOPS_LAYER == T * per_token_moe == T * (6 * 6_881_280 + 13_762_560)
    whole = bench.prefill_full_flops(T, D)
    proj = 2 * T * (H * 3 * QD + QD * H)
    attn = 4 * QD * T * (T + 1) // 2
    dense = 2 * T * 3 * D.dense_inter * H
    moe = 2 * T * (K * 3 * I * H + 3 * S * H + E * H)
    assert whole == D.n_layers * (proj + attn) + D.first_dense * dense + (D.n_layers - D.first_dense) * moe \
        + 2 * V * H
    assert 2.0e12 < whole < 3.5e12


def test_synth_numpy_backend_matches_native():
    """The numpy restatement of the generator (used by the reference arm so
    that it maps no library of this package) gives the same bits."""
    import numpy as np
    from ds_ocr_b200 import synth
    try:
        for fn, dt, n in ((synth.fill_bf16, np.uint16, 5_000_011), (synth.fill_f32, np.float32, 4097),
                          (synth.fill_f32_bf16exact, np.float32, 70_001)):
            synth.use_numpy_backend(False)
            a = fn(np.empty(n, dt), synth.seed_of("t", n), 0.3, 0.1)
            synth.use_numpy_backend(True)
            b = fn(np.empty(n, dt), synth.seed_of("t", n), 0.3, 0.1)
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
    finally:
        synth.use_numpy_backend(False)
