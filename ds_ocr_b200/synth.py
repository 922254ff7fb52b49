"""Seeded synthetic weights and inputs with the DeepSeek3B-MoE decoder shapes.

The reference's checkpoints are not available, so every benchmark and test
runs on random-init weights of the real architecture: BF16 N(0, 0.02)
matrices, F32 RMSNorm weights of 1.0, F32 N(0, 1) activations, and (for the
decode benchmark) a prefilled KV cache whose values are BF16-representable
N(0, 1). Values come from the counter-based generator in csrc/synth.c, so a
(seed, index) pair always yields the same number on any machine.

The same generator is restated in numpy below (`use_numpy_backend`). The
reference arm of the benchmark draws its weights with it, so that process
maps no library of this package: it runs the reference and nothing else.
"""
import ctypes
import os
import zlib
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import _lib

# DeepSeek3B-MoE decoder constants (ds_ocr.h:59-71).
HIDDEN = 1280
N_LAYERS = 12
N_HEADS = 10
HEAD_DIM = 128
DENSE_INTER = 6848
MOE_INTER = 896
N_EXPERTS = 64
N_SHARED = 2
SHARED_INTER = N_SHARED * MOE_INTER
TOP_K = 6
VOCAB = 129280
FIRST_DENSE = 1
RMS_EPS = 1e-6
ROPE_THETA = 10000.0


def seed_of(*parts):
    """Stable 32-bit seed for a named tensor, e.g. seed_of(3, "expert_gu", 17)."""
    return zlib.crc32("/".join(str(p) for p in parts).encode()) | (1 << 32)


def _addr(a):
    return a.ctypes.data


_NUMPY = False


def use_numpy_backend(on=True):
    """Draw every tensor with the numpy restatement of csrc/synth.c instead of
    the compiled generator (same values; slower, and loads no library)."""
    global _NUMPY
    _NUMPY = bool(on)


_U = np.uint64


def _splitmix64(z):
    z = z + _U(0x9E3779B97F4A7C15)
    z = (z ^ (z >> _U(30))) * _U(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> _U(27))) * _U(0x94D049BB133111EB)
    return z ^ (z >> _U(31))


def _np_chunk(out, lo, hi, seed, mean, std, kind):
    with np.errstate(over="ignore"):
        k = _splitmix64(np.array([seed], _U) * _U(0xD1B54A32D192ED03) + _U(0x8CB92BA72F3D8DD7))[0]
        i2 = np.arange(lo, hi, dtype=_U) * _U(2)
        a = _splitmix64(k ^ i2)
        b = _splitmix64(k ^ (i2 + _U(1)))
    u1 = ((a >> _U(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)
    u2 = ((b >> _U(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)
    # mean and std are F32 in the C generator, widened to double
    v = (float(np.float32(mean)) + float(np.float32(std))
         * (np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2))).astype(np.float32)
    flat = out.reshape(-1)
    if kind == 1:
        flat[lo:hi] = v
        return
    u = v.view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    if kind == 0:
        flat[lo:hi] = r
    else:
        flat[lo:hi] = (r.astype(np.uint32) << 16).view(np.float32)


def _np_fill(out, seed, mean, std, kind):
    n = out.size
    step = 1 << 22
    if n <= step:
        _np_chunk(out, 0, n, seed, mean, std, kind)
        return
    workers = max(1, min(32, os.cpu_count() or 1))
    with ThreadPoolExecutor(workers) as ex:
        list(ex.map(lambda lo: _np_chunk(out, lo, min(n, lo + step), seed, mean, std, kind), range(0, n, step)))


def fill_bf16(out, seed, std=0.02, mean=0.0):
    if _NUMPY:
        _np_fill(out, seed, mean, std, 0)
    else:
        _lib.load().ds_synth_normal_bf16(_addr(out), out.size, seed, mean, std)
    return out


def fill_f32(out, seed, std=1.0, mean=0.0):
    if _NUMPY:
        _np_fill(out, seed, mean, std, 1)
    else:
        _lib.load().ds_synth_normal_f32(_addr(out), out.size, seed, mean, std)
    return out


def fill_f32_bf16exact(out, seed, std=1.0, mean=0.0):
    if _NUMPY:
        _np_fill(out, seed, mean, std, 2)
    else:
        _lib.load().ds_synth_normal_f32_bf16exact(_addr(out), out.size, seed, mean, std)
    return out


def normal_bf16(shape, seed, std=0.02):
    return fill_bf16(np.empty(shape, np.uint16), seed, std)


def normal_f32(shape, seed, std=1.0):
    return fill_f32(np.empty(shape, np.float32), seed, std)


def bf16_to_f32(a):
    return (a.astype(np.uint32) << 16).view(np.float32)


class Dims:
    """Model dimensions; defaults are the DeepSeek3B-MoE decoder."""

    def __init__(self, **kw):
        self.hidden = kw.get("hidden", HIDDEN)
        self.n_layers = kw.get("n_layers", N_LAYERS)
        self.n_heads = kw.get("n_heads", N_HEADS)
        self.head_dim = kw.get("head_dim", HEAD_DIM)
        self.dense_inter = kw.get("dense_inter", DENSE_INTER)
        self.moe_inter = kw.get("moe_inter", MOE_INTER)
        self.n_experts = kw.get("n_experts", N_EXPERTS)
        self.n_shared = kw.get("n_shared", N_SHARED)
        self.top_k = kw.get("top_k", TOP_K)
        self.vocab = kw.get("vocab", VOCAB)
        self.first_dense = kw.get("first_dense", FIRST_DENSE)

    @property
    def shared_inter(self):
        return self.n_shared * self.moe_inter


class MoeWeights:
    """One MoE layer in the reference's layout (ds_ocr.c:696-768):
    block  = [E x gate_up_fused (2I x H)] + shared gate_up (2S x H), BF16
    down   = [E x (H x I)], shared_down = H x S, router = E x H."""

    def __init__(self, d, layer, tag="moe"):
        H, I, S, E = d.hidden, d.moe_inter, d.shared_inter, d.n_experts
        self.d = d
        self.router = normal_bf16((E, H), seed_of(tag, layer, "router"))
        self.block = np.empty(E * 2 * I * H + 2 * S * H, np.uint16)
        for e in range(E):
            fill_bf16(self.block[e * 2 * I * H:(e + 1) * 2 * I * H], seed_of(tag, layer, "gate_up", e))
        fill_bf16(self.block[E * 2 * I * H:], seed_of(tag, layer, "shared_gate_up"))
        self.down = np.empty(E * H * I, np.uint16)
        for e in range(E):
            fill_bf16(self.down[e * H * I:(e + 1) * H * I], seed_of(tag, layer, "down", e))
        self.shared_down = normal_bf16((H, S), seed_of(tag, layer, "shared_down"))
        self.int8 = None

    def expert_gate_up(self, e):
        n = 2 * self.d.moe_inter * self.d.hidden
        return self.block[e * n:(e + 1) * n]

    def expert_down(self, e):
        n = self.d.hidden * self.d.moe_inter
        return self.down[e * n:(e + 1) * n]

    def shared_gate_up(self):
        return self.block[self.d.n_experts * 2 * self.d.moe_inter * self.d.hidden:]


class Int8Moe:
    """INT8 copy of a MoeWeights (the --int4 path), contiguous per tensor kind."""

    def __init__(self, d):
        H, I, S, E = d.hidden, d.moe_inter, d.shared_inter, d.n_experts
        self.gu_q = np.empty(E * 2 * I * H, np.int8)
        self.gu_s = np.empty(E * 2 * I, np.float32)
        self.gu_o = np.empty(E * 2 * I, np.float32)
        self.dn_q = np.empty(E * H * I, np.int8)
        self.dn_s = np.empty(E * H, np.float32)
        self.dn_o = np.empty(E * H, np.float32)
        self.sgu_q = np.empty(2 * S * H, np.int8)
        self.sgu_s = np.empty(2 * S, np.float32)
        self.sgu_o = np.empty(2 * S, np.float32)
        self.sdn_q = np.empty(H * S, np.int8)
        self.sdn_s = np.empty(H, np.float32)
        self.sdn_o = np.empty(H, np.float32)


class LayerWeights:
    def __init__(self, d, layer):
        H, q = d.hidden, d.n_heads * d.head_dim
        self.index = layer
        self.wq = normal_bf16((q, H), seed_of("attn", layer, "wq"))
        self.wk = normal_bf16((q, H), seed_of("attn", layer, "wk"))
        self.wv = normal_bf16((q, H), seed_of("attn", layer, "wv"))
        self.wo = normal_bf16((H, q), seed_of("attn", layer, "wo"))
        self.input_norm = np.ones(H, np.float32)
        self.post_norm = np.ones(H, np.float32)
        self.dense = layer < d.first_dense
        if self.dense:
            D = d.dense_inter
            self.dense_gate = normal_bf16((D, H), seed_of("dense", layer, "gate"))
            self.dense_up = normal_bf16((D, H), seed_of("dense", layer, "up"))
            self.dense_down = normal_bf16((H, D), seed_of("dense", layer, "down"))
            self.moe = None
        else:
            self.dense_gate = self.dense_up = self.dense_down = None
            self.moe = MoeWeights(d, layer)


class Model:
    """Full decoder: layers, final norm, LM head (tied with the embeddings)."""

    def __init__(self, d=None, **kw):
        self.d = d or Dims(**kw)
        self.layers = [LayerWeights(self.d, l) for l in range(self.d.n_layers)]
        self.final_norm = np.ones(self.d.hidden, np.float32)
        self.lm_head = normal_bf16((self.d.vocab, self.d.hidden), seed_of("lm_head"))

    def embed(self, token):
        return bf16_to_f32(self.lm_head[token]).copy()


def kv_prefix(d, n_tokens, stream=0):
    """Prefilled KV cache: per layer K, V [n_tokens x (heads*head_dim)] F32 with
    BF16-representable N(0, 1) values."""
    kd = d.n_heads * d.head_dim
    ks, vs = [], []
    for l in range(d.n_layers):
        ks.append(fill_f32_bf16exact(np.empty((n_tokens, kd), np.float32), seed_of("kv", stream, l, "k")))
        vs.append(fill_f32_bf16exact(np.empty((n_tokens, kd), np.float32), seed_of("kv", stream, l, "v")))
    return ks, vs
