"""Greedy decode of the DeepSeek3B-MoE decoder through the ds_cuda C ABI.

`Decoder` mirrors the reference's decode entry point ds_decoder_forward
(ds_moe_decoder.c:911): forward(embed) runs one step and returns the greedy
token, advancing the KV cache. generate(n) runs n steps on the device
without host round trips (each step's token embedding feeds the next).
"""
import ctypes

import numpy as np

from . import synth
from ._lib import DsCudaError, load
from .cuda import Context, _a


class DecoderConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "n_layers", "n_heads", "head_dim", "dense_inter", "moe_inter",
                                            "n_experts", "n_shared", "top_k", "vocab", "first_dense")] + \
               [("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("kv_max", ctypes.c_int),
                ("use_int8", ctypes.c_int), ("engine", ctypes.c_int)]


_LW_FIELDS = ("wq", "wk", "wv", "wo", "input_norm", "post_attn_norm", "dense_gate", "dense_up", "dense_down",
              "router", "expert_block", "down", "shared_down", "gu_q", "gu_scale", "gu_off", "dn_q", "dn_scale",
              "dn_off", "sgu_q", "sgu_scale", "sgu_off", "sdn_q", "sdn_scale", "sdn_off")


class LayerWeightsC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in _LW_FIELDS]


def layer_struct(lw):
    s = LayerWeightsC()
    s.wq, s.wk, s.wv, s.wo = _a(lw.wq), _a(lw.wk), _a(lw.wv), _a(lw.wo)
    s.input_norm, s.post_attn_norm = _a(lw.input_norm), _a(lw.post_norm)
    s.dense_gate, s.dense_up, s.dense_down = _a(lw.dense_gate), _a(lw.dense_up), _a(lw.dense_down)
    m = lw.moe
    if m is not None:
        s.router, s.expert_block, s.down, s.shared_down = _a(m.router), _a(m.block), _a(m.down), _a(m.shared_down)
        q = m.int8
        if q is not None:
            s.gu_q, s.gu_scale, s.gu_off = _a(q.gu_q), _a(q.gu_s), _a(q.gu_o)
            s.dn_q, s.dn_scale, s.dn_off = _a(q.dn_q), _a(q.dn_s), _a(q.dn_o)
            s.sgu_q, s.sgu_scale, s.sgu_off = _a(q.sgu_q), _a(q.sgu_s), _a(q.sgu_o)
            s.sdn_q, s.sdn_scale, s.sdn_off = _a(q.sdn_q), _a(q.sdn_s), _a(q.sdn_o)
    return s


def quantize_int8(model, ctx=None):
    """The --int4 switch: per-row INT8 copies of every MoE layer's experts,
    quantised on the GPU (bit-identical to ds_int4_quantize_bf16)."""
    own = ctx is None
    ctx = ctx or Context(0)
    d = model.d
    H, I, S, E = d.hidden, d.moe_inter, d.shared_inter, d.n_experts
    for lw in model.layers:
        m = lw.moe
        if m is None:
            continue
        q = synth.Int8Moe(d)
        for e in range(E):
            a, b, c = ctx.int8_quantize_bf16(m.expert_gate_up(e), 2 * I, H)
            q.gu_q[e * 2 * I * H:(e + 1) * 2 * I * H], q.gu_s[e * 2 * I:(e + 1) * 2 * I], q.gu_o[e * 2 * I:(e + 1) * 2 * I] = a, b, c
            a, b, c = ctx.int8_quantize_bf16(m.expert_down(e), H, I)
            q.dn_q[e * H * I:(e + 1) * H * I], q.dn_s[e * H:(e + 1) * H], q.dn_o[e * H:(e + 1) * H] = a, b, c
        q.sgu_q[:], q.sgu_s[:], q.sgu_o[:] = ctx.int8_quantize_bf16(m.shared_gate_up(), 2 * S, H)
        q.sdn_q[:], q.sdn_s[:], q.sdn_o[:] = ctx.int8_quantize_bf16(m.shared_down, H, S)
        m.int8 = q
    if own:
        ctx.close()
    return model


class Decoder:
    ENGINE_GRAPH, ENGINE_PERSISTENT = 0, 1

    def __init__(self, model, ctx=None, kv_max=1024, use_int8=False, engine=0):
        self.ctx = ctx or Context(0)
        self.lib = self.ctx.lib
        self.model = model
        d = model.d
        self.cfg = DecoderConfig(d.hidden, d.n_layers, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter,
                                 d.n_experts, d.n_shared, d.top_k, d.vocab, d.first_dense, synth.RMS_EPS,
                                 synth.ROPE_THETA, kv_max, int(use_int8), int(engine))
        self._layers = (LayerWeightsC * d.n_layers)(*[layer_struct(lw) for lw in model.layers])
        self.ctx._pin(*[getattr(lw, n) for lw in model.layers for n in ("wq", "wk", "wv", "wo", "input_norm",
                                                                        "post_norm", "dense_gate", "dense_up",
                                                                        "dense_down")])
        for lw in model.layers:
            if lw.moe is not None:
                m = lw.moe
                self.ctx._pin(m.router, m.block, m.down, m.shared_down)
                if m.int8 is not None:
                    self.ctx._pin(*m.int8.__dict__.values())
        self.ctx._pin(model.final_norm, model.lm_head)
        self.id = self.ctx.check(self.lib.ds_cuda_decoder_create(self.ctx.h, ctypes.byref(self.cfg), self._layers,
                                                                 _a(model.final_norm), _a(model.lm_head)),
                                 "decoder_create")

    @classmethod
    def from_safetensors(cls, path, dims, ctx=None, kv_max=1024, use_int8=False, engine=0):
        """A decoder whose weights come from a safetensors checkpoint (a
        directory of model.safetensors / model-*.safetensors, or one file) in
        the reference's tensor naming; dims: a synth.Dims of its shapes."""
        self = cls.__new__(cls)
        self.ctx = ctx or Context(0)
        self.lib = self.ctx.lib
        self.model = type("Shapes", (), {"d": dims})()
        d = dims
        self.cfg = DecoderConfig(d.hidden, d.n_layers, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter,
                                 d.n_experts, d.n_shared, d.top_k, d.vocab, d.first_dense, synth.RMS_EPS,
                                 synth.ROPE_THETA, kv_max, int(use_int8), int(engine))
        self.id = 0
        self.id = self.ctx.check(self.lib.ds_cuda_decoder_create_from_safetensors(self.ctx.h, str(path).encode(),
                                                                                ctypes.byref(self.cfg)),
                                 "decoder_create_from_safetensors")
        return self

    def set_embeddings(self, table):
        """The token embedding table of the device decode loop (default: the
        LM head); a [vocab x hidden] BF16 array kept alive by the caller."""
        t = np.ascontiguousarray(table, np.uint16)
        self.ctx._pin(t)
        self.ctx.check(self.lib.ds_cuda_decoder_set_embeddings(self.ctx.h, self.id, _a(t)), "decoder_set_embeddings")

    def load_kv(self, ks, vs, pos0=0):
        if ks[0].shape[0] == 0:
            self.set_len(pos0)
            return
        for l, (k, v) in enumerate(zip(ks, vs)):
            k = np.ascontiguousarray(k, np.float32)
            v = np.ascontiguousarray(v, np.float32)
            self.ctx.check(self.lib.ds_cuda_decoder_load_kv(self.ctx.h, self.id, l, pos0, k.shape[0], _a(k), _a(v)),
                           "decoder_load_kv")
        self.set_len(pos0 + ks[0].shape[0])

    def set_len(self, n):
        self.ctx.check(self.lib.ds_cuda_decoder_set_len(self.ctx.h, self.id, n), "decoder_set_len")

    def prefill(self, embeds, want_x=False):
        """ds_decoder_prefill on [T x hidden] embeddings at the current
        position: the first generated token (and the last row's final
        normed state and logit with want_x)."""
        e = np.ascontiguousarray(embeds, np.float32)
        fx = np.empty(self.model.d.hidden, np.float32) if want_x else None
        lg = np.empty(1, np.float32)
        tok = self.ctx.check(self.lib.ds_cuda_decoder_prefill(self.ctx.h, self.id, _a(e), e.shape[0], _a(fx), _a(lg)),
                             "decoder_prefill")
        return (tok, fx, float(lg[0])) if want_x else tok

    def prefill_dev(self, d_embeds, n_tokens, stream=None):
        self.ctx.check(self.lib.ds_cuda_decoder_prefill_dev(self.ctx.h, self.id, d_embeds, n_tokens, stream),
                       "decoder_prefill_dev")

    def kv(self, layer, pos0, n):
        kd = self.model.d.n_heads * self.model.d.head_dim
        k = np.empty((n, kd), np.float32)
        v = np.empty((n, kd), np.float32)
        self.ctx.check(self.lib.ds_cuda_decoder_get_kv(self.ctx.h, self.id, layer, pos0, n, _a(k), _a(v)),
                       "decoder_get_kv")
        return k, v

    @property
    def length(self):
        return self.ctx.check(self.lib.ds_cuda_decoder_get_len(self.ctx.h, self.id), "decoder_get_len")

    def forward(self, embed, want_x=False):
        embed = np.ascontiguousarray(embed, np.float32)
        fx = np.empty(self.model.d.hidden, np.float32) if want_x else None
        lg = np.empty(1, np.float32)
        tok = self.ctx.check(self.lib.ds_cuda_decoder_forward(self.ctx.h, self.id, _a(embed), _a(fx), _a(lg)),
                             "decoder_forward")
        return (tok, fx, float(lg[0])) if want_x else tok

    def generate(self, n_steps, first_embed=None):
        toks = np.empty(n_steps, np.int32)
        fe = None if first_embed is None else np.ascontiguousarray(first_embed, np.float32)
        self.ctx.check(self.lib.ds_cuda_decoder_generate(self.ctx.h, self.id, _a(fe), n_steps, _a(toks)),
                       "decoder_generate")
        return toks

    def generate_dev(self, n_steps, stream=None):
        self.ctx.check(self.lib.ds_cuda_decoder_generate_dev(self.ctx.h, self.id, n_steps, stream),
                       "decoder_generate_dev")

    @property
    def launches_per_step(self):
        return self.ctx.check(self.lib.ds_cuda_decoder_launches_per_step(self.ctx.h, self.id), "launches")

    def set_sampling(self, repeat_penalty=1.0, no_repeat_ngram_size=0, temperature=0.0):
        """The reference's ctx->repeat_penalty / no_repeat_ngram_size /
        temperature (ds_moe_decoder.c:1021-1263); defaults: greedy argmax."""
        self.ctx.check(self.lib.ds_cuda_decoder_set_sampling(self.ctx.h, self.id, repeat_penalty,
                                                             no_repeat_ngram_size, temperature),
                       "decoder_set_sampling")

    def set_history(self, tokens):
        """Replace the generated-token history (ctx->token_history)."""
        t = np.ascontiguousarray(tokens, np.int32)
        self.ctx.check(self.lib.ds_cuda_decoder_set_history(self.ctx.h, self.id, _a(t) if t.size else None, t.size),
                       "decoder_set_history")

    def history(self):
        n = self.ctx.check(self.lib.ds_cuda_decoder_get_history(self.ctx.h, self.id, None, 0), "decoder_get_history")
        out = np.empty(n, np.int32)
        if n:
            self.ctx.check(self.lib.ds_cuda_decoder_get_history(self.ctx.h, self.id, _a(out), n),
                           "decoder_get_history")
        return out

    def set_window(self, sliding_window_size, prefill_token_count):
        """V3's reference sliding-window attention (0 disables)."""
        self.ctx.check(self.lib.ds_cuda_decoder_set_window(self.ctx.h, self.id, sliding_window_size,
                                                           prefill_token_count), "decoder_set_window")

    def set_uniforms(self, u):
        """Uniforms for temperature sampling, one per sampled step."""
        u = np.ascontiguousarray(u, np.float32)
        self.ctx.check(self.lib.ds_cuda_decoder_set_uniforms(self.ctx.h, self.id, _a(u) if u.size else None, u.size),
                       "decoder_set_uniforms")

    def close(self):
        if self.id and self.ctx.h:
            self.lib.ds_cuda_decoder_destroy(self.ctx.h, self.id)
            self.id = 0


class BatchDecoder:
    """Greedy decode of n_streams independent streams at once (the
    multi-stream decode of config 3): forward(embeds) advances every stream
    by one token. Streams have their own KV caches and positions."""

    def __init__(self, model, n_streams, ctx=None, kv_max=1024):
        self.ctx = ctx or Context(0)
        self.lib = self.ctx.lib
        self.model = model
        self.S = n_streams
        d = model.d
        self.cfg = DecoderConfig(d.hidden, d.n_layers, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter,
                                 d.n_experts, d.n_shared, d.top_k, d.vocab, d.first_dense, synth.RMS_EPS,
                                 synth.ROPE_THETA, kv_max, 0, 0)
        self._layers = (LayerWeightsC * d.n_layers)(*[layer_struct(lw) for lw in model.layers])
        for lw in model.layers:
            self.ctx._pin(lw.wq, lw.wk, lw.wv, lw.wo, lw.input_norm, lw.post_norm, lw.dense_gate, lw.dense_up,
                          lw.dense_down)
            if lw.moe is not None:
                self.ctx._pin(lw.moe.router, lw.moe.block, lw.moe.down, lw.moe.shared_down)
        self.ctx._pin(model.final_norm, model.lm_head)
        self.id = self.ctx.check(self.lib.ds_cuda_batch_decoder_create(
            self.ctx.h, ctypes.byref(self.cfg), self._layers, _a(model.final_norm), _a(model.lm_head), n_streams),
            "batch_decoder_create")

    def load_kv(self, stream, ks, vs, pos0=0):
        for l, (k, v) in enumerate(zip(ks, vs)):
            k = np.ascontiguousarray(k, np.float32)
            v = np.ascontiguousarray(v, np.float32)
            if k.shape[0]:
                self.ctx.check(self.lib.ds_cuda_batch_decoder_load_kv(self.ctx.h, self.id, stream, l, pos0,
                                                                      k.shape[0], _a(k), _a(v)), "batch_load_kv")
        self.set_len(stream, pos0 + ks[0].shape[0])

    def set_len(self, stream, n):
        self.ctx.check(self.lib.ds_cuda_batch_decoder_set_len(self.ctx.h, self.id, stream, n), "batch_set_len")

    def forward(self, embeds=None, want_x=False):
        toks = np.empty(self.S, np.int32)
        fx = np.empty((self.S, self.model.d.hidden), np.float32) if want_x else None
        e = None if embeds is None else np.ascontiguousarray(embeds, np.float32)
        self.ctx.check(self.lib.ds_cuda_batch_decoder_forward(self.ctx.h, self.id, _a(e), _a(toks), _a(fx)),
                       "batch_forward")
        return (toks, fx) if want_x else toks

    def generate(self, n_steps, first_embeds=None):
        toks = np.empty((n_steps, self.S), np.int32)
        e = None if first_embeds is None else np.ascontiguousarray(first_embeds, np.float32)
        self.ctx.check(self.lib.ds_cuda_batch_decoder_generate(self.ctx.h, self.id, _a(e), n_steps, _a(toks)),
                       "batch_generate")
        return toks

    def generate_dev(self, n_steps, stream=None):
        self.ctx.check(self.lib.ds_cuda_batch_decoder_generate_dev(self.ctx.h, self.id, n_steps, stream),
                       "batch_generate_dev")

    def set_sampling(self, repeat_penalty=1.0, no_repeat_ngram_size=0, temperature=0.0):
        """The reference's repeat_penalty / no_repeat_ngram_size /
        temperature (ds_moe_decoder.c:1021-1263) for every stream."""
        self.ctx.check(self.lib.ds_cuda_batch_decoder_set_sampling(self.ctx.h, self.id, repeat_penalty,
                                                                   no_repeat_ngram_size, temperature),
                       "batch_set_sampling")

    def set_history(self, stream, tokens):
        """Replace one stream's generated-token history."""
        t = np.ascontiguousarray(tokens, np.int32)
        self.ctx.check(self.lib.ds_cuda_batch_decoder_set_history(self.ctx.h, self.id, stream,
                                                                  _a(t) if t.size else None, t.size),
                       "batch_set_history")

    def history(self, stream):
        n = self.ctx.check(self.lib.ds_cuda_batch_decoder_get_history(self.ctx.h, self.id, stream, None, 0),
                           "batch_get_history")
        out = np.empty(n, np.int32)
        if n:
            self.ctx.check(self.lib.ds_cuda_batch_decoder_get_history(self.ctx.h, self.id, stream, _a(out), n),
                           "batch_get_history")
        return out

    def set_uniforms(self, u):
        """Uniforms for temperature sampling: [n_streams x n], row s for
        stream s, one per sampled step."""
        u = np.ascontiguousarray(u, np.float32)
        assert u.ndim == 2 and u.shape[0] == self.S
        self.ctx.check(self.lib.ds_cuda_batch_decoder_set_uniforms(self.ctx.h, self.id, _a(u) if u.size else None,
                                                                   u.shape[1]), "batch_set_uniforms")

    def set_window(self, sliding_window_size, prefill_token_counts):
        """V3's reference sliding-window attention (0 disables), with each
        stream's prefill length."""
        p = np.ascontiguousarray(prefill_token_counts, np.int32)
        assert p.size == self.S
        self.ctx.check(self.lib.ds_cuda_batch_decoder_set_window(self.ctx.h, self.id, sliding_window_size, _a(p)),
                       "batch_set_window")

    def close(self):
        if self.id:
            self.lib.ds_cuda_batch_decoder_destroy(self.ctx.h, self.id)
            self.id = 0
