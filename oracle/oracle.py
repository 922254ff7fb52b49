"""Python binding of the CPU oracle (liboracle.so) and of the compiled
reference (oracle/_ref/libdsref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, always as the checker or the timed CPU
baseline, never as the product path.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdsref.so")
P = ctypes.c_void_p
c_int, c_float = ctypes.c_int, ctypes.c_float


def build_oracle():
    subprocess.check_call(["make", "-s", "-C", HERE, "liboracle.so"])


def reference_dir():
    """Where the reference's source tree lies: $DS_REFERENCE_DIR, else the
    `reference_path` that BASELINE.json at the repo root names, else None."""
    d = os.environ.get("DS_REFERENCE_DIR")
    if d:
        return d
    try:
        import json
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            return json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None


def build_ref(ref_dir=None):
    """Compile the reference from its own sources (needs the reference tree)."""
    ref_dir = ref_dir or reference_dir()
    if not ref_dir or not os.path.isdir(ref_dir):
        return False
    subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF={ref_dir}"])
    return True


def addr(a):
    return None if a is None else a.ctypes.data


class Dims(ctypes.Structure):
    _fields_ = [(n, c_int) for n in ("hidden", "n_heads", "head_dim", "inter_dense", "moe_inter", "n_experts",
                                      "n_shared", "top_k", "vocab", "n_layers", "first_dense")] + \
               [("eps", c_float), ("theta", c_float), ("simulate_bf16", c_int), ("renorm_topk", c_int)]


class Layer(ctypes.Structure):
    _fields_ = [(n, P) for n in ("wq", "wk", "wv", "wo", "input_norm", "post_norm", "dense_gate", "dense_up",
                                 "dense_down", "router", "expert_block", "down", "shared_down",
                                 "gu_q", "gu_scale", "gu_off", "dn_q", "dn_scale", "dn_off",
                                 "sgu_q", "sgu_scale", "sgu_off", "sdn_q", "sdn_scale", "sdn_off")]


def make_dims(d, simulate=0, renorm=0):
    return Dims(d.hidden, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter, d.n_experts, d.n_shared, d.top_k,
                d.vocab, d.n_layers, d.first_dense, 1e-6, 10000.0, simulate, renorm)


def make_layer(lw):
    """orc_layer_t for a ds_ocr_b200.synth.LayerWeights (keeps no references:
    the caller must keep lw alive)."""
    L = Layer()
    for n in ("wq", "wk", "wv", "wo", "input_norm", "post_norm", "dense_gate", "dense_up", "dense_down"):
        setattr(L, n, addr(getattr(lw, n)))
    m = lw.moe
    if m is not None:
        L.router, L.expert_block, L.down, L.shared_down = addr(m.router), addr(m.block), addr(m.down), addr(m.shared_down)
        q = m.int8
        if q is not None:
            for n in ("gu_q", "dn_q", "sgu_q", "sdn_q"):
                setattr(L, n, addr(getattr(q, n)))
            for a, b in (("gu_scale", "gu_s"), ("gu_off", "gu_o"), ("dn_scale", "dn_s"), ("dn_off", "dn_o"),
                         ("sgu_scale", "sgu_s"), ("sgu_off", "sgu_o"), ("sdn_scale", "sdn_s"), ("sdn_off", "sdn_o")):
                setattr(L, a, addr(getattr(q, b)))
    return L


_orc = None


def oracle():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            build_oracle()
        o = ctypes.CDLL(ORACLE_SO)
        sig = {
            "orc_fast_expf": (c_float, [c_float]),
            "orc_bf16_roundtrip": (c_float, [c_float]),
            "orc_matvec_bf16": (None, [P, P, P, c_int, c_int]),
            "orc_dot_bf16_row": (c_float, [P, P, c_int, c_int]),
            "orc_argmax_bf16": (c_int, [P, P, c_int, c_int, P]),
            "orc_router_topk": (None, [P, c_int, c_int, c_int, P, P]),
            "orc_swiglu": (None, [P, P, P, c_int]),
            "orc_expert_fused": (None, [P, P, P, P, c_int, c_int, c_int]),
            "orc_int8_quantize": (c_int, [P, c_int, c_int, P, P, P]),
            "orc_int8_matvec": (None, [P, P, P, P, P, c_int, c_int]),
            "orc_expert_fused_int8": (None, [P, P, P, P, P, P, P, P, c_int, c_int, c_int]),
            "orc_moe_forward": (None, [P, P, P, P, c_int, P, P]),
            "orc_rms_norm": (None, [P, P, P, c_int, c_float]),
            "orc_residual_rms_norm": (None, [P, P, P, P, P, c_int, c_float]),
            "orc_rope_table": (None, [P, P, c_int, c_int, c_float]),
            "orc_apply_rope": (None, [P, P, P, c_int, c_int]),
            "orc_attention_decode": (None, [P, P, P, P, c_int, c_int, c_int, c_int, c_float]),
            "orc_decoder_step": (c_int, [P, P, P, P, P, P, c_int, c_int, P, P, c_int, P, P, P]),
            "orc_prefill_moe": (None, [P, P, P, c_int, P, P, P]),
            "orc_decoder_step_swa": (c_int, [P, P, P, P, P, P, c_int, c_int, P, P, c_int, P, P, P, c_int, c_int]),
            "orc_decoder_prefill": (c_int, [P, P, P, P, P, P, c_int, c_int, P, P, P, c_int, P, P]),
            "orc_lm_select": (c_int, [P, P, c_int, c_int, P, c_int, c_float, c_int, c_float, c_float, P, P]),
        }
        for k, (r, a) in sig.items():
            f = getattr(o, k)
            f.restype, f.argtypes = r, a
        _orc = o
    return _orc


_ref = None


def ref_available():
    return os.path.exists(REF_SO)


def ref():
    """The compiled, unmodified reference (plus harness). Raises if absent."""
    global _ref
    if _ref is None:
        r = ctypes.CDLL(REF_SO)
        sig = {
            "ref_set_threads": (None, [c_int]),
            "ref_get_threads": (c_int, []),
            "ref_set_simulate": (None, [c_int]),
            "ref_layer_slot_count": (c_int, []),
            "ref_ctx_new": (P, [c_int, c_int, c_int]),
            "ref_ctx_set_layer": (None, [P, c_int, P]),
            "ref_ctx_set_head": (None, [P, P, P]),
            "ref_ctx_quantize": (c_int, [P]),
            "ref_ctx_int8_block": (c_int, [P, c_int, c_int, c_int, P, P, P]),
            "ref_ctx_kv_set": (None, [P, c_int, c_int, c_int, P, P]),
            "ref_ctx_kv_get": (None, [P, c_int, c_int, c_int, P, P]),
            "ref_ctx_set_len": (None, [P, c_int]),
            "ref_ctx_get_len": (c_int, [P]),
            "ref_decoder_step": (c_int, [P, P, P, P]),
            "ref_layer_forward": (None, [P, c_int, P, P]),
            "ref_moe_forward": (None, [P, c_int, P, P]),
            "ref_argmax": (c_int, [P, P, c_int, c_int, P]),
            "ref_matvec": (None, [P, P, P, c_int, c_int]),
            "ref_rms_norm": (None, [P, P, P, c_int, c_int]),
            "ref_quantize": (c_int, [P, c_int, c_int, P, P, P]),
            "ref_int8_matvec": (None, [P, P, P, P, P, c_int, c_int]),
            "ref_fast_expf": (c_float, [c_float]),
            "ref_prefill_moe": (None, [P, c_int, P, c_int, P, P, P]),
            "ref_ctx_free": (None, [P]),
            "ref_ctx_set_sampling": (None, [P, c_float, c_int, c_float]),
            "ref_ctx_set_history": (c_int, [P, P, c_int]),
            "ref_ctx_get_history": (c_int, [P, P, c_int]),
            "ref_decoder_step_gen": (c_int, [P, P]),
            "ref_srand": (None, [ctypes.c_uint]),
            "ref_ctx_set_window": (None, [P, c_int, c_int]),
            "ref_decoder_prefill": (c_int, [P, P, c_int, P]),
            "ref_st_count": (c_int, [ctypes.c_char_p]),
            "ref_st_find": (c_int, [ctypes.c_char_p, ctypes.c_char_p, P, P, P, P, P]),
        }
        for k, (res, a) in sig.items():
            f = getattr(r, k)
            f.restype, f.argtypes = res, a
        _ref = r
    return _ref


class RefDecoder:
    """A reference ds_ctx_t built on a ds_ocr_b200.synth.Model's weights."""

    def __init__(self, model, kv_max=4096, threads=1):
        r = ref()
        self.r = r
        self.model = model
        r.ref_set_threads(threads)
        d = model.d
        self.ctx = r.ref_ctx_new(d.n_layers, kv_max, d.vocab)
        n = r.ref_layer_slot_count()
        self._keep = []
        for l, lw in enumerate(model.layers):
            self.set_layer(l, lw)
        r.ref_ctx_set_head(self.ctx, addr(model.final_norm), addr(model.lm_head))

    def set_layer(self, l, lw):
        """Point reference layer l at a synth.LayerWeights (or at a bare
        synth.MoeWeights, for MoE-only use)."""
        m = getattr(lw, "moe", None) if not hasattr(lw, "block") else lw
        g = (lambda n: addr(getattr(lw, n, None)))
        ptrs = [g("wq"), g("wk"), g("wv"), g("wo"), g("input_norm"), g("post_norm"),
                g("dense_gate"), g("dense_up"), g("dense_down"),
                addr(m.router) if m else None, addr(m.block) if m else None, addr(m.down) if m else None,
                addr(m.shared_down) if m else None]
        arr = (ctypes.c_void_p * self.r.ref_layer_slot_count())(*ptrs)
        self._keep.append(arr)
        self.r.ref_ctx_set_layer(self.ctx, l, arr)

    def load_kv(self, ks, vs):
        for l, (k, v) in enumerate(zip(ks, vs)):
            self.r.ref_ctx_kv_set(self.ctx, l, 0, k.shape[0], addr(k), addr(v))
        self.r.ref_ctx_set_len(self.ctx, ks[0].shape[0])

    def step(self, embed):
        fx = np.empty(self.model.d.hidden, np.float32)
        lg = np.empty(1, np.float32)
        tok = self.r.ref_decoder_step(self.ctx, addr(embed), addr(fx), addr(lg))
        return tok, fx, float(lg[0])

    def set_sampling(self, repeat_penalty=1.0, no_repeat_ngram_size=0, temperature=0.0):
        self.r.ref_ctx_set_sampling(self.ctx, repeat_penalty, no_repeat_ngram_size, temperature)

    def set_history(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        assert self.r.ref_ctx_set_history(self.ctx, addr(t) if t.size else None, t.size) == 0

    def history(self):
        out = np.empty(self.r.ref_ctx_get_history(self.ctx, None, 0), np.int32)
        self.r.ref_ctx_get_history(self.ctx, addr(out), out.size)
        return out

    def prefill(self, embeds):
        """ds_decoder_prefill on [T x hidden] embeddings: (first token, logit)."""
        e = np.ascontiguousarray(embeds, np.float32)
        lg = np.empty(1, np.float32)
        tok = self.r.ref_decoder_prefill(self.ctx, addr(e), e.shape[0], addr(lg))
        return tok, float(lg[0])

    def kv(self, layer, pos0, n):
        kd = self.model.d.n_heads * self.model.d.head_dim
        k = np.empty((n, kd), np.float32)
        v = np.empty((n, kd), np.float32)
        self.r.ref_ctx_kv_get(self.ctx, layer, pos0, n, addr(k), addr(v))
        return k, v

    def set_window(self, sliding_window_size, prefill_token_count):
        """V3's reference sliding-window attention (ds_moe_decoder.c:409-436)."""
        self.r.ref_ctx_set_window(self.ctx, sliding_window_size, prefill_token_count)

    def step_gen(self, embed):
        """A generation-loop step: decode, then append the token to the history."""
        return self.r.ref_decoder_step_gen(self.ctx, addr(embed))

    def moe_forward(self, layer, x):
        out = np.empty(self.model.d.hidden, np.float32)
        self.r.ref_moe_forward(self.ctx, layer, addr(out), addr(x))
        return out

    def quantize(self):
        """--int4: quantise every MoE layer with the reference's quantiser and
        copy the blocks into each layer's Int8Moe."""
        from ds_ocr_b200.synth import Int8Moe
        self.r.ref_ctx_quantize(self.ctx)
        d = self.model.d
        H, I, S = d.hidden, d.moe_inter, d.shared_inter
        for l, lw in enumerate(self.model.layers):
            if lw.moe is None:
                continue
            q = Int8Moe(d)
            for e in range(d.n_experts):
                self.r.ref_ctx_int8_block(self.ctx, l, 0, e, addr(q.gu_q[e * 2 * I * H:]), addr(q.gu_s[e * 2 * I:]),
                                          addr(q.gu_o[e * 2 * I:]))
                self.r.ref_ctx_int8_block(self.ctx, l, 1, e, addr(q.dn_q[e * H * I:]), addr(q.dn_s[e * H:]),
                                          addr(q.dn_o[e * H:]))
            self.r.ref_ctx_int8_block(self.ctx, l, 2, 0, addr(q.sgu_q), addr(q.sgu_s), addr(q.sgu_o))
            self.r.ref_ctx_int8_block(self.ctx, l, 3, 0, addr(q.sdn_q), addr(q.sdn_s), addr(q.sdn_o))
            lw.moe.int8 = q

    def prefill_moe(self, layer, x, logits=None):
        d = self.model.d
        n = x.shape[0]
        idx = np.empty((n, d.top_k), np.int32)
        w = np.empty((n, d.top_k), np.float32)
        self.r.ref_prefill_moe(self.ctx, layer, addr(x), n, addr(logits), addr(idx), addr(w))
        return idx, w

    def close(self):
        if self.ctx:
            self.r.ref_ctx_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OracleDecoder:
    """The oracle's decoder step on a synth.Model, KV as F32 [L][kv_max][H]."""

    def __init__(self, model, kv_max=4096, simulate=0, renorm=0):
        self.o = oracle()
        self.model = model
        d = model.d
        self.dims = make_dims(d, simulate, renorm)
        self.refresh()
        kd = d.n_heads * d.head_dim
        self.kv_max = kv_max
        self.k = np.zeros((d.n_layers, kv_max, kd), np.float32)
        self.v = np.zeros((d.n_layers, kv_max, kd), np.float32)
        self.cos = np.empty((kv_max, d.head_dim), np.float32)
        self.sin = np.empty((kv_max, d.head_dim), np.float32)
        self.o.orc_rope_table(addr(self.cos), addr(self.sin), kv_max, d.head_dim, 10000.0)
        self.pos = 0

    def refresh(self):
        """Rebuild the layer descriptors (after weights gained an INT8 copy)."""
        self.layers = (Layer * self.model.d.n_layers)(*[make_layer(lw) for lw in self.model.layers])

    def load_kv(self, ks, vs):
        n = ks[0].shape[0]
        for l in range(len(ks)):
            self.k[l, :n] = ks[l]
            self.v[l, :n] = vs[l]
        self.pos = n

    window = 0    # V3 sliding window (0: full causal attention)
    ref_len = 0   # prefill length the window keeps

    def step(self, embed, use_int8=False):
        d = self.model.d
        if use_int8:
            self.refresh()
        fx = np.empty(d.hidden, np.float32)
        lg = np.empty(1, np.float32)
        tok = self.o.orc_decoder_step_swa(self.layers, ctypes.byref(self.dims), addr(self.model.final_norm),
                                          addr(self.model.lm_head), addr(self.k), addr(self.v), self.kv_max,
                                          self.pos, addr(self.cos), addr(self.sin), int(use_int8), addr(embed),
                                          addr(fx), addr(lg), self.window, self.ref_len)
        self.pos += 1
        return tok, fx, float(lg[0])

    def prefill(self, embeds):
        """The oracle's ds_decoder_prefill on [T x hidden] embeddings at the
        current position: (first token, last normed row, logit)."""
        d = self.model.d
        e = np.ascontiguousarray(embeds, np.float32)
        lx = np.empty(d.hidden, np.float32)
        lg = np.empty(1, np.float32)
        tok = self.o.orc_decoder_prefill(self.layers, ctypes.byref(self.dims), addr(self.model.final_norm),
                                         addr(self.model.lm_head), addr(self.k), addr(self.v), self.kv_max, self.pos,
                                         addr(self.cos), addr(self.sin), addr(e), e.shape[0], addr(lx), addr(lg))
        self.pos += e.shape[0]
        return tok, lx, float(lg[0])

    def select(self, final_x, history, repeat_penalty=1.0, no_repeat_ngram_size=0, temperature=0.0, r=0.0):
        """LM-head selection with the sampling settings on a final hidden state:
        (token, value, full_path)."""
        d = self.model.d
        h = np.ascontiguousarray(history, np.int32)
        val = np.empty(1, np.float32)
        full = np.empty(1, np.int32)
        tok = self.o.orc_lm_select(addr(final_x), addr(self.model.lm_head), d.hidden, d.vocab,
                                   addr(h) if h.size else None, h.size, repeat_penalty, no_repeat_ngram_size,
                                   temperature, r, addr(val), addr(full))
        return tok, float(val[0]), bool(full[0])

    def moe_forward(self, layer, x, use_int8=False):
        d = self.model.d
        if use_int8:
            self.refresh()
        out = np.empty(d.hidden, np.float32)
        idx = np.empty(d.top_k, np.int32)
        w = np.empty(d.top_k, np.float32)
        self.o.orc_moe_forward(addr(out), addr(x), ctypes.byref(self.layers[layer]), ctypes.byref(self.dims),
                               int(use_int8), addr(idx), addr(w))
        return out, idx, w

    def prefill_moe(self, layer, x, logits=None):
        d = self.model.d
        n = x.shape[0]
        idx = np.empty((n, d.top_k), np.int32)
        w = np.empty((n, d.top_k), np.float32)
        self.o.orc_prefill_moe(ctypes.byref(self.layers[layer]), ctypes.byref(self.dims), addr(x), n, addr(logits),
                               addr(idx), addr(w))
        return idx, w
