"""Batched MoE prefill through the ds_cuda C ABI: the MoE block of the
reference's ds_decoder_prefill (ds_moe_decoder.c:630-809) for n tokens at
once, x += MoE(RMSNorm(x)) per layer, on the tensor cores.

`Prefill.moe_layer(lw, x, logits)` mirrors one pass of that block on host
arrays (x is updated in place, like the reference's x); `moe_layer_dev`
runs it on device buffers (torch tensors or raw device addresses) without
synchronising, for timing.
"""
import ctypes

import numpy as np

from . import synth
from .cuda import Context, _a
from .decoder import DecoderConfig, layer_struct


class Prefill:
    def __init__(self, d, ctx=None):
        self.ctx = ctx or Context(0)
        self.lib = self.ctx.lib
        self.d = d
        self.cfg = DecoderConfig(d.hidden, d.n_layers, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter,
                                 d.n_experts, d.n_shared, d.top_k, d.vocab, d.first_dense, synth.RMS_EPS,
                                 synth.ROPE_THETA, 0, 0, 0)
        self._structs = {}

    def _layer(self, lw):
        s = self._structs.get(id(lw))
        if s is None:
            m = lw.moe
            self.ctx._pin(lw.post_norm, m.router, m.block, m.down, m.shared_down)
            s = self._structs[id(lw)] = (lw, layer_struct(lw))
        return ctypes.byref(s[1])

    def moe_layer(self, lw, x, logits=None):
        """x [n x hidden] F32 (updated in place); logits [n x n_experts] or
        None (router scores from the weights). Returns (top_idx, top_w)."""
        assert x.dtype == np.float32 and x.flags.c_contiguous
        n = x.shape[0]
        k = self.d.top_k
        idx = np.empty((n, k), np.int32)
        w = np.empty((n, k), np.float32)
        lg = None if logits is None else np.ascontiguousarray(logits, np.float32)
        self.ctx.check(self.lib.ds_cuda_prefill_moe(self.ctx.h, ctypes.byref(self.cfg), self._layer(lw), _a(x), n,
                                                    _a(lg), _a(idx), _a(w)), "prefill_moe")
        return idx, w

    def moe_layer_dev(self, lw, d_x, n, d_logits=None, d_idx=None, d_w=None, stream=None):
        """Device-buffer variant (addresses as ints); enqueued only."""
        self.ctx.check(self.lib.ds_cuda_prefill_moe_dev(self.ctx.h, ctypes.byref(self.cfg), self._layer(lw), d_x, n,
                                                        d_logits, d_idx, d_w, stream), "prefill_moe_dev")

    def timing(self, enable=True):
        self.ctx.check(self.lib.ds_cuda_prefill_timing(self.ctx.h, int(enable)), "prefill_timing")

    def stage_ms(self):
        """The last call's stage times (ms): norm+route, plan, scatter,
        gate/up GEMM, down GEMM, combine."""
        out = np.zeros(6, np.float32)
        self.ctx.check(self.lib.ds_cuda_prefill_stage_ms(self.ctx.h, _a(out)), "prefill_stage_ms")
        return out

    def check(self):
        """Synchronise and raise if a prefill kernel's bounded wait gave up."""
        self.ctx.check(self.lib.ds_cuda_prefill_check(self.ctx.h), "prefill_check")
