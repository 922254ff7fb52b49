"""Python view of the ds_cuda C ABI (include/ds_cuda.h).

`Context` mirrors the reference's Metal offload context (ds_metal.h) and the
CUDA entry points with the ds_kernels / ds_quantize signatures. Arrays are
numpy host arrays; every call raises DsCudaError on a negative status, with
ds_cuda_last_error()'s message. There is no CPU fallback.
"""
import ctypes

import numpy as np

from ._lib import DsCudaError, load


def _a(x):
    return None if x is None else x.ctypes.data


def _f32(x):
    x = np.ascontiguousarray(x, np.float32)
    return x


class Int8Block(ctypes.Structure):
    """ds_cuda_int8_block_t == the reference's ds_int4_block_t layout."""
    _fields_ = [("qweight", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("offset", ctypes.c_void_p),
                ("out_dim", ctypes.c_int), ("in_dim", ctypes.c_int), ("bytes", ctypes.c_size_t)]

    @classmethod
    def of(cls, q, s, o, out_dim, in_dim):
        return cls(q.ctypes.data, s.ctypes.data, o.ctypes.data, out_dim, in_dim, out_dim * in_dim + 8 * out_dim)


class Context:
    def __init__(self, device=0):
        self.lib = load()
        self.device = device
        self.h = self.lib.ds_cuda_init(device)
        if not self.h:
            raise DsCudaError("ds_cuda_init failed: no usable sm_100 CUDA device")
        self._keep = []

    def close(self):
        if self.h:
            self.lib.ds_cuda_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc, what=""):
        if rc < 0:
            raise DsCudaError(f"{what} failed ({rc}): {self.lib.ds_cuda_last_error(self.h).decode()}")
        return rc

    @property
    def stream(self):
        return self.lib.ds_cuda_stream(self.h)

    def synchronize(self):
        self.check(self.lib.ds_cuda_synchronize(self.h), "synchronize")

    def set_numerics(self, simulate_bf16=0, renorm_topk=0):
        self.check(self.lib.ds_cuda_set_numerics(self.h, int(simulate_bf16), int(renorm_topk)), "set_numerics")

    # -- registration ------------------------------------------------------
    def register(self, arr):
        """Copy a host array to HBM (keyed by its address); keeps it alive."""
        self._keep.append(arr)
        if arr.dtype == np.uint16:
            rc = self.lib.ds_cuda_register_bf16(self.h, _a(arr), arr.size)
        elif arr.dtype == np.float32:
            rc = self.lib.ds_cuda_register_f32(self.h, _a(arr), arr.size)
        else:
            rc = self.lib.ds_cuda_register_expert_block(self.h, _a(arr), arr.nbytes)
        return self.check(rc, "register")

    def unregister(self, arr):
        rc = self.check(self.lib.ds_cuda_unregister(self.h, _a(arr)), "unregister")
        self._keep = [a for a in self._keep if a is not arr]
        return rc

    def _pin(self, *arrs):
        """Weights passed by pointer are registered on first use and keyed by
        host address: keep them alive so the address cannot be reused."""
        for a in arrs:
            if a is not None and not any(a is k for k in self._keep[-64:]):
                self._keep.append(a)

    def device_ptr(self, arr):
        return self.lib.ds_cuda_device_ptr(self.h, _a(arr))

    @property
    def registered_bytes(self):
        return self.lib.ds_cuda_registered_bytes(self.h)

    # -- Metal-shaped MoE calls -------------------------------------------
    def moe_experts(self, x, gate_ups, downs, weights, hidden, inter):
        k = len(gate_ups)
        self._pin(*gate_ups, *downs)
        gp = (ctypes.c_void_p * max(k, 1))(*[_a(g) for g in gate_ups])
        dp = (ctypes.c_void_p * max(k, 1))(*[_a(d) for d in downs])
        w = _f32(weights)
        x = _f32(x)
        out = np.empty(hidden, np.float32)
        self.check(self.lib.ds_cuda_moe_experts(self.h, _a(x), gp, dp, _a(w), k, hidden, inter, _a(out)), "moe_experts")
        return out

    def shared_experts(self, x, gate_up, down, hidden, shared_inter, output):
        self._pin(gate_up, down)
        x = _f32(x)
        self.check(self.lib.ds_cuda_shared_experts(self.h, _a(x), _a(gate_up), _a(down), hidden, shared_inter,
                                                   _a(output)), "shared_experts")
        return output

    def expert_forward_fused(self, x, gate_up, down, hidden, inter):
        self._pin(gate_up, down)
        x = _f32(x)
        out = np.empty(hidden, np.float32)
        self.check(self.lib.ds_cuda_expert_forward_fused(self.h, _a(out), _a(x), _a(gate_up), _a(down), hidden,
                                                         inter), "expert_forward_fused")
        return out

    def expert_forward_fused_int4(self, x, gu_block, dn_block, hidden, inter):
        x = _f32(x)
        out = np.empty(hidden, np.float32)
        self.check(self.lib.ds_cuda_expert_forward_fused_int4(self.h, _a(out), _a(x), ctypes.byref(gu_block),
                                                              ctypes.byref(dn_block), hidden, inter),
                   "expert_forward_fused_int4")
        return out

    def moe_layer(self, x, mw, return_routing=False):
        d = mw.d
        self._pin(mw.router, mw.block, mw.down, mw.shared_down)
        x = _f32(x)
        out = np.empty(d.hidden, np.float32)
        idx = np.empty(d.top_k, np.int32)
        w = np.empty(d.top_k, np.float32)
        self.check(self.lib.ds_cuda_moe_layer(self.h, _a(x), _a(out), _a(mw.router), _a(mw.block), _a(mw.down),
                                              _a(mw.shared_down), d.hidden, d.moe_inter, d.shared_inter,
                                              d.n_experts, d.top_k, _a(idx), _a(w)), "moe_layer")
        return (out, idx, w) if return_routing else out

    def moe_layer_int8(self, x, mw, return_routing=False):
        d, q = mw.d, mw.int8
        self._pin(mw.router, *[getattr(q, n) for n in ("gu_q", "gu_s", "gu_o", "dn_q", "dn_s", "dn_o", "sgu_q",
                                                        "sgu_s", "sgu_o", "sdn_q", "sdn_s", "sdn_o")])
        x = _f32(x)
        out = np.empty(d.hidden, np.float32)
        idx = np.empty(d.top_k, np.int32)
        w = np.empty(d.top_k, np.float32)
        self.check(self.lib.ds_cuda_moe_layer_int8(
            self.h, _a(x), _a(out), _a(mw.router), _a(q.gu_q), _a(q.gu_s), _a(q.gu_o), _a(q.dn_q), _a(q.dn_s),
            _a(q.dn_o), _a(q.sgu_q), _a(q.sgu_s), _a(q.sgu_o), _a(q.sdn_q), _a(q.sdn_s), _a(q.sdn_o), d.hidden,
            d.moe_inter, d.shared_inter, d.n_experts, d.top_k, _a(idx), _a(w)), "moe_layer_int8")
        return (out, idx, w) if return_routing else out

    # -- LM head -----------------------------------------------------------
    def argmax_matvec_bf16(self, x, W, in_dim, out_dim):
        self._pin(W)
        x = _f32(x)
        lg = np.empty(1, np.float32)
        tok = self.check(self.lib.ds_cuda_argmax_matvec_bf16(self.h, _a(x), _a(W), in_dim, out_dim, _a(lg)), "argmax")
        return tok, float(lg[0])

    def lm_head_argmax(self, x, W, hidden, vocab):
        self._pin(W)
        x = _f32(x)
        return self.check(self.lib.ds_cuda_lm_head_argmax(self.h, _a(x), _a(W), hidden, vocab), "lm_head_argmax")

    def argmax_batch(self, X, W, in_dim, out_dim):
        self._pin(W)
        X = _f32(X)
        B = X.shape[0]
        tok = np.empty(B, np.int32)
        lg = np.empty(B, np.float32)
        self.check(self.lib.ds_cuda_argmax_matvec_bf16_batch(self.h, _a(X), _a(W), in_dim, out_dim, B, _a(tok),
                                                             _a(lg)), "argmax_batch")
        return tok, lg

    def matvec_bf16(self, x, W, in_dim, out_dim, bias=None):
        self._pin(W, bias)
        x = _f32(x)
        y = np.empty(out_dim, np.float32)
        self.check(self.lib.ds_cuda_matvec_bf16(self.h, _a(y), _a(x), _a(W), _a(bias), in_dim, out_dim), "matvec")
        return y

    def int8_quantize_bf16(self, W, out_dim, in_dim):
        q = np.empty(out_dim * in_dim, np.int8)
        s = np.empty(out_dim, np.float32)
        o = np.empty(out_dim, np.float32)
        self.check(self.lib.ds_cuda_int8_quantize_bf16(self.h, _a(W), out_dim, in_dim, _a(q), _a(s), _a(o)),
                   "int8_quantize")
        return q, s, o
