"""ds_cuda_moe_experts_noalloc: the expert chain for callers that cannot
allocate device memory (a plugin that is only handed device buffers, a
process with a fixed device-memory budget). The test owns every buffer; the
entry point must give the same result as ds_cuda_moe_experts, on two calls
in a row (the second reuses the static scratch the first one left behind).
Collected last on purpose: a failure here does not hide any other test."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2
from ds_ocr_b200 import cuda, synth

pytestmark = pytest.mark.gpu
H, I = 1280, 896


def test_noalloc_matches_moe_experts(orc):
    import torch
    ctx = cuda.Context(0)
    lib = ctx.lib
    try:
        mw = synth.MoeWeights(synth.Dims(), 7)
        ctx.register(mw.block)
        ctx.register(mw.down)
        for call, (experts, seed) in enumerate((([3, 17, 40, 5, 63, 22], 11), ([9, 1, 50], 12))):
            x = synth.normal_f32(H, seed)
            w = np.linspace(0.3, 0.05, len(experts)).astype(np.float32)
            gus = [mw.expert_gate_up(e) for e in experts]
            dns = [mw.expert_down(e) for e in experts]
            ref = ctx.moe_experts(x, gus, dns, w, H, I)
            k = len(experts)
            dgu = (ctypes.c_void_p * k)(*[ctx.device_ptr(g) for g in gus])
            ddn = (ctypes.c_void_p * k)(*[ctx.device_ptr(d) for d in dns])
            assert all(dgu) and all(ddn)
            tx = torch.from_numpy(x).cuda()
            tout = torch.full((H,), float("nan"), device="cuda")
            torch.cuda.synchronize()
            rc = lib.ds_cuda_moe_experts_noalloc(tx.data_ptr(), dgu, ddn, w.ctypes.data, k, H, I,
                                                 tout.data_ptr(), None)
            assert rc == 0, f"call {call}"
            torch.cuda.synchronize()
            assert rel_l2(tout.cpu().numpy(), ref) < 1e-6, f"call {call}"
            # and against the CPU oracle: sum_k w_k * ds_expert_forward_fused
            # (ds_kernels.c:322-357, combine :359-371)
            want = np.zeros(H, np.float32)
            y = np.empty(H, np.float32)
            for g, d, wk in zip(gus, dns, w):
                orc.orc_expert_fused(y.ctypes.data, x.ctypes.data, g.ctypes.data, d.ctypes.data, H, I, 0)
                want += np.float32(wk) * y
            assert rel_l2(tout.cpu().numpy(), want) < 1e-5, f"call {call}"
        # 8 experts of 1792 rows pass the per-argument limits but need 14336
        # floats of scratch: refused by the 12288-float bound
        assert lib.ds_cuda_moe_experts_noalloc(tx.data_ptr(), dgu, ddn, w.ctypes.data, 8, H, 1792,
                                               tout.data_ptr(), None) < 0
        # per-argument limits: inter beyond 2048, top_k beyond 8
        assert lib.ds_cuda_moe_experts_noalloc(tx.data_ptr(), dgu, ddn, w.ctypes.data, 1, H, 2056,
                                               tout.data_ptr(), None) < 0
        assert lib.ds_cuda_moe_experts_noalloc(tx.data_ptr(), dgu, ddn, w.ctypes.data, 9, H, 8,
                                               tout.data_ptr(), None) < 0
    finally:
        ctx.close()
