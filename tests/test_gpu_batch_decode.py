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
