"""Expert-parallel prefill on 2 GPUs (NCCL all-to-all between the stage
kernels) against the single-GPU prefill: bit-identical outputs and routing.
Skipped where fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
N_TOKENS = 700


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(d):
    from ds_ocr_b200 import synth
    x = synth.normal_f32((N_TOKENS, d.hidden), 21)
    lg = synth.normal_f32((N_TOKENS, d.n_experts), 22) + 0.5 * synth.normal_f32(d.n_experts, 23)[None, :]
    lg[:50, :8] += 30.0  # tokens whose experts all live on rank 0
    return x, lg


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from ds_ocr_b200 import cuda, synth
    from ds_ocr_b200.ep import CudaStages, ExpertParallelPrefill, token_range
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        model = synth.Model(n_layers=3, vocab=256)
        ctx = cuda.Context(rank)
        st = CudaStages(model.d, ctx)
        ep = ExpertParallelPrefill(model.d, st, dist, rank, world, st.device)
        x, lg = _inputs(model.d)
        a, b = token_range(N_TOKENS, rank, world)
        xl = torch.from_numpy(x[a:b].copy()).cuda()
        for l in (1, 2):
            ll = torch.from_numpy(lg[a:b].copy()).cuda()
            idx, w = ep.moe_layer(model.layers[l], xl, ll)
        st.check()
        q.put((rank, xl.cpu().numpy(), idx.cpu().numpy()))
        dist.barrier()
        ctx.close()
    except Exception as e:  # reported to the parent instead of a silent hang
        q.put((rank, None, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_bit_identical_to_one():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from ds_ocr_b200 import cuda, synth
    from ds_ocr_b200.prefill import Prefill
    model = synth.Model(n_layers=3, vocab=256)
    x, lg = _inputs(model.d)
    ref = x.copy()
    ctx = cuda.Context(0)
    pf = Prefill(model.d, ctx)
    for l in (1, 2):
        idx_ref, _ = pf.moe_layer(model.layers[l], ref, lg)
    ctx.close()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, xl, idx = q.get(timeout=240)
        assert xl is not None, f"rank {r}: {idx}"
        got[r] = (xl, idx)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out = np.concatenate([got[0][0], got[1][0]])
    idx = np.concatenate([got[0][1], got[1][1]])
    assert np.array_equal(idx, idx_ref)
    assert np.array_equal(out, ref)
