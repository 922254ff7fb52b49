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


class _SelfDist:
    @staticmethod
    def all_to_all_single(out, inp, out_splits=None, in_splits=None):
        out.copy_(inp)


def test_ep_one_rank_path_matches_prefill(cuda_ctx):
    # the expert-parallel code path (dispatch, pairs, payload rows, combine
    # through the return index) at one rank equals the fused single-GPU call
    import torch
    from ds_ocr_b200 import synth
    from ds_ocr_b200.ep import CudaStages, ExpertParallelPrefill
    from ds_ocr_b200.prefill import Prefill
    model = synth.Model(n_layers=2, vocab=256)
    x, lg = _inputs(model.d)
    ref = x.copy()
    idx_ref, w_ref = Prefill(model.d, cuda_ctx).moe_layer(model.layers[1], ref, lg)
    st = CudaStages(model.d, cuda_ctx)
    ep = ExpertParallelPrefill(model.d, st, _SelfDist, 0, 1, st.device)
    with torch.cuda.stream(st.stream):
        tx = torch.from_numpy(x).to(st.device)
        tl = torch.from_numpy(lg).to(st.device)
    idx, w = ep.moe_layer(model.layers[1], tx, tl)
    st.check()
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert np.array_equal(tx.cpu().numpy(), ref)


@pytest.mark.parametrize("n", [300, 3000])
def test_dispatch_and_pairs_kernels(cuda_ctx, n):
    # the bookkeeping kernels against the CPU stand-in's reading of the same
    # contract, for 4 ranks of 16 experts (3000 tokens: several tokens and
    # rows per thread)
    import torch
    from test_ep_cpu import StandInStages
    from ds_ocr_b200 import synth
    from ds_ocr_b200.ep import CudaStages
    model = synth.Model(n_layers=2, vocab=256)
    st = CudaStages(model.d, cuda_ctx)
    K, H, G = model.d.top_k, model.d.hidden, 4
    rng = np.random.default_rng(3)
    idx = np.stack([rng.choice(64, K, replace=False) for _ in range(n)]).astype(np.int32)
    idx[:20] = np.arange(K)  # all on rank 0
    hi = rng.integers(-30000, 30000, (n, H)).astype(np.int16)
    lo = rng.integers(-30000, 30000, (n, H)).astype(np.int16)
    with torch.cuda.stream(st.stream):
        t_idx, t_hi, t_lo = (torch.from_numpy(a).to(st.device) for a in (idx, hi, lo))
        payload, counts, inv = st.dispatch(t_idx, t_hi, t_lo, G, 64 // G)
    ref = StandInStages()
    import test_ep_cpu as T
    saved = T.K, T.H
    T.K, T.H = K, H  # the stand-in reads the shapes from its module
    try:
        r_payload, r_counts, r_inv = ref.dispatch(torch.from_numpy(idx), torch.from_numpy(hi), torch.from_numpy(lo),
                                                  G, 64 // G)
        # the payload as if each destination's section had come from a
        # different rank (the offsets in a row are relative to its section)
        recv = list(r_counts[:G])
        rpr, rpe, rper = ref.pairs(r_payload, recv)
    finally:
        T.K, T.H = saved
    assert counts == r_counts
    rows = sum(counts[:G])
    assert torch.equal(payload[:rows].cpu(), r_payload)
    assert torch.equal(inv[:n * K].cpu(), r_inv)
    pr, pe, per = st.pairs(payload[:rows], recv)
    assert torch.equal(pr.cpu(), rpr) and torch.equal(pe.cpu(), rpe) and per == rper


def test_native_ep_one_rank_matches_prefill(cuda_ctx):
    # the library's own expert-parallel layer (NCCL from C) at one rank:
    # every transfer goes to itself; bit-identical to the fused single-GPU call
    import torch
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from ds_ocr_b200 import synth
    from ds_ocr_b200.ep import NativeExpertParallelPrefill
    from ds_ocr_b200.prefill import Prefill
    model = synth.Model(n_layers=3, vocab=256)
    x, lg = _inputs(model.d)
    ref = x.copy()
    for l in (1, 2):
        idx_ref, _ = Prefill(model.d, cuda_ctx).moe_layer(model.layers[l], ref, lg)
    ep = NativeExpertParallelPrefill(model.d, cuda_ctx, 0, 1, NativeExpertParallelPrefill.unique_id(cuda_ctx))
    try:
        tx = torch.from_numpy(x).cuda()
        tl = torch.from_numpy(lg).cuda()
        torch.cuda.synchronize()
        pf = Prefill(model.d, cuda_ctx)
        pf.timing(True)  # the per-stage events cover the expert-parallel layer too
        for l in (1, 2):
            idx, _ = ep.moe_layer(model.layers[l], tx, tl)
        cuda_ctx.synchronize()
        ms = pf.stage_ms()
        assert all(np.isfinite(ms)) and min(ms) >= 0
        pf.timing(False)
    finally:
        ep.close()
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert np.array_equal(tx.cpu().numpy(), ref)


def _native_rank(rank, world, q_uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    from ds_ocr_b200 import cuda, synth
    from ds_ocr_b200.ep import NativeExpertParallelPrefill, token_range
    torch.cuda.set_device(rank)
    ctx = cuda.Context(rank)
    try:
        model = synth.Model(n_layers=3, vocab=256)
        if rank == 0:
            uid = NativeExpertParallelPrefill.unique_id(ctx)
            for _ in range(world - 1):
                q_uid.put(uid)
        else:
            uid = q_uid.get(timeout=120)
        ep = NativeExpertParallelPrefill(model.d, ctx, rank, world, uid)
        x, lg = _inputs(model.d)
        a, b = token_range(N_TOKENS, rank, world)
        xl = torch.from_numpy(x[a:b].copy()).cuda()
        for l in (1, 2):
            ll = torch.from_numpy(lg[a:b].copy()).cuda()
            idx, _ = ep.moe_layer(model.layers[l], xl, ll)
        ctx.synchronize()
        q.put((rank, xl.cpu().numpy(), idx.cpu().numpy()))
        ep.close()
    except Exception as e:  # reported to the parent instead of a silent hang
        q.put((rank, None, repr(e)))
        raise
    finally:
        ctx.close()


def test_native_ep_two_gpus_bit_identical_to_one():
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
    q, q_uid = mpc.Queue(), mpc.Queue()
    procs = [mpc.Process(target=_native_rank, args=(r, 2, q_uid, q)) for r in range(2)]
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
    assert np.array_equal(np.concatenate([got[0][1], got[1][1]]), idx_ref)
    assert np.array_equal(np.concatenate([got[0][0], got[1][0]]), ref)
