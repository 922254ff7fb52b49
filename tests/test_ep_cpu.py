"""Expert-parallel prefill host logic (dispatch, return, combine order) on
CPU: two gloo ranks with numpy-like stand-in stages must reproduce the
single-rank result bit for bit, including tokens whose experts all live on
the other rank and a rank that owns no tokens' experts at all."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ds_ocr_b200 import synth
from ds_ocr_b200.ep import ExpertParallelPrefill, token_range

H, E, K = 64, 8, 3


class StandInStages:
    """Deterministic CPU versions of route / experts / combine with the
    kernels' data layout: split BF16 planes, per-pair outputs, combine in
    ascending expert order with FMA-free float32 arithmetic."""

    def route(self, lw, x, logits):
        xn = x / torch.sqrt((x * x).mean(dim=1, keepdim=True) + 1e-6)
        hi = xn.to(torch.bfloat16)
        lo = (xn - hi.float()).to(torch.bfloat16)
        p = torch.softmax(logits, dim=1)
        w, idx = torch.topk(p, K, dim=1)
        return hi.view(torch.int16), lo.view(torch.int16), idx.to(torch.int32), w

    @staticmethod
    def _val(hi, lo):
        return hi.view(torch.bfloat16).float() + lo.view(torch.bfloat16).float()

    def dispatch(self, idx, hi, lo, G, e_per):
        n = idx.shape[0]
        dest = idx.long() // e_per
        rows, tok, meta, inv = [], [], [], torch.zeros(n * K, dtype=torch.int32)
        counts, pairs = [0] * G, [0] * G
        base = 0
        for g in range(G):
            for s_ in range(n):
                ks = [k for k in range(K) if dest[s_, k] == g]
                if not ks:
                    continue
                counts[g] += 1
                # expert ids of this destination, then in the last slot the
                # row's first pair within the destination's pairs
                m = [int(idx[s_, k]) if k in ks else -1 for k in range(K)] + [-1] * (7 - K) + [pairs[g]]
                rows.append(torch.cat([hi[s_], lo[s_], torch.tensor(m, dtype=torch.int32).view(torch.int16)]))
                for k in ks:
                    inv[s_ * K + k] = base
                    base += 1
                    pairs[g] += 1
        payload = torch.stack(rows) if rows else torch.zeros((1, 2 * H + 16), dtype=torch.int16)
        return payload, counts + pairs, inv

    def pairs(self, payload, recv_counts):
        R = payload.shape[0]
        meta = payload[:, 2 * H:].contiguous().view(torch.int32)[:, :K] if R else torch.zeros((0, K), dtype=torch.int32)
        src = torch.repeat_interleave(torch.arange(len(recv_counts)), torch.tensor(recv_counts))
        valid = meta >= 0
        pr = torch.nonzero(valid)[:, 0].to(torch.int32)
        pe = meta[valid].to(torch.int32)
        per = torch.bincount(src[pr.long()], minlength=len(recv_counts)).tolist() if pr.numel() else [0] * len(recv_counts)
        return pr, pe, per

    def experts(self, lw, rows_hi, rows_lo, rows_ld, pair_row, pair_expert, sh_hi, sh_lo):
        v = self._val(rows_hi[:, :H].contiguous(), rows_lo[:, :H].contiguous())[pair_row.long()]
        e = pair_expert.float()[:, None]
        y = torch.tanh(v * (e + 1.0) + 0.1 * e)
        ys = 0.5 * self._val(sh_hi, sh_lo)
        return y, ys

    def combine(self, x, idx, w, y, y_row, ys):
        n = x.shape[0]
        order = torch.argsort(idx, dim=1, stable=True)
        acc = torch.zeros_like(x)
        for j in range(K):
            k = order[:, j]
            rows = torch.arange(n) * K + k
            if y_row is not None:
                rows = y_row[rows].long()
            acc = acc + w[torch.arange(n), k][:, None] * y[rows]
        x += acc + ys


class SelfDist:
    """torch.distributed stand-in for one rank (all-to-all is a copy)."""

    @staticmethod
    def all_to_all_single(out, inp, out_splits=None, in_splits=None):
        out.copy_(inp)


def inputs(n):
    x = torch.from_numpy(synth.normal_f32((n, H), 11))
    lg = torch.from_numpy(synth.normal_f32((n, E), 12))
    lg[: n // 4, :E // 2] += 20.0      # first quarter: experts of rank 0 only
    lg[n // 4: n // 2, E // 2:] += 20.0  # second quarter: experts of rank 1 only
    return x, lg


class D:
    hidden, n_experts, top_k = H, E, K


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, lg = inputs(n)
    a, b = token_range(n, rank, world)
    ep = ExpertParallelPrefill(D, StandInStages(), dist, rank, world, torch.device("cpu"))
    xl = x[a:b].clone()
    idx, w = ep.moe_layer(None, xl, lg[a:b].contiguous())
    pairs, imbalance = ep.load()
    q.put((rank, xl, idx, pairs, imbalance))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("n", [40, 7])
def test_two_ranks_match_one(n):
    x, lg = inputs(n)
    ref = x.clone()
    ExpertParallelPrefill(D, StandInStages(), SelfDist, 0, 1, torch.device("cpu")).moe_layer(None, ref, lg)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    got, loads = dict(), dict()
    for _ in range(2):
        r, xl, idx, pairs, imbalance = q.get(timeout=120)
        got[r] = xl
        loads[r] = (pairs, imbalance)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out = torch.cat([got[0], got[1]])
    assert torch.equal(out, ref)
    assert not torch.equal(out, x)
    # the load report: both ranks see the same counts, every (token, slot)
    # pair computed exactly once, imbalance = max / mean
    assert loads[0] == loads[1]
    pairs, imbalance = loads[0]
    assert sum(pairs) == n * K
    assert imbalance == pytest.approx(max(pairs) / (sum(pairs) / 2))
