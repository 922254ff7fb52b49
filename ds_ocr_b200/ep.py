"""Expert-parallel batched MoE prefill over the GPUs of one box.

The reference runs the prefill MoE block (ds_moe_decoder.c:630-809) on one
host. Here G ranks (one process per GPU, torch.distributed over NCCL) split
the work:
  * tokens are split evenly by index: rank r owns rows [r*n/G, (r+1)*n/G);
  * experts are split into contiguous blocks: rank r runs experts
    [r*E/G, (r+1)*E/G); the shared expert is replicated and runs on each
    rank's own tokens.
Per layer:
  1. route      (local): RMSNorm into two BF16 planes, softmax/top-k;
  2. dispatch   (all-to-all): each token's split row goes once to every rank
                that owns one of its experts, with the list of those experts;
  3. experts    (local): the grouped tensor-core GEMMs over the received
                (row, expert) pairs, plus the shared expert on local rows;
  4. return     (all-to-all): one output row per (token, expert) back to the
                token's rank, in the order it asked for them;
  5. combine    (local): x += sum over the token's experts in ascending
                order of w * y, plus shared, the same arithmetic as one GPU,
                so the result is bit-identical to the single-GPU path.
Counts travel first (all-to-all of G integers) so every rank knows its
receive sizes. The stage kernels come from `stages` (CudaStages below for
the product; the CPU tests pass a numpy stand-in with the same interface).
"""
import ctypes

from . import synth
from .decoder import DecoderConfig, layer_struct


class CudaStages:
    """The three prefill stages of the C ABI on torch device tensors."""

    def __init__(self, d, ctx):
        import torch
        self.torch = torch
        self.ctx = ctx
        self.lib = ctx.lib
        self.d = d
        self.cfg = DecoderConfig(d.hidden, d.n_layers, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter,
                                 d.n_experts, d.n_shared, d.top_k, d.vocab, d.first_dense, synth.RMS_EPS,
                                 synth.ROPE_THETA, 0, 0, 0)
        self._structs = {}
        self.device = torch.device("cuda", ctx.device)
        # a torch-owned stream: the stage kernels, the bookkeeping tensor ops
        # and the collectives all run in its order
        self.stream = torch.cuda.Stream(self.device)

    def _st(self):
        return self.stream.cuda_stream

    def _layer(self, lw):
        s = self._structs.get(id(lw))
        if s is None:
            m = lw.moe
            self.ctx._pin(lw.post_norm, m.router, m.block, m.down, m.shared_down)
            s = self._structs[id(lw)] = (lw, layer_struct(lw))
        return ctypes.byref(s[1])

    @staticmethod
    def _p(t):
        return None if t is None or t.numel() == 0 else t.data_ptr()

    def route(self, lw, x, logits):
        torch = self.torch
        n, H, K = x.shape[0], self.d.hidden, self.d.top_k
        hi = torch.empty((n, H), dtype=torch.int16, device=self.device)
        lo = torch.empty((n, H), dtype=torch.int16, device=self.device)
        idx = torch.empty((n, K), dtype=torch.int32, device=self.device)
        w = torch.empty((n, K), dtype=torch.float32, device=self.device)
        self.ctx.check(self.lib.ds_cuda_prefill_route_dev(self.ctx.h, ctypes.byref(self.cfg), self._layer(lw),
                                                          self._p(x), n, self._p(logits), self._p(hi), self._p(lo),
                                                          self._p(idx), self._p(w), self._st()), "prefill_route")
        return hi, lo, idx, w

    def dispatch(self, idx, hi, lo, n_ranks, e_per):
        """Pack this rank's rows for the other ranks. Returns (payload
        [rows x (2H + 16)] int16, send_tok, counts [2G] on the host: rows
        then pairs per destination, inv [n*K])."""
        torch = self.torch
        n, K, H = idx.shape[0], self.d.top_k, self.d.hidden
        cap = max(1, n * min(K, n_ranks))
        payload = torch.empty((cap, 2 * H + 16), dtype=torch.int16, device=self.device)
        send_tok = torch.empty(cap, dtype=torch.int32, device=self.device)
        counts = torch.empty(2 * n_ranks, dtype=torch.int32, device=self.device)
        inv = torch.empty(max(1, n * K), dtype=torch.int32, device=self.device)
        self.ctx.check(self.lib.ds_cuda_ep_dispatch_dev(self.ctx.h, n, K, n_ranks, e_per, self._p(idx), self._p(hi),
                                                        self._p(lo), H, payload.data_ptr(), send_tok.data_ptr(),
                                                        counts.data_ptr(), inv.data_ptr(), self._st()),
                       "ep_dispatch")
        self.stream.synchronize()  # the host read below, whatever the caller's current stream
        return payload, counts.tolist(), inv

    def pairs(self, payload, recv_counts):
        """(row, expert) pairs of the received payload rows; returns
        (pair_row, pair_expert, pairs per source rank on the host)."""
        torch = self.torch
        R, K, G = payload.shape[0], self.d.top_k, len(recv_counts)
        pr = torch.empty(max(1, R * K), dtype=torch.int32, device=self.device)
        pe = torch.empty(max(1, R * K), dtype=torch.int32, device=self.device)
        out = torch.empty(G + 1, dtype=torch.int32, device=self.device)
        rc = (ctypes.c_int * G)(*recv_counts)
        self.ctx.check(self.lib.ds_cuda_ep_pairs_dev(self.ctx.h, R, K, G, rc, self._p(payload), self.d.hidden,
                                                     pr.data_ptr(), pe.data_ptr(), out.data_ptr(), self._st()),
                       "ep_pairs")
        self.stream.synchronize()
        o = out.tolist()
        return pr[:o[G]], pe[:o[G]], o[:G]

    def experts(self, lw, rows_hi, rows_lo, rows_ld, pair_row, pair_expert, sh_hi, sh_lo):
        torch = self.torch
        H = self.d.hidden
        P, S = pair_row.shape[0], sh_hi.shape[0]
        y = torch.empty((P, H), dtype=torch.float32, device=self.device)
        ys = torch.empty((S, H), dtype=torch.float32, device=self.device)
        self.ctx.check(self.lib.ds_cuda_prefill_experts_dev(
            self.ctx.h, ctypes.byref(self.cfg), self._layer(lw), self._p(rows_hi), self._p(rows_lo), rows_ld,
            rows_hi.shape[0], self._p(pair_row), self._p(pair_expert), P, self._p(y), self._p(sh_hi),
            self._p(sh_lo), S, self._p(ys), self._st()), "prefill_experts")
        return y, ys

    def combine(self, x, idx, w, y, y_row, ys):
        self.ctx.check(self.lib.ds_cuda_prefill_combine_dev(self.ctx.h, ctypes.byref(self.cfg), self._p(x),
                                                            x.shape[0], self._p(idx), self._p(w), self._p(y),
                                                            self._p(y_row), self._p(ys), self._st()),
                       "prefill_combine")

    def check(self):
        self.stream.synchronize()
        self.ctx.check(self.lib.ds_cuda_prefill_check(self.ctx.h), "prefill_check")


def token_range(n, rank, world):
    return n * rank // world, n * (rank + 1) // world


class ExpertParallelPrefill:
    """One rank of the expert-parallel prefill. `dist` is torch.distributed
    with an initialised process group; `stages` runs the kernels."""

    def __init__(self, d, stages, dist, rank, world, device):
        import torch
        self.torch = torch
        self.d = d
        self.st = stages
        self.dist = dist
        self.rank, self.world = rank, world
        self.device = device
        if d.n_experts % world:
            raise ValueError(f"{d.n_experts} experts do not split over {world} ranks")
        self.e_per = d.n_experts // world
        self.pairs_done = 0  # (row, expert) pairs this rank's experts computed

    def _a2a(self, send, send_counts, recv_counts):
        """all-to-all(v) along dim 0 (counts are host lists of rows)."""
        torch = self.torch
        out = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(out, send.contiguous(), recv_counts, send_counts)
        return out

    def _counts(self, counts):
        torch = self.torch
        c = torch.tensor(counts, dtype=torch.int64, device=self.device)
        r = torch.empty_like(c)
        self.dist.all_to_all_single(r, c)
        return r.tolist()

    def load(self):
        """Expert work per rank since construction: the (row, expert) pairs
        each rank computed, and the imbalance max / mean (1.0 = even).
        Collective: every rank calls it."""
        torch = self.torch
        mine = torch.tensor([self.pairs_done], dtype=torch.int64, device=self.device)
        every = [torch.empty_like(mine) for _ in range(self.world)]
        self.dist.all_gather(every, mine)
        pairs = [int(t.item()) for t in every]
        mean = sum(pairs) / len(pairs)
        return pairs, (max(pairs) / mean if mean > 0 else 1.0)

    def moe_layer(self, lw, x, logits):
        """x [n_local x H] F32 (this rank's tokens, updated in place);
        logits [n_local x E] or None. Returns (idx, w) of the local tokens.
        Runs on the stages' stream (made current here); callers order their
        own work on x against it."""
        s = getattr(self.st, "stream", None)
        if s is None:
            return self._moe_layer(lw, x, logits)
        with self.torch.cuda.stream(s):
            return self._moe_layer(lw, x, logits)

    def _moe_layer(self, lw, x, logits):
        torch = self.torch
        G, H = self.world, self.d.hidden
        hi, lo, idx, w = self.st.route(lw, x, logits)
        # dispatch: one payload row per (token, owning rank)
        payload, counts, inv = self.st.dispatch(idx, hi, lo, G, self.e_per)
        send_rows, back_recv = counts[:G], counts[G:]
        recv_rows = self._counts(send_rows)
        width = payload.shape[1] // 2  # payload rows travel as int32
        r_payload = self._a2a(payload[:sum(send_rows)].view(torch.int32), send_rows, recv_rows)
        r_payload = r_payload.view(torch.int16).reshape(-1, 2 * width)
        # local experts over the received pairs; the shared expert on local rows
        pair_row, pair_expert, back_send = self.st.pairs(r_payload, recv_rows)
        self.pairs_done += int(pair_row.shape[0])
        y, ys = self.st.experts(lw, r_payload, r_payload[:, H:], 2 * width, pair_row, pair_expert, hi, lo)
        # outputs return in request order; inv locates each (token, k)
        y_back = self._a2a(y, back_send, back_recv)
        self.st.combine(x, idx, w, y_back, inv, ys)
        return idx, w


class NativeExpertParallelPrefill:
    """One rank of the expert-parallel prefill run inside the library
    (ds_cuda_prefill_moe_ep: dispatch and return over NCCL from C, no
    torch.distributed on the data path). `uid` is the 128-byte id from
    unique_id() on rank 0, shared with the other ranks out of band."""

    @staticmethod
    def unique_id(ctx):
        buf = ctypes.create_string_buffer(128)
        ctx.check(ctx.lib.ds_cuda_ep_unique_id(ctx.h, buf), "ep_unique_id")
        return buf.raw

    def __init__(self, d, ctx, rank, world, uid):
        self.d, self.ctx, self.rank, self.world = d, ctx, rank, world
        self.cfg = DecoderConfig(d.hidden, d.n_layers, d.n_heads, d.head_dim, d.dense_inter, d.moe_inter,
                                 d.n_experts, d.n_shared, d.top_k, d.vocab, d.first_dense, synth.RMS_EPS,
                                 synth.ROPE_THETA, 0, 0, 0)
        self._structs = {}
        self._uid = ctypes.create_string_buffer(bytes(uid), 128)
        ctx.check(ctx.lib.ds_cuda_ep_init(ctx.h, rank, world, self._uid), "ep_init")

    def _layer(self, lw):
        s = self._structs.get(id(lw))
        if s is None:
            m = lw.moe
            self.ctx._pin(lw.post_norm, m.router, m.block, m.down, m.shared_down)
            s = self._structs[id(lw)] = (lw, layer_struct(lw))
        return ctypes.byref(s[1])

    def moe_layer(self, lw, x, logits=None, stream=None):
        """x: this rank's [n x H] F32 rows (torch CUDA tensor, updated in
        place); logits [n x E] or None. Returns (idx, w) device tensors."""
        import torch
        n, K = x.shape[0], self.d.top_k
        idx = torch.empty((n, K), dtype=torch.int32, device=x.device)
        w = torch.empty((n, K), dtype=torch.float32, device=x.device)
        self.ctx.check(self.ctx.lib.ds_cuda_prefill_moe_ep(
            self.ctx.h, ctypes.byref(self.cfg), self._layer(lw), x.data_ptr(), n,
            None if logits is None else logits.data_ptr(), idx.data_ptr(), w.data_ptr(), stream), "prefill_moe_ep")
        return idx, w

    def close(self):
        self.ctx.lib.ds_cuda_ep_free(self.ctx.h)
