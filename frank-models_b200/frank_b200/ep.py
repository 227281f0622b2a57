"""Expert parallelism for the MoE FFN block: one process per GPU, NCCL
all-to-all over NVLink/NVSwitch.

The reference has no distribution (its MoE block runs on one device); this
layer splits the experts of ``moe_ffn_block`` (components/moe/
moe_ffn_block.mlir:34-209) evenly over P ranks.  Every rank holds its own
tokens; a step is

 1. router + softmax + top-k on the local tokens            (local kernels)
 2. stable expert permutation: because the experts of a rank are
    contiguous, expert-sorted rows are already grouped by destination rank
 3. all-to-all of the per-(rank, local expert) row counts   (NCCL)
 4. grouped NCCL send/recv of the bf16 token rows and their gate weights,
    one chunk per (peer, local expert), each received straight into its
    expert-major position, then the local experts' grouped GEMMs
 5. the fp32 output rows go back chunk for chunk (NCCL send/recv) into the
    sender's expert-sorted order
 6. combine the k rows of every local token in slot order (local kernel)

Each token row is processed by exactly the same kernels with the same
accumulation order as on one GPU, so the result equals the single-GPU
result bit for bit.  The row counts are read on the host once per step
(they size the all-to-all-v).

The device primitives are reached through ``prims`` (default: the C ABI
via :mod:`frank_b200.ops`) so that the host-side exchange logic can be
exercised on CPU ranks (gloo) with stand-in primitives in tests.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist


@dataclass
class Segments:
    """Row segments of one exchange direction (host int64 arrays)."""

    src_start: np.ndarray
    dst_start: np.ndarray
    length: np.ndarray

    @property
    def prefix(self) -> np.ndarray:
        p = np.zeros(self.length.size + 1, dtype=np.int64)
        np.cumsum(self.length, out=p[1:])
        return p


def plan_exchange(send_cnt: np.ndarray, recv_cnt: np.ndarray):
    """Host-side plan of one step's exchange.

    send_cnt[p, e]: rows this rank sends to rank p for p's local expert e
    (in its expert-sorted order); recv_cnt[p, e]: rows this rank receives
    from rank p for its own local expert e.  Returns
      send_splits, recv_splits  -- rows per peer for the all-to-all-v
      to_expert_major           -- Segments: received (source-major) rows ->
                                   expert-major rows
      local_offsets             -- [E_l + 1] expert row offsets (expert-major)
    The reverse direction uses to_expert_major with src/dst swapped.
    """
    send_cnt = np.asarray(send_cnt, dtype=np.int64)
    recv_cnt = np.asarray(recv_cnt, dtype=np.int64)
    P, El = recv_cnt.shape
    send_splits = send_cnt.sum(axis=1)
    recv_splits = recv_cnt.sum(axis=1)
    # source-major position of (p, e): rank p's block, then expert e inside it
    src_block = np.zeros(P, dtype=np.int64)
    np.cumsum(recv_splits[:-1], out=src_block[1:])
    within_src = np.zeros((P, El), dtype=np.int64)
    np.cumsum(recv_cnt[:, :-1], axis=1, out=within_src[:, 1:])
    src_start = src_block[:, None] + within_src
    # expert-major position of (p, e): expert e's block, then source p inside it
    per_expert = recv_cnt.sum(axis=0)
    local_offsets = np.zeros(El + 1, dtype=np.int64)
    np.cumsum(per_expert, out=local_offsets[1:])
    within_e = np.zeros((P, El), dtype=np.int64)
    np.cumsum(recv_cnt[:-1, :], axis=0, out=within_e[1:, :])
    dst_start = local_offsets[None, :El] + within_e
    seg = Segments(src_start.reshape(-1), dst_start.reshape(-1), recv_cnt.reshape(-1))
    return send_splits, recv_splits, seg, local_offsets


class CudaPrims:
    """Device primitives backed by the C ABI (libfrankmoe.so)."""

    def __init__(self):
        from . import ops

        self.ops = ops

    def route(self, x, wr, k, normalize):
        return self.ops.router_topk(x, wr, k, normalize)

    def permute(self, ids, E):
        ss, off, pos, _ = self.ops.permute(ids, E)
        return ss, off, pos

    def gather(self, x, w, sorted_slots):
        return self.ops.gather_rows(x, sorted_slots), self.ops.gather_weights(w.reshape(-1), sorted_slots)

    def expert_ffn(self, xs, w_rows, offsets, w_up, w_gate, w_down, out):
        return self.ops.expert_ffn(xs, w_rows, offsets, w_up, w_gate, w_down, out=out)

    def combine(self, d, slot_pos, T, k, out):
        return self.ops.combine(d, slot_pos, T, k, out)


class ExpertParallelMoE:
    """The MoE FFN block with the experts split over the ranks of ``group``.

    wr: full router [E, H]; w_*_local: this rank's packed experts
    ([E/P, F, H] up/gate, [E/P, H, F] down), i.e. experts
    [rank*E/P, (rank+1)*E/P).
    """

    def __init__(self, wr, w_up_local, w_gate_local, w_down_local, n_expert: int, n_expert_used: int,
                 normalize_weights: bool, group=None, prims=None, out_dtype=torch.float32):
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_expert % self.P:
            raise ValueError(f"n_expert={n_expert} is not divisible by the {self.P} ranks")
        self.E, self.k, self.normalize = int(n_expert), int(n_expert_used), bool(normalize_weights)
        self.El = self.E // self.P
        self.wr = wr
        self.w_up, self.w_gate, self.w_down = w_up_local, w_gate_local, w_down_local
        if w_up_local.shape[0] != self.El:
            raise ValueError(f"rank {self.rank} holds {w_up_local.shape[0]} experts, expected {self.El}")
        self.H, self.F = w_down_local.shape[1], w_down_local.shape[2]
        self.prims = prims if prims is not None else CudaPrims()
        self.out_dtype = out_dtype
        self.last_plan = None

    @classmethod
    def synthetic(cls, cfg, rank, world, device, seed=0, group=None):
        """Seeded synthetic weights of configuration ``cfg``; every rank draws
        the full set with the same seed and keeps its own experts."""
        from . import configs

        wr, wu, wg, wd = configs.block_weights_packed_torch(cfg, device, seed=seed)
        El = cfg.E // world
        sl = slice(rank * El, (rank + 1) * El)
        wu, wg, wd = (w[sl].contiguous() for w in (wu, wg, wd))
        torch.cuda.empty_cache()
        return cls(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize, group=group)

    def _exchange(self, send_buf, recv_buf, send_chunks, recv_chunks):
        """Grouped point-to-point exchange of row chunks.  send_chunks[p] /
        recv_chunks[p] list (start, length) row ranges for peer p, in the
        same (local expert) order on both sides; zero-length chunks are
        skipped on both sides alike.  The rank's own chunks are copied
        locally."""
        ops = []
        for p in range(self.P):
            if p == self.rank:
                for (s0, n), (d0, m) in zip(send_chunks[p], recv_chunks[p]):
                    if n:
                        recv_buf[d0:d0 + m].copy_(send_buf[s0:s0 + n])
                continue
            peer = dist.get_global_rank(self.group, p) if self.group is not None else p
            for s0, n in send_chunks[p]:
                if n:
                    ops.append(dist.P2POp(dist.isend, send_buf[s0:s0 + n], peer, self.group))
            for d0, m in recv_chunks[p]:
                if m:
                    ops.append(dist.P2POp(dist.irecv, recv_buf[d0:d0 + m], peer, self.group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x.shape
        dev = x.device
        pr = self.prims
        w, ids = pr.route(x, self.wr, self.k, self.normalize)
        sorted_slots, offsets, slot_pos = pr.permute(ids, self.E)
        xs, ws = pr.gather(x, w, sorted_slots)
        # per-(destination rank, its local expert) counts
        cnt = (offsets[1:] - offsets[:-1]).to(torch.int64).reshape(self.P, self.El)
        recv_cnt_t = torch.empty_like(cnt)
        dist.all_to_all_single(recv_cnt_t, cnt.contiguous(), group=self.group)
        both = torch.stack([cnt, recv_cnt_t]).cpu().numpy()  # the one host sync per step
        send_cnt, recv_cnt = both[0], both[1]
        _, recv_splits, seg, local_off = plan_exchange(send_cnt, recv_cnt)
        self.last_plan = (send_cnt, recv_cnt)
        R = int(recv_splits.sum())
        n = xs.shape[0]
        # my expert-sorted rows for (p, e) are contiguous at the global expert offset
        send_start = np.zeros(self.P * self.El + 1, dtype=np.int64)
        np.cumsum(send_cnt.reshape(-1), out=send_start[1:])
        send_chunks = [[(int(send_start[p * self.El + e]), int(send_cnt[p, e])) for e in range(self.El)]
                       for p in range(self.P)]
        # received rows land directly in expert-major order
        dst = seg.dst_start.reshape(self.P, self.El)
        recv_chunks = [[(int(dst[p, e]), int(recv_cnt[p, e])) for e in range(self.El)] for p in range(self.P)]
        xl = torch.empty((R, H), dtype=xs.dtype, device=dev)
        wl = torch.empty((R,), dtype=torch.float32, device=dev)
        self._exchange(xs, xl, send_chunks, recv_chunks)
        self._exchange(ws, wl, send_chunks, recv_chunks)
        dl = torch.empty((R, H), dtype=torch.float32, device=dev)
        offs = torch.from_numpy(local_off.astype(np.int32)).to(dev, non_blocking=True)
        if R:
            pr.expert_ffn(xl, wl, offs, self.w_up, self.w_gate, self.w_down, dl)
        # results go back chunk for chunk into this rank's expert-sorted order
        ret = torch.empty((n, H), dtype=torch.float32, device=dev)
        self._exchange(dl, ret, recv_chunks, send_chunks)
        y = out if out is not None else torch.empty((T, H), dtype=self.out_dtype, device=dev)
        pr.combine(ret, slot_pos, T, self.k, y)
        return y
