"""Expert parallelism for the MoE FFN block: one process per GPU, NCCL
all-to-all over NVLink/NVSwitch.

The reference has no distribution (its MoE block runs on one device); this
layer splits the experts of ``moe_ffn_block`` (components/moe/
moe_ffn_block.mlir:34-209) evenly over P ranks.  Every rank holds its own
tokens; a step is

 1. router + softmax + top-k on the local tokens            (local kernels)
 2. stable expert permutation: because the experts of a rank are
    contiguous (in placement order: by default expert ids themselves, or
    a load-balanced placement that renames them first), expert-sorted rows
    are already grouped by destination rank
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
(they size the all-to-all-v, or the peer buffers of the p2p mode).

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


def balanced_placement(load, P: int) -> np.ndarray:
    """Expert placement that evens out the rows the ranks process.

    load[g]: rows routed to global expert g (e.g. from a calibration batch);
    returns the E expert ids in rank-major order: rank p owns
    ``placement[p*E/P:(p+1)*E/P]``.  Greedy longest-processing-time with
    equal expert counts: experts by decreasing load (ties to the lower id)
    each go to the least-loaded rank that still has room (ties to the lower
    rank); each rank's experts are kept in ascending id order.  Deterministic,
    so every rank computes the same placement from the same load."""
    load = np.asarray(load, dtype=np.int64).reshape(-1)
    E = load.size
    if P < 1 or E % P:
        raise ValueError(f"balanced_placement: {E} experts do not split over {P} ranks")
    El = E // P
    order = sorted(range(E), key=lambda g: (-int(load[g]), g))
    rank_load = [0] * P
    owned = [[] for _ in range(P)]
    for g in order:
        p = min((q for q in range(P) if len(owned[q]) < El), key=lambda q: (rank_load[q], q))
        owned[p].append(g)
        rank_load[p] += int(load[g])
    return np.array([g for q in range(P) for g in sorted(owned[q])], dtype=np.int64)


def measure_expert_load(x, wr, k: int, normalize: bool, n_expert: int, group=None, prims=None) -> np.ndarray:
    """Rows every global expert receives from a calibration batch: each rank
    routes its own tokens ``x``; the per-expert counts are summed over the
    ranks of ``group`` (collective: every rank calls it)."""
    pr = prims if prims is not None else CudaPrims()
    _, ids = pr.route(x, wr, k, normalize)
    cnt = torch.bincount(ids.reshape(-1).long(), minlength=n_expert)[:n_expert].to(torch.int64)
    dist.all_reduce(cnt, group=group)
    return cnt.cpu().numpy()


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
    [rank*E/P, (rank+1)*E/P), or with ``placement`` (the E expert ids in
    rank-major order, see :func:`balanced_placement`) the experts
    ``placement[rank*E/P:(rank+1)*E/P]`` in that order.  A placement only
    renames the experts between routing and permutation (ids -> position in
    the placement), so every row meets the same expert weights and the same
    kernels: the output does not change with it, the rows per rank do.
    """

    def __init__(self, wr, w_up_local, w_gate_local, w_down_local, n_expert: int, n_expert_used: int,
                 normalize_weights: bool, group=None, prims=None, out_dtype=torch.float32, mode: str | None = None,
                 step_timeout_s: float | None = None, monitor_group=None, placement=None):
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
        self.placement = None
        self._slot_of = None
        if placement is not None:
            pl = np.asarray(placement, dtype=np.int64).reshape(-1)
            if pl.size != self.E or not np.array_equal(np.sort(pl), np.arange(self.E)):
                raise ValueError(f"placement must be a permutation of the {self.E} expert ids")
            if not np.array_equal(pl, np.arange(self.E)):
                self.placement = pl
                slot_of = np.empty(self.E, dtype=np.int32)
                slot_of[pl] = np.arange(self.E, dtype=np.int32)
                self._slot_of_host = torch.from_numpy(slot_of)
        self.last_plan = None
        self.profile = False       # record CUDA events between the phases of each call
        self._marks = []
        # "p2p": rows move by P2P stores into symmetric (peer-mapped) buffers from
        # the dispatch kernel and the down-GEMM epilogue; "nccl": grouped NCCL
        # send/recv of row chunks (also the path the CPU tests drive).
        if mode is None:
            mode = "p2p" if (prims is None and w_up_local.is_cuda and self.P <= 8) else "nccl"
        if mode not in ("p2p", "nccl"):
            raise ValueError(f"mode must be 'p2p' or 'nccl', got {mode!r}")
        self.mode = mode
        self._symm = None
        # Failure detection.  With step_timeout_s set, every step starts with a
        # host-side presence check of all ranks (a gloo monitored barrier with
        # that deadline): a rank that never joins the step makes the others
        # raise FrankError(FRANK_ETIMEOUT) naming it, before any of this step's
        # kernels or collectives is issued, instead of waiting forever.  A
        # collective that fails later in the step (a peer that died mid-step,
        # ended by the process group's own timeout) raises
        # FrankError(FRANK_ENCCL).  The presence check needs a gloo group: the
        # given monitor_group, the step's own group when that is gloo, or a
        # gloo group created here (collectively: every rank constructs its
        # ExpertParallelMoE at the same point).
        self.step_timeout_s = step_timeout_s
        self.monitor_group = monitor_group
        if step_timeout_s is not None and monitor_group is None:
            if dist.get_backend(group) == "gloo":
                self.monitor_group = group if group is not None else dist.group.WORLD
            else:
                self.monitor_group = dist.new_group(ranks=list(range(dist.get_world_size())), backend="gloo")

    @classmethod
    def synthetic(cls, cfg, rank, world, device, seed=0, group=None, placement=None):
        """Seeded synthetic weights of configuration ``cfg``; every rank draws
        the full set with the same seed and keeps its own experts (those of
        ``placement`` when given)."""
        from . import configs

        wr, wu, wg, wd = configs.block_weights_packed_torch(cfg, device, seed=seed)
        El = cfg.E // world
        if placement is None:
            sl = slice(rank * El, (rank + 1) * El)
        else:
            sl = torch.as_tensor(np.asarray(placement, dtype=np.int64)[rank * El:(rank + 1) * El], device=device)
        wu, wg, wd = (w[sl].contiguous() for w in (wu, wg, wd))
        torch.cuda.empty_cache()
        return cls(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize, group=group, placement=placement)

    def _placed(self, ids: torch.Tensor) -> torch.Tensor:
        """Routed expert ids -> positions in the placement (identity without one)."""
        if self.placement is None:
            return ids
        if self._slot_of is None or self._slot_of.device != ids.device:
            self._slot_of = self._slot_of_host.to(ids.device)
        return self._slot_of[ids.long()].contiguous()

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
            for req in self._comm(dist.batch_isend_irecv, ops):
                self._comm(req.wait)

    # phase boundaries (nccl mode / p2p mode):
    #   route+permute(+gather) | counts (nccl: +plan) | dispatch (p2p: plan + dispatch + host size check, +barrier) | expert GEMMs
    #   | return (p2p: barrier only, the rows went back from the GEMM epilogue) | combine
    PHASES = ("route_permute", "counts_plan", "dispatch", "expert_ffn", "return", "combine")

    def _mark(self):
        if self.profile:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._marks[-1].append(e)

    def rows_received(self) -> int:
        """Rows this rank's experts processed in the most recent call (synchronises)."""
        if self.mode == "p2p" and self._symm is not None:
            return int(self._symm["local_off"][-1].item())
        return int(self.last_plan[1].sum()) if self.last_plan is not None else 0

    def phase_ms(self) -> dict:
        """Mean per-phase milliseconds over the profiled calls since the last read."""
        torch.cuda.synchronize()
        acc = np.zeros(len(self.PHASES))
        calls = [m for m in self._marks if len(m) == len(self.PHASES) + 1]
        for m in calls:
            acc += [m[i].elapsed_time(m[i + 1]) for i in range(len(self.PHASES))]
        self._marks = []
        return dict(zip(self.PHASES, (acc / max(len(calls), 1)).tolist()))

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from ._lib import ETIMEOUT, FrankError

        if self.step_timeout_s is not None:
            import datetime

            try:
                dist.monitored_barrier(group=self.monitor_group,
                                       timeout=datetime.timedelta(seconds=self.step_timeout_s))
            except RuntimeError as e:
                raise FrankError(ETIMEOUT, f"expert-parallel step on rank {self.rank}: a peer did not join within "
                                           f"{self.step_timeout_s} s ({e})") from e
        if self.mode == "p2p":
            return self._call_p2p(x, out)
        return self._call_nccl(x, out)

    def _comm(self, fn, *args, **kwargs):
        """Run one collective of the step; its failure (a peer gone, the
        process group's timeout) becomes FrankError(FRANK_ENCCL)."""
        from ._lib import ENCCL, FrankError

        try:
            return fn(*args, **kwargs)
        except RuntimeError as e:
            raise FrankError(ENCCL, f"expert-parallel step on rank {self.rank}: {fn.__name__} failed ({e})") from e

    # ------------------------------------------------------------ p2p mode --
    def _symmetric(self, T: int, rows: int, dev):
        """Symmetric receive / return buffers: recv_x [cap, H] bf16, recv_w [cap]
        fp32 (cap >= the most rows any rank receives this step), ret [k*Tmax, H]
        fp32 (Tmax >= every rank's token count), hs [cap, F] bf16, and the peer
        addresses of every rank's copy.  ``T`` and ``rows`` are the same on
        every rank (derived from the all-gathered counts), so every rank takes
        the same grow-or-keep decision and the collective allocation below is
        entered by all of them or by none.  Buffers only grow (by 25% headroom)."""
        S = self._symm
        if S is not None and S["T"] >= T and S["cap"] >= rows:
            return S
        import os

        # plain peer mappings only: no multicast object is bound to these buffers
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem

        H, k = self.H, self.k
        T = max(T, S["T"] if S else 0)
        cap = max(rows + rows // 4, S["cap"] if S else 0, 1)
        n = k * T

        def al(b):
            return (b + 255) // 256 * 256

        sizes = [al(cap * H * 2), al(cap * 4), al(n * H * 4)]
        base = [0, sizes[0], sizes[0] + sizes[1]]
        self._symm = None
        torch.cuda.synchronize()
        buf = symm_mem.empty(sum(sizes), dtype=torch.uint8, device=dev)
        grp = self.group if self.group is not None else dist.group.WORLD
        hdl = symm_mem.rendezvous(buf, group=grp.group_name)
        ptrs = [int(p) for p in hdl.buffer_ptrs]
        import ctypes

        arr = lambda vals: (ctypes.c_void_p * self.P)(*vals)  # noqa: E731
        self._symm = {
            "T": T, "buf": buf, "hdl": hdl, "cap": cap, "ret_rows": n,
            "recv_x": buf[base[0]:base[0] + cap * H * 2].view(torch.bfloat16).view(cap, H),
            "recv_w": buf[base[1]:base[1] + cap * 4].view(torch.float32),
            "ret": buf[base[2]:base[2] + n * H * 4].view(torch.float32).view(n, H),
            "peer_x": arr([q + base[0] for q in ptrs]),
            "peer_w": arr([q + base[1] for q in ptrs]),
            "peer_ret": arr([q + base[2] for q in ptrs]),
            "dst_base": torch.empty(self.E, dtype=torch.int32, device=dev),
            "local_off": torch.empty(self.El + 1, dtype=torch.int32, device=dev),
            "row_rank": torch.empty(cap, dtype=torch.int32, device=dev),
            "row_pos": torch.empty(cap, dtype=torch.int32, device=dev),
            "counts": self._counts,  # this step's gathered counts (allocated once, kept across growth)
            "flag": torch.zeros(1, dtype=torch.int32, device=dev),
            "spec_flag": torch.zeros(1, dtype=torch.int32, device=dev),  # refusals of a plan on too small buffers
            "hs": torch.empty(cap * self.F * 2 + 256, dtype=torch.uint8, device=dev),
        }
        return self._symm

    def step_sizes(self, counts: np.ndarray):
        """(max tokens of any rank, max rows any rank receives) from the
        all-gathered per-expert counts [P, E]: rank q routed counts[q].sum()
        = k * T_q slots; rank r receives the column block of its experts."""
        counts = np.asarray(counts, dtype=np.int64)
        t_max = int(counts.sum(axis=1).max()) // self.k
        per_rank = counts.sum(axis=0).reshape(self.P, self.El).sum(axis=1)
        return t_max, int(per_rank.max())

    def _check_tokens(self, t_max: int, T: int):
        if t_max < T:
            from ._lib import ENCCL, FrankError

            raise FrankError(ENCCL, f"expert-parallel step on rank {self.rank}: gathered counts cover {t_max} "
                                    f"tokens per rank, this rank holds {T}")

    def _side_stream(self, dev):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=dev)
            self._counts_host = torch.empty((self.P, self.E), dtype=torch.int32).pin_memory()
        return self._side

    def _barrier(self, flag):
        # stream-ordered: every rank's preceding kernels (and their stores into
        # peer memory) have completed when this collective completes
        self._comm(dist.all_reduce, flag, group=self.group)

    def _call_p2p(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from . import _lib, ops

        T, H = x.shape
        dev = x.device
        lib = _lib.load()
        st = torch.cuda.current_stream().cuda_stream
        if getattr(self, "_counts", None) is None or self._counts.device != dev:
            self._counts = torch.empty((self.P, self.E), dtype=torch.int32, device=dev)
        if self.profile:
            self._marks.append([])
        self._mark()
        if getattr(self, "_wr_pack", None) is None:
            self._wr_pack = ops.router_pack(self.wr)
        w, ids = ops.router_topk(x, self.wr, self.k, self.normalize, pack=self._wr_pack)
        sorted_slots, offsets, slot_pos, _ = ops.permute(self._placed(ids), self.E)
        cnt = (offsets[1:] - offsets[:-1]).contiguous()
        self._mark()
        counts = self._counts
        self._comm(dist.all_gather_into_tensor, counts, cnt, group=self.group)

        def plan_and_dispatch(S, overflow):
            _lib.check(lib.frank_ep_plan(S["counts"].data_ptr(), self.P, self.El, self.rank, S["dst_base"].data_ptr(),
                                         S["local_off"].data_ptr(), S["row_rank"].data_ptr(),
                                         S["row_pos"].data_ptr(), S["cap"], overflow, st))
            _lib.check(lib.frank_ep_dispatch(x.data_ptr(), T, H, w.data_ptr(), sorted_slots.data_ptr(),
                                             offsets.data_ptr(), self.E, self.El, self.k * T,
                                             S["dst_base"].data_ptr(), S["peer_x"], S["peer_w"], self.P, S["cap"],
                                             overflow, st))

        # The buffers must hold this step's rows, which only the gathered
        # counts tell.  From the second step on, the counts are copied to the
        # host on a side stream while the plan and the dispatch already run
        # with the current buffers (rows past a buffer are refused into a
        # scratch word); the host then checks the sizes.  Every rank sees the
        # same counts, so if they do not fit, all ranks wait for the refused
        # dispatch, grow their buffers together and redo plan and dispatch.
        self._mark()
        S = self._symm
        if S is None:
            t_max, rows_max = self.step_sizes(counts.cpu().numpy())
            self._check_tokens(t_max, T)
            S = self._symmetric(t_max, rows_max, dev)
            plan_and_dispatch(S, None)
        else:
            gathered = torch.cuda.Event()
            gathered.record()
            side = self._side_stream(dev)
            side.wait_event(gathered)
            with torch.cuda.stream(side):
                self._counts_host.copy_(counts, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(side)
            plan_and_dispatch(S, S["spec_flag"].data_ptr())
            copied.synchronize()
            t_max, rows_max = self.step_sizes(self._counts_host.numpy())
            self._check_tokens(t_max, T)
            if S["T"] < t_max or S["cap"] < rows_max:
                torch.cuda.synchronize()
                self._comm(dist.barrier, group=self.group)  # every rank's refused dispatch has finished
                S = self._symmetric(t_max, rows_max, dev)
                plan_and_dispatch(S, None)
        self._barrier(S["flag"])
        self._mark()
        _lib.check(lib.frank_expert_ffn_scatter(
            S["recv_x"].data_ptr(), S["recv_w"].data_ptr(), S["local_off"].data_ptr(), self.El, S["cap"], H, self.F,
            self.w_up.data_ptr(), self.w_gate.data_ptr(), self.w_down.data_ptr(), S["row_rank"].data_ptr(),
            S["row_pos"].data_ptr(), S["peer_ret"], self.P, S["ret_rows"], S["hs"].data_ptr(), S["hs"].numel(), st))
        self._mark()
        self._barrier(S["flag"])
        self._mark()
        y = out if out is not None else torch.empty((T, H), dtype=self.out_dtype, device=dev)
        ops.combine(S["ret"][:self.k * T], slot_pos, T, self.k, y)
        self._mark()
        return y

    # ----------------------------------------------------------- nccl mode --
    def _call_nccl(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x.shape
        dev = x.device
        pr = self.prims
        if self.profile:
            self._marks.append([])
        self._mark()
        w, ids = pr.route(x, self.wr, self.k, self.normalize)
        sorted_slots, offsets, slot_pos = pr.permute(self._placed(ids), self.E)
        xs, ws = pr.gather(x, w, sorted_slots)
        # per-(destination rank, its local expert) counts
        cnt = (offsets[1:] - offsets[:-1]).to(torch.int64).reshape(self.P, self.El)
        self._mark()
        recv_cnt_t = torch.empty_like(cnt)
        self._comm(dist.all_to_all_single, recv_cnt_t, cnt.contiguous(), group=self.group)
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
        self._mark()
        self._exchange(xs, xl, send_chunks, recv_chunks)
        self._exchange(ws, wl, send_chunks, recv_chunks)
        dl = torch.empty((R, H), dtype=torch.float32, device=dev)
        offs = torch.from_numpy(local_off.astype(np.int32)).to(dev, non_blocking=True)
        self._mark()
        if R:
            pr.expert_ffn(xl, wl, offs, self.w_up, self.w_gate, self.w_down, dl)
        # results go back chunk for chunk into this rank's expert-sorted order
        ret = torch.empty((n, H), dtype=torch.float32, device=dev)
        self._mark()
        self._exchange(dl, ret, recv_chunks, send_chunks)
        self._mark()
        y = out if out is not None else torch.empty((T, H), dtype=self.out_dtype, device=dev)
        pr.combine(ret, slot_pos, T, self.k, y)
        self._mark()
        return y
