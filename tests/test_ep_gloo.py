"""Expert-parallel host logic on CPU ranks (gloo, world size 2 and 4).

The exchange plan, the per-(peer, expert) chunk exchange and the combine order are
the product code (frank_b200/ep.py); the device primitives are replaced by
NumPy stand-ins built from the oracle, so no GPU is involved.  Every rank's
output must equal the single-device oracle on that rank's tokens.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as O


class NumpyPrims:
    """Stand-ins for the CUDA primitives with the same contracts."""

    def route(self, x, wr, k, normalize):
        w, ids = O.route(x.numpy().astype(np.float64), wr.numpy().astype(np.float64), k, normalize)
        return torch.from_numpy(w.astype(np.float32)), torch.from_numpy(ids)

    def permute(self, ids, E):
        ss, off, pos = O.permutation(ids.numpy(), E)
        return torch.from_numpy(ss), torch.from_numpy(off), torch.from_numpy(pos)

    def gather(self, x, w, sorted_slots):
        T = x.shape[0]
        s = sorted_slots.numpy()
        return x[torch.from_numpy(s % T)].clone(), w.reshape(-1)[sorted_slots.long()].clone()

    def expert_ffn(self, xs, w_rows, offsets, w_up, w_gate, w_down, out):
        off = offsets.numpy()
        for e in range(len(off) - 1):
            lo, hi = off[e], off[e + 1]
            if lo == hi:
                continue
            xe = xs[lo:hi].double().numpy()
            g = xe @ w_gate[e].double().numpy().T
            u = xe @ w_up[e].double().numpy().T
            d = O.swiglu(g, u) @ w_down[e].double().numpy().T
            out[lo:hi] = torch.from_numpy((d * w_rows[lo:hi].double().numpy()[:, None]).astype(np.float32))
        return out

    def combine(self, d, slot_pos, T, k, out):
        pos = slot_pos.numpy().reshape(k, T)
        acc = np.zeros((T, d.shape[1]), dtype=np.float32)
        for j in range(k):
            acc += d.numpy()[pos[j]]
        out.copy_(torch.from_numpy(acc))
        return out


def _worker(rank, world, port, cfg, q, placed=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from frank_b200 import ep

        T, H, F, E, k, norm = cfg
        rng = np.random.default_rng(0)
        wr = rng.standard_normal((E, H)).astype(np.float32) * 0.5
        wu = rng.standard_normal((E, F, H)).astype(np.float32) * 0.1
        wg = rng.standard_normal((E, F, H)).astype(np.float32) * 0.1
        wd = rng.standard_normal((E, H, F)).astype(np.float32) * 0.1
        x = np.random.default_rng(100 + rank).standard_normal((T, H)).astype(np.float32)
        El = E // world
        sl = slice(rank * El, (rank + 1) * El)
        placement = None
        if placed:
            # calibration batch of other tokens: every rank ends with the same placement
            xc = np.random.default_rng(200 + rank).standard_normal((T, H)).astype(np.float32)
            load = ep.measure_expert_load(torch.from_numpy(xc), torch.from_numpy(wr), k, norm, E,
                                          prims=NumpyPrims())
            placement = ep.balanced_placement(load, world)
            sl = placement[rank * El:(rank + 1) * El]
        moe = ep.ExpertParallelMoE(torch.from_numpy(wr), torch.from_numpy(wu[sl]), torch.from_numpy(wg[sl]),
                                   torch.from_numpy(wd[sl]), E, k, norm, prims=NumpyPrims(), placement=placement)
        y = moe(torch.from_numpy(x)).numpy()
        ref = O.moe_ffn_block_grouped(x.astype(np.float64), wr.astype(np.float64),
                                      wu.transpose(1, 2, 0).astype(np.float64),
                                      wg.transpose(1, 2, 0).astype(np.float64),
                                      wd.transpose(1, 2, 0).astype(np.float64), E, k, H, F, norm)
        err = float(np.max(np.abs(y - ref)))
        send_cnt, recv_cnt = moe.last_plan
        q.put((rank, err, int(send_cnt.sum()), int(recv_cnt.sum()),
               None if placement is None else placement.tolist()))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,cfg,placed", [
    (2, (37, 16, 12, 8, 2, False), False),
    (2, (50, 8, 8, 4, 3, True), False),
    (4, (29, 16, 8, 16, 4, False), False),
    (4, (1, 8, 8, 8, 2, True), False),   # a single token per rank: most ranks receive nothing from some peers
    (2, (37, 16, 12, 8, 2, False), True),  # load-balanced expert placement from a calibration batch
    (4, (29, 16, 8, 16, 4, True), True),
])
def test_expert_parallel_matches_single_device(world, cfg, placed):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, q, placed)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(world))
    T, k = cfg[0], cfg[4]
    for rank, err, sent, recvd, _ in res:
        assert err < 1e-4, f"rank {rank}: max abs error {err}"
        assert sent == T * k
    assert sum(r[3] for r in res) == world * T * k
    if placed:
        pls = [r[4] for r in res]
        assert all(pl == pls[0] for pl in pls)  # every rank derived the same placement
        assert sorted(pls[0]) == list(range(cfg[3]))


def test_balanced_placement():
    from frank_b200.ep import balanced_placement

    # Zipf-like load over 8 experts on 2 ranks: the two heaviest go to different ranks
    load = np.array([100, 50, 33, 25, 20, 17, 14, 12])
    pl = balanced_placement(load, 2)
    assert sorted(pl.tolist()) == list(range(8))
    r0, r1 = set(pl[:4].tolist()), set(pl[4:].tolist())
    assert 0 in r0 and 1 in r1
    loads = [load[list(r0)].sum(), load[list(r1)].sum()]
    assert max(loads) <= 146  # optimum 143 (100 + the three lightest); contiguous halves give 208 / 63
    assert list(pl[:4]) == sorted(pl[:4]) and list(pl[4:]) == sorted(pl[4:])
    # equal loads: experts dealt round-robin (ties to the lower id, then the lower rank)
    assert balanced_placement(np.ones(8), 4).tolist() == [0, 4, 1, 5, 2, 6, 3, 7]
    # deterministic, and every rank gets E/P experts
    pl2 = balanced_placement(np.arange(16)[::-1] ** 2, 4)
    assert pl2.tolist() == balanced_placement(np.arange(16)[::-1] ** 2, 4).tolist()
    with pytest.raises(ValueError):
        balanced_placement(np.ones(6), 4)


def test_placement_validation():
    from frank_b200 import ep

    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        E, H, F = 4, 8, 8
        wr = torch.zeros(E, H)
        w = (torch.zeros(E, F, H), torch.zeros(E, F, H), torch.zeros(E, H, F))
        for bad in ([0, 0, 1, 2], [0, 1, 2], [0, 1, 2, 4]):
            with pytest.raises(ValueError):
                ep.ExpertParallelMoE(wr, *w, E, 2, False, prims=NumpyPrims(), placement=bad)
        # the identity placement is the contiguous split (no renaming)
        moe = ep.ExpertParallelMoE(wr, *w, E, 2, False, prims=NumpyPrims(), placement=[0, 1, 2, 3])
        assert moe.placement is None
        moe = ep.ExpertParallelMoE(wr, *w, E, 2, False, prims=NumpyPrims(), placement=[2, 0, 3, 1])
        ids = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32)
        assert moe._placed(ids).tolist() == [[1, 3], [0, 2]]
    finally:
        dist.destroy_process_group()
