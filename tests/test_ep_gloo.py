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


def _worker(rank, world, port, cfg, q):
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
        moe = ep.ExpertParallelMoE(torch.from_numpy(wr), torch.from_numpy(wu[sl]), torch.from_numpy(wg[sl]),
                                   torch.from_numpy(wd[sl]), E, k, norm, prims=NumpyPrims())
        y = moe(torch.from_numpy(x)).numpy()
        ref = O.moe_ffn_block_grouped(x.astype(np.float64), wr.astype(np.float64),
                                      wu.transpose(1, 2, 0).astype(np.float64),
                                      wg.transpose(1, 2, 0).astype(np.float64),
                                      wd.transpose(1, 2, 0).astype(np.float64), E, k, H, F, norm)
        err = float(np.max(np.abs(y - ref)))
        send_cnt, recv_cnt = moe.last_plan
        q.put((rank, err, int(send_cnt.sum()), int(recv_cnt.sum())))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,cfg", [
    (2, (37, 16, 12, 8, 2, False)),
    (2, (50, 8, 8, 4, 3, True)),
    (4, (29, 16, 8, 16, 4, False)),
    (4, (1, 8, 8, 8, 2, True)),     # a single token per rank: most ranks receive nothing from some peers
])
def test_expert_parallel_matches_single_device(world, cfg):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(world))
    T, k = cfg[0], cfg[4]
    for rank, err, sent, recvd in res:
        assert err < 1e-4, f"rank {rank}: max abs error {err}"
        assert sent == T * k
    assert sum(r[3] for r in res) == world * T * k


def test_plan_exchange_layout():
    from frank_b200.ep import plan_exchange

    recv = np.array([[2, 0, 1], [1, 3, 0]])  # from rank 0: e0=2,e1=0,e2=1 ; from rank 1: e0=1,e1=3,e2=0
    send = np.array([[1, 1, 1], [2, 2, 2]])
    ss, rs, seg, off = plan_exchange(send, recv)
    assert ss.tolist() == [3, 6] and rs.tolist() == [3, 4]
    assert off.tolist() == [0, 3, 6, 7]
    # source-major: [r0e0 r0e0 r0e2 | r1e0 r1e1 r1e1 r1e1]; expert-major: [e0: r0 r0 r1 | e1: r1 r1 r1 | e2: r0]
    assert seg.src_start.tolist() == [0, 2, 2, 3, 4, 7]
    assert seg.dst_start.tolist() == [0, 3, 6, 2, 3, 7]
    assert seg.length.tolist() == [2, 0, 1, 1, 3, 0]
