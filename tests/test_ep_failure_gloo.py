"""Failure detection of the expert-parallel step on CPU ranks (gloo).

(a) A rank that never enters the step: with ``step_timeout_s`` set, the other
    rank's call raises FrankError(FRANK_ETIMEOUT) within a few seconds, from
    the presence check at the start of the step (no collective of the step
    has been issued).
(b) A rank that fails inside the step (its router raises) after the presence
    check: the other rank's next collective ends with the process group's
    timeout and the call raises FrankError(FRANK_ENCCL) instead of waiting
    forever.
No GPU is involved: the device primitives are the NumPy stand-ins of
test_ep_gloo.py.
"""

import datetime
import os
import socket
import time

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.test_ep_gloo import NumpyPrims


class FailingPrims(NumpyPrims):
    """Routes normally on the first step, raises on the second."""

    calls = 0

    def route(self, x, wr, k, normalize):
        self.calls += 1
        if self.calls > 1:
            raise RuntimeError("injected failure in the router of this rank")
        return super().route(x, wr, k, normalize)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, scenario, done, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    try:
        from frank_b200 import _lib, ep

        T, H, F, E, k = 16, 8, 8, 4, 2
        rng = np.random.default_rng(0)
        wr = torch.from_numpy(rng.standard_normal((E, H)).astype(np.float32))
        w = [torch.from_numpy(rng.standard_normal(s).astype(np.float32) * 0.1)
             for s in ((E, F, H), (E, F, H), (E, H, F))]
        El = E // world
        sl = slice(rank * El, (rank + 1) * El)
        failing = scenario == "raises_in_step" and rank == 1
        moe = ep.ExpertParallelMoE(wr, *(t[sl] for t in w), E, k, False,
                                   prims=FailingPrims() if failing else NumpyPrims(), step_timeout_s=2.0)
        x = torch.from_numpy(np.random.default_rng(rank).standard_normal((T, H)).astype(np.float32))
        moe(x)  # one healthy step on every rank first
        if scenario == "never_joins" and rank == 1:
            done.wait(60)  # stays alive, never enters the next step
            q.put((rank, "absent", 0, 0.0))
            return
        t0 = time.monotonic()
        try:
            moe(x)
            q.put((rank, "ok", 0, time.monotonic() - t0))
        except _lib.FrankError as e:
            q.put((rank, "frank_error", e.code, time.monotonic() - t0))
        except RuntimeError as e:
            q.put((rank, "runtime_error:" + str(e)[:80], 0, time.monotonic() - t0))
        done.set()
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(scenario):
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scenario, done, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=120)
        res[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_rank_that_never_joins_gives_timeout():
    from frank_b200._lib import ETIMEOUT

    res = _run("never_joins")
    kind, code, secs = res[0]
    assert kind == "frank_error" and code == ETIMEOUT, res
    assert secs < 10, f"took {secs:.1f} s"


def test_rank_failing_inside_the_step_gives_collective_error():
    from frank_b200._lib import ENCCL

    res = _run("raises_in_step")
    assert res[1][0].startswith("runtime_error:injected"), res  # the failing rank's own exception
    kind, code, secs = res[0]
    assert kind == "frank_error" and code == ENCCL, res
    assert secs < 20, f"took {secs:.1f} s"
