"""Expert parallelism on real GPUs (NCCL): every rank's output must equal the
single-GPU block on the same tokens bit for bit, also when the ranks hold
different numbers of tokens (the peer buffers are sized from the gathered
counts of every step).  Needs >= 2 visible GPUs; ranks are child processes,
one per GPU."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfg, mode, ragged, q, placed=False):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from frank_b200 import configs, ep, ops

        wr, wu, wg, wd = configs.block_weights_packed_torch(cfg, dev, seed=0)
        x = configs.block_x_torch(cfg, dev, seed=10 + rank)
        if ragged:  # rank r holds T - 37 r tokens (one rank: T / 2, so the next call must grow the buffers)
            x = x[:(cfg.T // 2 if world == 1 else cfg.T - 37 * rank)].contiguous()
        El = cfg.E // world
        sl = slice(rank * El, (rank + 1) * El)
        placement = None
        if placed:  # experts placed by the load of a calibration batch of other tokens
            xc = configs.block_x_torch(cfg, dev, seed=50 + rank)
            placement = ep.balanced_placement(ep.measure_expert_load(xc, wr, cfg.k, cfg.normalize, cfg.E), world)
            if world == 1:  # one rank holds every expert: still renamed, in reverse order
                placement = placement[::-1].copy()
            sl = torch.as_tensor(placement[rank * El:(rank + 1) * El], device=dev)
        moe = ep.ExpertParallelMoE(wr, wu[sl].contiguous(), wg[sl].contiguous(), wd[sl].contiguous(), cfg.E, cfg.k,
                                   cfg.normalize, mode=mode, placement=placement)
        y = moe(x)
        if ragged and rank == world - 1:
            # the last rank's batch grows to T: every rank's buffers grow together
            x = configs.block_x_torch(cfg, dev, seed=99)
        y = moe(x)
        y2 = moe(x)
        single = ops.MoEFFNBlock(wr, ops.PackedExperts(wu), ops.PackedExperts(wg), ops.PackedExperts(wd), cfg.E,
                                 cfg.k, cfg.normalize)
        ref = single(x)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(y, ref)), bool(torch.equal(y, y2)),
               float((y - ref).abs().max().item()), ops.read_device_error()))
    finally:
        dist.destroy_process_group()


def _fg_cfg():
    from frank_b200 import configs

    return configs.BlockConfig("bf16_fg_ep", T=1000, H=2048, F=768, E=128, k=8, normalize=False, dtype="bf16",
                               zipf=1.2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_ep_balanced_placement_equals_single_gpu(mode):
    """Experts placed by load (Zipf-skewed routing): the same output bit for
    bit, with the rows spread more evenly than the contiguous split."""
    cfg = _fg_cfg()
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, mode, False, q, True)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for rank, equal, det, err, dev_err in sorted(q.get(timeout=10) for _ in range(world)):
        assert equal, f"rank {rank}: max |ep - single| = {err}"
        assert det and dev_err == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("ragged", [False, True], ids=["equal_T", "ragged_T"])
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
@pytest.mark.parametrize("cfg_name", ["bf16_fg_ep", "bf16_c3like_ep"])
def test_ep_equals_single_gpu(cfg_name, mode, ragged):
    from frank_b200 import configs

    cfg = {
        "bf16_fg_ep": configs.BlockConfig("bf16_fg_ep", T=1000, H=2048, F=768, E=128, k=8, normalize=False,
                                          dtype="bf16", zipf=1.2),
        "bf16_c3like_ep": configs.BlockConfig("bf16_c3like_ep", T=2048, H=1024, F=2048, E=8, k=2, normalize=True,
                                              dtype="bf16"),
    }[cfg_name]
    world = min(torch.cuda.device_count(), 8)
    while cfg.E % world:
        world //= 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, mode, ragged, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for rank, equal, det, err, dev_err in sorted(q.get(timeout=10) for _ in range(world)):
        assert equal, f"rank {rank}: max |ep - single| = {err}"
        assert det and dev_err == 0


@pytest.mark.parametrize("placed", [False, True], ids=["contiguous", "placed"])
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_ep_single_rank(mode, placed):
    """The expert-parallel step with one rank (all experts local, the
    exchange going through this GPU's own symmetric buffers): bit-identical
    to the single-GPU block, two calls with a growing batch (the second
    call's counts do not fit the first call's buffers: the step is planned
    and dispatched into them, refused, and redone into grown buffers).
    ``placed``: the experts renamed by a (reversed) placement."""
    from frank_b200 import configs

    cfg = configs.BlockConfig("bf16_fg_ep1", T=700, H=1024, F=512, E=32, k=4, normalize=True, dtype="bf16",
                              zipf=1.2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_worker, args=(0, 1, _free_port(), cfg, mode, True, q, placed))
    p.start()
    p.join(timeout=300)
    assert p.exitcode == 0
    rank, equal, det, err, dev_err = q.get(timeout=10)
    assert equal, f"max |ep - single| = {err}"
    assert det and dev_err == 0
