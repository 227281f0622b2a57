"""Bit-exact routing and permutation on the GPU.

(a) Given identical fp32 logits, the softmax/top-k kernel returns exactly the
    oracle's expert ids (ties to the lowest index) and its weights within
    fp32 rounding.
(b) The router kernel, which computes the logits itself, agrees with the
    oracle's ids except where the k-th and (k+1)-th probabilities are closer
    than the fp32 accumulation-order bound.
(c) The permutation (histogram + scan + scatter, no atomics) equals
    argsort(ids.reshape(-1), stable) and the bincount prefix exactly.
"""

import numpy as np
import pytest
import torch

from frank_b200 import ops
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("E,k,T,norm", [(8, 2, 1000, False), (8, 2, 333, True), (128, 8, 777, False),
                                        (128, 8, 64, True), (4, 1, 5, False), (256, 32, 50, True),
                                        (5, 5, 17, True)])
def test_softmax_topk_bitexact_ids(E, k, T, norm):
    rng = np.random.default_rng(E * 1000 + k)
    logits = rng.standard_normal((E, T)).astype(np.float32)
    w, ids = ops.softmax_topk(torch.from_numpy(logits).cuda(), k, norm)
    rw, rids = O.route_from_logits(logits, k, norm)
    assert np.array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


def test_softmax_topk_ties_lowest_index():
    # quantised logits: many exact ties
    rng = np.random.default_rng(3)
    E, k, T = 16, 4, 2000
    logits = rng.integers(-2, 3, size=(E, T)).astype(np.float32)
    logits[:, :10] = 0.0  # all-equal tokens
    w, ids = ops.softmax_topk(torch.from_numpy(logits).cuda(), k, False)
    rw, rids = O.route_from_logits(logits, k, False)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert ids[:, 0].cpu().tolist() == [0, 1, 2, 3]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
# (the vector router splits H over up to 8 warps when the tokens alone do
# not fill the SMs: 1032 columns split into uneven 8-aligned slices)
@pytest.mark.parametrize("E,k,H,T", [(8, 2, 4096, 512), (128, 8, 2048, 300), (8, 1, 64, 33), (8, 2, 4096, 2048),
                                     (6, 2, 1032, 97), (8, 2, 4096, 1), (8, 2, 4096, 16384)])
def test_router_matches_oracle(dtype, E, k, H, T):
    rng = np.random.default_rng(H + T)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(dtype)
    wr = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    w, ids = ops.router_topk(x.cuda(), torch.from_numpy(wr).cuda(), k, False)
    xf = x.float().numpy().astype(np.float64)
    logits = wr.astype(np.float64) @ xf.T
    rw, rids = O.route_from_logits(logits, k, False)
    ids = ids.cpu().numpy()
    # tokens whose k-th/(k+1)-th logit gap is below the accumulation bound may differ
    srt = -np.sort(-logits, axis=0)
    gap = srt[k - 1] - srt[k] if k < E else np.full(T, np.inf)
    bound = 1e-5 * np.sqrt(H) * np.abs(logits).max()
    safe = gap > bound
    assert np.array_equal(ids[:, safe], rids[:, safe])
    assert safe.mean() > 0.95
    np.testing.assert_allclose(w.cpu().numpy()[:, safe], rw[:, safe], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("E,k,T,kind", [(8, 2, 16384, "uniform"), (128, 8, 8192, "zipf"), (128, 8, 1, "uniform"),
                                        (8, 2, 3, "one"), (64, 4, 777, "sparse"), (1024, 2, 5000, "uniform"),
                                        (8, 2, 0, "uniform"),
                                        # one-block form: n <= 4096 slots and E <= 256; the
                                        # three-pass form past either limit
                                        (8, 2, 2048, "uniform"), (256, 8, 512, "zipf"),
                                        (256, 8, 513, "uniform"), (8, 2, 2049, "one"), (257, 1, 100, "uniform")])
def test_permute_bitexact(E, k, T, kind):
    rng = np.random.default_rng(T + E)
    if kind == "uniform":
        ids = rng.integers(0, E, size=(k, T))
    elif kind == "zipf":
        p = np.arange(1, E + 1, dtype=np.float64) ** -1.2
        ids = rng.choice(E, size=(k, T), p=p / p.sum())
    elif kind == "one":
        ids = np.full((k, T), E - 1)
    else:
        ids = rng.choice([0, 5, 63], size=(k, T))
    ids = ids.astype(np.int32)
    ss, off, pos, err = ops.permute(torch.from_numpy(ids).cuda(), E)
    rss, roff, rpos = O.permutation(ids, E)
    assert np.array_equal(ss.cpu().numpy(), rss)
    assert np.array_equal(off.cpu().numpy(), roff)
    assert np.array_equal(pos.cpu().numpy(), rpos)
    assert int(err.item()) == 0


def test_permute_flags_bad_ids():
    ids = torch.tensor([[0, 9, 1, -3]], dtype=torch.int32, device="cuda")
    _, off, _, err = ops.permute(ids, 4)
    assert int(err.item()) == 1
    assert int(off[-1].item()) == 4


@pytest.mark.parametrize("E,k,H,T,wdt", [(128, 8, 2048, 8192, torch.float32), (16, 4, 512, 300, torch.bfloat16),
                                         (8, 2, 4096, 1000, torch.float32), (128, 8, 2048, 5, torch.float32)])
def test_router_pack_same_results(E, k, H, T, wdt):
    """A router pack (fp32 copy + prepared bf16 split) routes exactly like the
    raw router weights on every router path (tensor-core, E <= 8, few tokens)."""
    rng = np.random.default_rng(E + T)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).bfloat16().cuda()
    wr = torch.from_numpy((rng.standard_normal((E, H)) * 0.02).astype(np.float32)).to(wdt).cuda()
    w0, i0 = ops.router_topk(x, wr, k, False)
    w1, i1 = ops.router_topk(x, wr, k, False, pack=ops.router_pack(wr))
    assert torch.equal(i0, i1) and torch.equal(w0, w1)
