"""The five benchmark/parity configurations of the MoE FFN path and their
seeded synthetic inputs.

Shapes come from the project's headline configurations (fp32 toy block,
mul_mat_id alone, Mixtral-8x7B block, fine-grained 128-expert block with a
Zipf(1.2) router skew, and decode-sized blocks).  Inputs are synthetic:
x ~ N(0, 1), all weights ~ N(0, 0.02), drawn in the order x, router,
gate, up, down.  Small configurations draw on the host with
``np.random.default_rng(seed)``; the large ones draw on the device with a
seeded ``torch.Generator`` (the same distributions), because drawing
billions of normals on the host would dominate start-up.

Weight layouts are the reference's: router [E, H], up/gate [F, H, E],
down [H, F, E] (components/moe/moe_ffn_block.mlir:35-39).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class BlockConfig:
    name: str
    T: int
    H: int
    F: int
    E: int
    k: int
    normalize: bool
    dtype: str  # "f32" or "bf16"
    zipf: float = 0.0  # router popularity skew (0 = uniform)

    @property
    def flops(self) -> float:
        """Algorithmic flops of one block call: router 2HE + 3 GEMMs 6kHF per token."""
        return float(self.T) * (2 * self.H * self.E + 6 * self.k * self.H * self.F)


C1 = BlockConfig("c1_fp32_toy", T=32, H=64, F=128, E=8, k=2, normalize=True, dtype="f32")
C3 = BlockConfig("c3_mixtral_8x7b", T=16384, H=4096, F=14336, E=8, k=2, normalize=False, dtype="bf16")
C4 = BlockConfig("c4_fine_grained_zipf", T=8192, H=2048, F=768, E=128, k=8, normalize=False, dtype="bf16",
                 zipf=1.2)


def c5(T: int) -> BlockConfig:
    return BlockConfig(f"c5_decode_T{T}", T=T, H=2048, F=768, E=128, k=8, normalize=False, dtype="bf16")


@dataclass(frozen=True)
class MulMatIdConfig:
    name: str
    T: int
    n_in: int
    n_out: int
    E: int
    k: int

    @property
    def flops(self) -> float:
        return 2.0 * self.T * self.k * self.n_in * self.n_out


C2 = MulMatIdConfig("c2_mul_mat_id", T=4096, n_in=4096, n_out=14336, E=8, k=2)

# Mixtral-shaped block with 2 experts and T=4096 (every token uses both):
# the same per-expert GEMM shapes as C3 (M = 4096 rows, N = 2 x 14336,
# K = 4096) in about 1.5 GB, for ncu captures that replay kernels.
C3_PROFILE = BlockConfig("c3_profile_2experts", T=4096, H=4096, F=14336, E=2, k=2, normalize=False, dtype="bf16")

BLOCK_CONFIGS = {c.name: c for c in (C1, C3, C4, c5(1), c5(8), c5(32), c5(64), C3_PROFILE)}


def zipf_log_bias(E: int, s: float, seed: int) -> np.ndarray:
    """ln p_e with p_e proportional to rank_e^-s over a seeded expert permutation."""
    rng = np.random.default_rng(seed + 1000)
    ranks = np.empty(E, dtype=np.int64)
    ranks[rng.permutation(E)] = np.arange(1, E + 1)
    p = ranks.astype(np.float64) ** (-s)
    p /= p.sum()
    return np.log(p)


def block_inputs_numpy(cfg: BlockConfig, seed: int = 0):
    """Host (numpy fp32) inputs in reference layouts: x, wr, w_up, w_gate, w_down."""
    rng = np.random.default_rng(seed)
    T, H, F, E = cfg.T, cfg.H, cfg.F, cfg.E
    x = rng.standard_normal((T, H), dtype=np.float32)
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    w_gate = (rng.standard_normal((F, H, E), dtype=np.float32) * 0.02).astype(np.float32)
    w_up = (rng.standard_normal((F, H, E), dtype=np.float32) * 0.02).astype(np.float32)
    w_down = (rng.standard_normal((H, F, E), dtype=np.float32) * 0.02).astype(np.float32)
    if cfg.zipf:
        x[:, 0] = 1.0
        wr[:, 0] += zipf_log_bias(E, cfg.zipf, seed).astype(np.float32)
    return x, wr, w_up, w_gate, w_down


def block_inputs_torch(cfg: BlockConfig, device, seed: int = 0, dtype=torch.bfloat16):
    """Device inputs drawn with a seeded torch.Generator, same distributions as
    :func:`block_inputs_numpy`.  Returns x [T,H] (dtype), wr [E,H] fp32 and
    the expert weights in reference layouts (dtype)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T, H, F, E = cfg.T, cfg.H, cfg.F, cfg.E

    def randn(*shape, scale=1.0):
        t = torch.empty(shape, dtype=torch.float32, device=device)
        t.normal_(0.0, scale, generator=g)
        return t

    x = randn(T, H)
    wr = randn(E, H, scale=0.02)
    if cfg.zipf:
        x[:, 0] = 1.0
        wr[:, 0] += torch.from_numpy(zipf_log_bias(E, cfg.zipf, seed).astype(np.float32)).to(device)
    x = x.to(dtype)
    w_gate = randn(F, H, E, scale=0.02).to(dtype)
    w_up = randn(F, H, E, scale=0.02).to(dtype)
    w_down = randn(H, F, E, scale=0.02).to(dtype)
    return x, wr, w_up, w_gate, w_down


def block_weights_packed_torch(cfg: BlockConfig, device, seed: int = 0, dtype=torch.bfloat16):
    """Large-config weights drawn directly in the packed [E, O, I] layout
    (statistically identical to drawing [O, I, E] and packing, without a
    second multi-GB copy).  Returns wr [E,H] fp32, w_up_p/w_gate_p [E,F,H],
    w_down_p [E,H,F]."""
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    T, H, F, E = cfg.T, cfg.H, cfg.F, cfg.E

    def randn(*shape, scale):
        t = torch.empty(shape, dtype=dtype, device=device)
        # draw in chunks to bound the fp32 temporary
        flat = t.view(-1)
        step = 1 << 27
        for i in range(0, flat.numel(), step):
            n = min(step, flat.numel() - i)
            tmp = torch.empty(n, dtype=torch.float32, device=device)
            tmp.normal_(0.0, scale, generator=g)
            flat[i:i + n].copy_(tmp)
        return t

    wr = randn(E, H, scale=0.02).float()
    if cfg.zipf:
        wr[:, 0] += torch.from_numpy(zipf_log_bias(E, cfg.zipf, seed).astype(np.float32)).to(device)
    w_gate = randn(E, F, H, scale=0.02)
    w_up = randn(E, F, H, scale=0.02)
    w_down = randn(E, H, F, scale=0.02)
    return wr, w_up, w_gate, w_down


def block_x_torch(cfg: BlockConfig, device, seed: int = 0, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.empty((cfg.T, cfg.H), dtype=torch.float32, device=device)
    x.normal_(0.0, 1.0, generator=g)
    if cfg.zipf:
        x[:, 0] = 1.0
    return x.to(dtype)


def mul_mat_id_inputs_numpy(cfg: MulMatIdConfig, seed: int = 0):
    """weights [O, I, E], input [I, k, T] (x replicated per slot), ids [k, T]
    (first k of a seeded permutation of the experts per token: distinct)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((cfg.n_in, cfg.T), dtype=np.float32)
    w = (rng.standard_normal((cfg.n_out, cfg.n_in, cfg.E), dtype=np.float32) * 0.02).astype(np.float32)
    ids = np.stack([rng.permutation(cfg.E)[: cfg.k] for _ in range(cfg.T)], axis=1).astype(np.int32)
    inp = np.ascontiguousarray(np.broadcast_to(x[:, None, :], (cfg.n_in, cfg.k, cfg.T)))
    return w, inp, ids
