"""Seeded synthetic workloads with the shapes and value distributions of the
BASELINE configurations (no dataset is involved; "DeepSeek-V3" and "Mixtral"
name shapes only).

* small   (config 0): E=4, K=512, N=256, M_e=[128, 64, 0, 192].
* dsv3    (configs 1-2): 32 local experts, hidden 7168, gate/up N=4096,
  intermediate 2048; 65536 routed rows split by a seeded multinomial over
  Dirichlet(1.0) expert probabilities, each group padded to a multiple of 32.
* mixtral (config 3): 8 experts, hidden 4096, FFN 14336; 32768 tokens, top-2
  routing from softmax over N(0,1) router logits.
* ep      (config 4): 256 experts sharded over G GPUs, 16384 tokens per GPU,
  top-8 routing from a Zipf(1.1) expert popularity.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

PAD = 32


def pad_up(v, m=PAD):
    return (np.asarray(v) + m - 1) // m * m


@dataclass
class GroupSplit:
    """Per-expert routed row counts (real) and their 32-padded sizes."""
    real: np.ndarray
    padded: np.ndarray = field(init=False)

    def __post_init__(self):
        self.real = np.asarray(self.real, dtype=np.int64)
        self.padded = pad_up(self.real).astype(np.int64)

    @property
    def E(self) -> int:
        return len(self.real)

    @property
    def M(self) -> int:
        return int(self.padded.sum())

    @property
    def real_rows(self) -> int:
        return int(self.real.sum())

    def offs_cumulative(self) -> np.ndarray:
        return np.cumsum(self.padded).astype(np.int32)

    def offs_leading_zero(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.padded)]).astype(np.int32)

    def row_mask(self) -> np.ndarray:
        """True for real rows, False for the zero padding rows."""
        m = np.zeros(self.M, dtype=bool)
        s = 0
        for r, p in zip(self.real, self.padded):
            m[s:s + r] = True
            s += p
        return m


def small_split() -> GroupSplit:
    return GroupSplit([128, 64, 0, 192])


def dirichlet_split(num_rows=65536, num_groups=32, alpha=1.0, seed=0) -> GroupSplit:
    rng = np.random.default_rng(seed)
    p = rng.dirichlet([alpha] * num_groups)
    return GroupSplit(rng.multinomial(num_rows, p))


def topk_softmax_split(num_tokens=32768, num_experts=8, topk=2, seed=0) -> GroupSplit:
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((num_tokens, num_experts))
    top = np.argpartition(-logits, topk - 1, axis=1)[:, :topk]
    return GroupSplit(np.bincount(top.reshape(-1), minlength=num_experts))


def zipf_topk_assign(num_tokens, num_experts=256, topk=8, s=1.1, seed=0) -> np.ndarray:
    """[num_tokens, topk] distinct expert ids per token, expert popularity
    proportional to 1/rank^s (Gumbel top-k sampling without replacement)."""
    rng = np.random.default_rng(seed)
    ranks = rng.permutation(num_experts) + 1
    logp = -s * np.log(ranks.astype(np.float64))
    g = rng.gumbel(size=(num_tokens, num_experts))
    return np.argpartition(-(logp[None, :] + g), topk - 1, axis=1)[:, :topk].astype(np.int64)


def zipf_log_popularity(num_experts=256, s=1.1, seed=0) -> np.ndarray:
    """log popularity of each expert, 1/rank^s over a seeded random ranking
    (shared by every rank of an expert-parallel group)."""
    ranks = np.random.default_rng(seed).permutation(num_experts) + 1
    return -s * np.log(ranks.astype(np.float64))


def zipf_topk_sample(num_tokens, logp, topk=8, seed=0) -> np.ndarray:
    """[num_tokens, topk] distinct experts per token drawn with popularity
    exp(logp) (Gumbel top-k, without replacement), in the token's own order of
    preference."""
    g = np.random.default_rng(seed).gumbel(size=(num_tokens, logp.size))
    score = logp[None, :] + g
    part = np.argpartition(-score, topk - 1, axis=1)[:, :topk]
    order = np.argsort(-np.take_along_axis(score, part, axis=1), axis=1)
    return np.take_along_axis(part, order, axis=1).astype(np.int32)


def expected_expert_load(logp, topk=8, samples=65536, seed=12345) -> np.ndarray:
    """Expected routed rows per expert per token (a fixed calibration sample of
    the same top-k sampler); used for load-aware expert placement."""
    ids = zipf_topk_sample(samples, logp, topk, seed)
    return np.bincount(ids.reshape(-1), minlength=logp.size) / samples


# ---------------------------------------------------------------- problem shapes
@dataclass
class FwdShape:
    name: str
    N: int
    K: int


DSV3_GATE_UP = FwdShape("dsv3_gate_up", N=4096, K=7168)
DSV3_DOWN = FwdShape("dsv3_down", N=7168, K=2048)
MIXTRAL_GATE_UP = FwdShape("mixtral_gate_up", N=28672, K=4096)
MIXTRAL_DOWN = FwdShape("mixtral_down", N=4096, K=14336)
SMALL = FwdShape("small", N=256, K=512)


def grouped_flops(split: GroupSplit, N: int, K: int, padded: bool = False) -> int:
    """2 * sum(M_e) * N * K over real (default) or padded rows."""
    rows = split.M if padded else split.real_rows
    return 2 * rows * N * K


# ---------------------------------------------------------------- tensors
def routed_activations(split: GroupSplit, K: int, std: float = 1.0, device="cuda",
                       seed: int = 0) -> torch.Tensor:
    """[M_padded, K] bf16, N(0, std^2) on real rows, zero on padding rows."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(split.M, K, generator=g, device=device, dtype=torch.float32).mul_(std)
    mask = torch.from_numpy(split.row_mask()).to(device)
    x[~mask] = 0
    return x.to(torch.bfloat16)


def expert_weights(E: int, N: int, K: int, std: float = 0.02, device="cuda",
                   seed: int = 1) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(E, N, K, generator=g, device=device, dtype=torch.float32).mul_(std).to(torch.bfloat16)
