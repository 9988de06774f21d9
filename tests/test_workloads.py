"""Seeded synthetic workload generators (shapes of the BASELINE configs)."""
import numpy as np


def test_small_split(mxg):
    s = mxg.workloads.small_split()
    assert s.real.tolist() == [128, 64, 0, 192] and s.M == 384
    assert s.offs_leading_zero().tolist() == [0, 128, 192, 192, 384]


def test_dirichlet_split_deterministic_and_padded(mxg):
    a = mxg.workloads.dirichlet_split(65536, 32, 1.0, seed=0)
    b = mxg.workloads.dirichlet_split(65536, 32, 1.0, seed=0)
    assert np.array_equal(a.real, b.real)
    assert a.real_rows == 65536 and a.E == 32
    assert np.all(a.padded % 32 == 0) and np.all(a.padded >= a.real)
    assert a.M - a.real_rows < 32 * 32
    assert a.row_mask().sum() == 65536


def test_topk_split(mxg):
    s = mxg.workloads.topk_softmax_split(32768, 8, 2, seed=0)
    assert s.real_rows == 65536
    assert np.all(np.abs(s.real - 8192) < 800)


def test_zipf_assign(mxg):
    a = mxg.workloads.zipf_topk_assign(1024, 256, 8, 1.1, seed=0)
    assert a.shape == (1024, 8)
    assert all(len(set(r)) == 8 for r in a.tolist())
    counts = np.bincount(a.reshape(-1), minlength=256)
    assert counts.max() > 4 * counts.mean()  # skewed popularity


def test_flops(mxg):
    s = mxg.workloads.small_split()
    assert mxg.workloads.grouped_flops(s, 256, 512) == 2 * 384 * 256 * 512
