"""Launch geometries of the tensor-core CTA-pair kernels, checked on the host.

The pair kernels (`csrc/kernels/tcpair.cuh`) run as clusters of 2 x 1 x S CTAs: the two CTAs of
a pair must be adjacent along x (the cluster dimension tensor-core CTA pairs are formed on), so
every pair grid has an even x size and a z size equal to its K splits; the argmax heads' partial
slots (the planner reads them from grid.x) are two per 256-column tile.  These are the shapes the
planner hands the runtime, so they are pinned here without a GPU, for the cfg5 shard (512 rows),
a batched-prefill chunk (16384 rows) and the forced-pair test modes.
"""
from __future__ import annotations

import pytest

from ckl.compile import library_accepts, library_geometry
from ckl.library import pack

PAIR_SMEM = 200 * 1024  # lower bound of a pair CTA's dynamic shared memory (one CTA per SM)


def gemm(M, K, N, layers=4, A=0, D=0, T=0, cache=0):
    return pack(M, K, N, layers, 0, A, D, T, 0, 0, cache or M)


def test_cfg5_shard_geometries(monkeypatch):
    monkeypatch.delenv("CKL_B200_TC_PAIRS", raising=False)
    monkeypatch.delenv("CKL_B200_TC_QKV", raising=False)
    # gate/up: 128 outputs per pair tile (128 gate + 128 up columns), 2 row pairs, no split.
    grid, block, shared = library_geometry("ckl.fused.panel_gate_up", gemm(512, 1024, 4096))
    assert grid == (64, 2, 1) and block == (320, 1, 1) and shared > PAIR_SMEM
    # LM head: 125 tiles of 256 columns -> 250 partial slots per row (grid.x).
    grid, _, _ = library_geometry("ckl.fused.panel_linear_argmax", gemm(512, 1024, 32000, 1))
    assert grid == (250, 2, 1)
    # Fused q/k/v: 3 x 1024 columns = 12 pair tiles, 2 row pairs, K split over 2 pairs.
    grid, _, _ = library_geometry("ckl.fused.panel_qkv",
                                  gemm(512, 1024, 1024, A=16, D=64, T=2080))
    assert grid == (24, 2, 2)
    # o and down keep the single-CTA kernel: 8 column tiles x 4 row tiles, K split 4 ways.
    for K in (1024, 4096):
        grid, _, _ = library_geometry("ckl.fused.panel_linear_residual", gemm(512, K, 1024))
        assert grid == (8, 4, 4)


def test_prefill_chunk_takes_pairs_without_splits(monkeypatch):
    monkeypatch.delenv("CKL_B200_TC_PAIRS", raising=False)
    rows = 16384
    grid, _, _ = library_geometry("ckl.fused.panel_linear_residual", gemm(rows, 4096, 1024))
    assert grid == (8, 64, 1)  # 4 tiles of 256 columns (x2 CTAs), 64 row pairs
    grid, _, _ = library_geometry("ckl.fused.panel_qkv",
                                  gemm(rows, 1024, 1024, A=16, D=64, T=2080, cache=512))
    assert grid == (24, 64, 1)
    grid, _, _ = library_geometry("ckl.fused.panel_argmax", gemm(rows, 1024, 32000, 1))
    assert grid == (250, 64, 1)


@pytest.mark.parametrize("mode", ["2", "3"])
@pytest.mark.parametrize("M,K,N", [(256, 64, 256), (300, 256, 512), (640, 1024, 1024),
                                   (384, 384, 384), (129, 96, 1000)])
def test_forced_pair_grids_are_cluster_shaped(monkeypatch, mode, M, K, N):
    monkeypatch.setenv("CKL_B200_TC_PAIRS", mode)
    grid, _, _ = library_geometry("ckl.fused.panel_linear_residual", gemm(M, K, N))
    row_tiles = -(-M // 128)
    width = 256 if mode == "2" else 128
    if row_tiles >= 2 and N >= width:
        assert grid[0] == 2 * -(-N // width) and grid[1] == -(-row_tiles // 2)
        assert grid[2] in (1, 2, 4, 8) and 2 * grid[2] <= (16 if width == 256 else 8)
        assert grid[0] * grid[1] * grid[2] <= 148 or grid[2] == 1
    else:  # one row tile or too few columns: the single-CTA kernel
        assert grid[1] == -(-M // 128) or grid[1] == -(-M // 256)


def test_fused_qkv_declines_unsupported_shapes(monkeypatch):
    monkeypatch.delenv("CKL_B200_TC_PAIRS", raising=False)
    assert not library_accepts("ckl.fused.panel_qkv", gemm(512, 384, 384, A=6, D=64, T=64))
    assert not library_accepts("ckl.fused.panel_qkv", gemm(128, 1024, 1024, A=16, D=64, T=64))
    monkeypatch.setenv("CKL_B200_TC_PAIRS", "0")
    assert not library_accepts("ckl.fused.panel_qkv", gemm(512, 1024, 1024, A=16, D=64, T=64))
    monkeypatch.delenv("CKL_B200_TC_PAIRS")
    monkeypatch.setenv("CKL_B200_TC_QKV", "0")
    assert not library_accepts("ckl.fused.panel_qkv", gemm(512, 1024, 1024, A=16, D=64, T=64))
