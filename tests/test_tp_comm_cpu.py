"""Host logic of the row-parallel reduction over peer memory (qik.tp_comm) and the
host validation of its C entry points; no GPU.

* ownership: ranks own ceil(M / world) rows rounded up to 256 (the GEMM's tallest
  tile), so tiles never straddle owners and the owners cover M;
* workspace layout: regions 256-byte aligned and disjoint, slots of R x N fp32 for two
  call parities and every source rank, two bf16 outputs, counters;
* counter targets wrap modulo 2^32 consistently with the kernels' signed distance;
* the per-owner arrival count of the scatter GEMM equals the number of (tile, CTA)
  units whose rows the owner holds, summed over owners it is the GEMM's whole tile count;
* the C entry points refuse bad arguments before touching the GPU.
"""
import ctypes

import pytest

from qik import tp_comm as T


@pytest.mark.parametrize("M,world", [(8704, 2), (8704, 8), (1000, 2), (300, 4), (256, 1), (1, 8)])
def test_rows_per_owner_cover_and_align(M, world):
    R = T.rows_per_owner(M, world)
    assert R % 256 == 0 and R * world >= M and R - 256 < -(-M // world)


@pytest.mark.parametrize("M,N,world", [(8704, 3072, 2), (8704, 3072, 8), (1000, 512, 2)])
def test_workspace_layout(M, N, world):
    lay = T.workspace_layout(M, N, world)
    R = lay["R"]
    assert lay["slot_bytes"] == R * N * 4
    regions = [(lay["recv"], 2 * world * lay["slot_bytes"]), (lay["out"], 2 * lay["out_bytes"]),
               (lay["cnt"], 4 * world), (lay["gcnt"], 4 * world)]
    for (a, n), (b, _) in zip(regions, regions[1:]):
        assert a % 256 == 0 and a + n <= b
    assert lay["total"] >= lay["gcnt"] + 4 * world
    assert lay["out_bytes"] % 16 == 0  # the parity-1 output stays 16-byte aligned


def test_counter_targets_wrap():
    per = 48
    e = (1 << 32) // per + 3  # past the wrap
    t0, t1 = T.counter_target(e - 1, per), T.counter_target(e, per)
    assert (t1 - t0) & 0xFFFFFFFF == per
    # the kernels compare int32(cnt - target) >= 0
    signed = lambda v: v - (1 << 32) if v >= 1 << 31 else v  # noqa: E731
    assert signed((t1 - t0) & 0xFFFFFFFF) > 0 and signed((t0 - t1) & 0xFFFFFFFF) < 0


@pytest.fixture(scope="module")
def lib():
    from qik import _lib as L
    return L.load(require_cuda=False)


@pytest.mark.parametrize("M,N,world", [(8704, 3072, 2), (8704, 3072, 8), (1000, 512, 2), (4352, 9216, 4)])
def test_scatter_signals_partition_the_tiles(lib, M, N, world):
    R = T.rows_per_owner(M, world)
    per_owner = [lib.qik_fp8_gemm_scatter_signals(M, N, R, o) for o in range(world)]
    # M > 256 picks CTA pairs (two arrivals per tile) with 256-row tiles 256, 240 or 192
    # wide: every owner counts its row tiles times the same number of column tiles
    col_tiles = {-(-N // bn) for bn in (256, 240, 192)}
    tn = None
    for o, n in enumerate(per_owner):
        rows = max(0, min(R, M - o * R))
        row_tiles = -(-rows // 256)
        if row_tiles == 0:
            assert n == 0
            continue
        assert n % (2 * row_tiles) == 0
        tn = n // (2 * row_tiles) if tn is None else tn
        assert n == 2 * row_tiles * tn
    assert tn in col_tiles
    assert sum(per_owner) == 2 * -(-M // 256) * tn


def test_entry_points_validate_on_host(lib):
    p = ctypes.c_void_p(256)
    arr = (ctypes.c_void_p * 2)(256, 512)
    # rows per owner must be a multiple of 256 covering M
    rc = lib.qik_fp8_gemm_scatter(p, p, 1000, 512, 256, 256, 256, p, p, 2, 500, arr, arr, None, None)
    assert rc == 1 and b"rows per owner" in lib.qik_last_error()
    rc = lib.qik_fp8_gemm_scatter(p, p, 1000, 512, 256, 256, 256, p, p, 9, 512, arr, arr, None, None)
    assert rc == 1 and b"world" in lib.qik_last_error()
    rc = lib.qik_tp_reduce_gather(p, p, 1, 2, 2, 1000, 512, 512, None, arr, arr, 128, None, None)
    assert rc == 1 and b"owner" in lib.qik_last_error()
    rc = lib.qik_tp_reduce_gather(p, p, 1, 2, 0, 1000, 500, 512, None, arr, arr, 128, None, None)
    assert rc == 1 and b"multiple of 8" in lib.qik_last_error()
    assert lib.qik_ipc_handle_bytes() == 64
