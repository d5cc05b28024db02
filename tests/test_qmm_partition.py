"""The prefill kernel's work partition, checked on the host (no GPU).

`mt_qmm_partition_check` runs the same segment / split / ownership bookkeeping
the tcgen05 kernel uses (cluster stream-K: C clusters of S CTAs, each cluster's
unit range cut at tile boundaries and every segment split by K among its CTAs;
the cluster holding a tile's first K-stage reduces it) and verifies exact
coverage: every K-stage of every tile computed once, one owner per split tile
summing every partial in K order, every workspace partial written once and read
once. The sweep covers the Qwen3-4B prefill plans and shapes around them.
"""
import ctypes as C

import pytest

from metal_autotune_b200 import lib

# resident clusters per size for the kernel's shared-memory footprint on B200
MAX_CLUSTERS = {1: 148, 2: 74, 3: 45, 4: 33, 6: 22, 8: 15}


def check(tiles, nk, S, C_):
    out = C.c_int64(-1)
    rc = lib.load().mt_qmm_partition_check(tiles, nk, S, C_, C.byref(out))
    return rc, out.value


@pytest.mark.parametrize("tiles,nk,S,C_,max_units", [
    (48, 20, 2, 48, 10),   # qkv: 48 clusters of 2, one tile each
    (20, 32, 4, 20, 8),    # o_proj
    (76, 20, 2, 74, 11),   # gate_up + SwiGLU: 76 tiles on 74 pairs
    (20, 76, 6, 20, 13),   # down
    (1187, 20, 1, 148, 161),
])
def test_qwen3_plans(tiles, nk, S, C_, max_units):
    rc, mu = check(tiles, nk, S, C_)
    assert rc == 0, lib.load().mt_last_error_string()
    assert mu == max_units


def test_partition_sweep():
    n = 0
    for tiles in (1, 2, 3, 5, 7, 10, 20, 36, 48, 76, 100, 150, 300):
        for nk in (1, 2, 3, 4, 5, 8, 20, 32, 76):
            for S, maxc in MAX_CLUSTERS.items():
                if S > 1 and S > nk:
                    continue
                for C_ in sorted({maxc, min(maxc, tiles), min(maxc, tiles * nk)}):
                    if S == 1:
                        C_ = min(tiles * nk, 148)
                    U = tiles * nk
                    # the host plan only uses S > 1 with at most 3 segments per cluster
                    segs = max(((j + 1) * U // C_ - 1) // nk - (j * U // C_) // nk + 1
                               for j in range(C_) if (j + 1) * U // C_ > j * U // C_)
                    if S > 1 and segs > 3:
                        continue
                    rc, mu = check(tiles, nk, S, C_)
                    assert rc == 0, (tiles, nk, S, C_, lib.load().mt_last_error_string())
                    assert mu >= -(-U // (S * C_))
                    n += 1
    assert n > 500


def test_bad_shapes_are_rejected():
    assert check(0, 20, 2, 10)[0] != 0
    assert check(10, 20, 9, 10)[0] != 0      # cluster larger than 8
    assert check(10, 20, 2, 200)[0] != 0     # more CTAs than the workspace provisions
    assert check(10, 1, 2, 5)[0] != 0        # K split finer than the K-stages
    assert check(10, 20, 4, 2)[0] != 0       # more than 3 segments per cluster
