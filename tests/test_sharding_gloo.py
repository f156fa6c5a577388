"""Multi-process sharding logic on the CPU (gloo, world size 2 and 3).

The weight-row partition (pfng_b200_shard_rows), the activation broadcast,
the all-gather of column slices and the column reassembly of the multi-GPU
path, run as real torch.distributed ranks on 127.0.0.1 with the oracle as
the per-rank matmul; the reassembled C must equal the unsharded oracle
result bit for bit.  The fused gather (GatheredC + pfng_b200_compute_gather)
is checked the same way, with shared memory in place of CUDA IPC.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn_ranks(world, m, n, k, granule, tmp_path, body="rank_main"):
    import sharding_worker
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    pkg_dir = os.path.join(os.path.dirname(tests_dir), "qgemm-perf-framework-ng_b200")
    old = os.environ.get("PYTHONPATH", "")
    os.environ["PYTHONPATH"] = os.pathsep.join([tests_dir, pkg_dir] + ([old] if old else []))
    try:
        mp.start_processes(getattr(sharding_worker, body), args=(world, _free_port(), m, n, k, granule, str(tmp_path)),
                           nprocs=world, join=True, start_method="spawn")
    finally:
        os.environ["PYTHONPATH"] = old


@pytest.mark.parametrize("world,n,granule", [(2, 300, 128), (3, 1000, 64), (2, 100, 128)])
def test_sharded_matmul_matches_unsharded(tmp_path, world, n, granule):
    m, k = 3, 256
    _spawn_ranks(world, m, n, k, granule, tmp_path)
    c = np.load(tmp_path / "c_sharded.npy")
    ref = np.load(tmp_path / "c_full.npy")
    np.testing.assert_array_equal(c.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("world,n,granule", [(2, 300, 128), (3, 1000, 64)])
def test_gathered_c_host_logic(tmp_path, world, n, granule):
    # GatheredC's handle exchange, destination order and offsets, and its
    # close protocol, over shared memory standing in for CUDA IPC
    _spawn_ranks(world, 3, n, 256, granule, tmp_path, body="gather_rank_main")
    assert (tmp_path / "gather_ok").exists()


def test_shard_rows_cover_once():
    import pfng_b200 as pb
    for n in (1, 100, 128, 300, 4096, 11008, 32000):
        for world in (1, 2, 3, 4, 8):
            spans = [pb.shard_rows(n, world, r, 128) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
                assert e0 == b1 and b0 <= e0
            # granule counts differ by at most one (only the last granule may be ragged)
            counts = [(e - b + 127) // 128 for b, e in spans]
            assert max(counts) - min(counts) <= 1
            assert all(b % 128 == 0 or b == n for b, _ in spans)
