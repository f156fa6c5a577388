"""Rank body of the multi-process (gloo, CPU) sharding test.

Mirrors the multi-GPU decode/prefill path of bench.py's configs[4] workload
with the oracle in place of the device kernels: rank 0 broadcasts the fp32
activations, every rank quantizes them and computes C for its shard of the
weight rows (pfng_b200_shard_rows), the [m][slice_width] slices are
all-gathered, and the columns are put back in place with the same index
arithmetic as the device unshard kernel (shard.cu).  Not a test module: the
spawned processes import it by name.
"""
import os

import numpy as np


def unshard_host(slices: np.ndarray, m: int, n: int, world: int, granule: int) -> np.ndarray:
    """[world][m][width] -> [m][n], the index arithmetic of unshard_kernel."""
    granules = (n + granule - 1) // granule
    base, extra = granules // world, granules % world
    out = np.empty((m, n), np.float32)
    for j in range(n):
        gi = j // granule
        big = extra * (base + 1)
        r = gi // (base + 1) if gi < big else extra + (gi - big) // base
        g0 = r * base + min(r, extra)
        out[:, j] = slices[r, :, j - g0 * granule]
    return out


def rank_main(rank: int, world: int, port: int, m: int, n: int, k: int, granule: int, result_dir: str) -> None:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import pfng_b200 as pb
    from oracle_lib import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        oracle = Oracle()
        rng = np.random.default_rng(11)  # every rank builds the same full weight matrix
        w_full = oracle.quantize("q4_0", (rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        x = torch.zeros((m, k), dtype=torch.float32)
        if rank == 0:
            x.copy_(torch.from_numpy(np.random.default_rng(12).standard_normal((m, k)).astype(np.float32)))
        dist.broadcast(x, src=0)
        a = oracle.quantize("q8_0", x.numpy())
        b, e = pb.shard_rows(n, world, rank, granule)
        width = max(pb.shard_rows(n, world, r, granule)[1] - pb.shard_rows(n, world, r, granule)[0]
                    for r in range(world))
        slice_ = np.zeros((m, width), np.float32)
        if e > b:
            slice_[:, : e - b] = oracle.mm("q4_0", w_full[b:e], a, m, e - b, k)
        parts = [torch.zeros((m, width)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(slice_))
        if rank == 0:
            c = unshard_host(np.stack([t.numpy() for t in parts]), m, n, world, granule)
            np.save(os.path.join(result_dir, "c_sharded.npy"), c)
            np.save(os.path.join(result_dir, "c_full.npy"), oracle.mm("q4_0", w_full, a, m, n, k))
        dist.barrier()
    finally:
        dist.destroy_process_group()
