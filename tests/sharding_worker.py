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


class ShmIpc:
    """Host stand-in for the CUDA IPC calls GatheredC makes: buffers are POSIX
    shared memory, the handle is the segment's name and a pointer is the
    mapping's address in this process."""

    def __init__(self):
        self.blocks = {}

    def _map(self, shm):
        import ctypes
        view = ctypes.c_char.from_buffer(shm.buf)
        ptr = ctypes.addressof(view)
        self.blocks[ptr] = (shm, view)
        return ptr

    def alloc(self, nbytes):
        from multiprocessing import shared_memory
        shm = shared_memory.SharedMemory(create=True, size=nbytes)
        return self._map(shm), shm.name.encode().ljust(64, b"\0")

    def open(self, handle):
        from multiprocessing import resource_tracker, shared_memory
        shm = shared_memory.SharedMemory(name=handle.rstrip(b"\0").decode())
        resource_tracker.unregister(shm._name, "shared_memory")  # the owner unlinks it
        return self._map(shm)

    def _drop(self, ptr):
        shm, view = self.blocks.pop(ptr)
        del view
        shm.close()
        return shm

    def close(self, ptr):
        self._drop(ptr)

    def free(self, ptr):
        self._drop(ptr).unlink()


def float_array(ptr: int, count: int) -> np.ndarray:
    import ctypes
    return np.ctypeslib.as_array((ctypes.c_float * count).from_address(ptr))


def gather_rank_main(rank: int, world: int, port: int, m: int, n: int, k: int, granule: int, result_dir: str) -> None:
    """GatheredC's host logic with real gloo ranks: each rank writes the
    oracle's C for its weight rows into every destination GatheredC gives it
    (what the GEMM epilogue does on the device), then every rank's full C
    must equal the unsharded oracle result."""
    import torch.distributed as dist
    from datetime import timedelta

    import pfng_b200 as pb
    from oracle_lib import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        oracle = Oracle()
        rng = np.random.default_rng(21)
        w_full = oracle.quantize("q4_0", (rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        a = oracle.quantize("q8_0", np.random.default_rng(22).standard_normal((m, k)).astype(np.float32))
        out = pb.GatheredC(m, n, ipc=ShmIpc())
        b, e = pb.shard_rows(n, world, rank, granule)
        dsts = out.destinations(b)
        assert len(dsts) == world and dsts[0] == out.ptr + 4 * b
        if e > b:
            part = oracle.mm("q4_0", w_full[b:e], a, m, e - b, k)
            for d in dsts:
                for i in range(m):
                    float_array(d + 4 * i * n, e - b)[:] = part[i]
        dist.barrier()
        c = float_array(out.ptr, m * n).reshape(m, n).copy()
        ref = oracle.mm("q4_0", w_full, a, m, n, k)
        np.testing.assert_array_equal(c.view(np.uint32), ref.view(np.uint32))
        out.close()
        assert out.bases is None
        if rank == 0:
            open(os.path.join(result_dir, "gather_ok"), "w").close()
    finally:
        dist.destroy_process_group()


def gather_gpu_rank_main(rank: int, world: int, port: int, m: int, n: int, k: int, granule: int,
                         path: str) -> None:
    """compute_gather across processes through CUDA IPC (one GPU per rank, or
    ranks sharing a GPU on a one-GPU box; no kernel waits on another rank):
    every rank's full C must hold, per rank's slice, exactly what compute()
    gives for that slice."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import pfng_b200 as pb

    torch.cuda.set_device(rank % torch.cuda.device_count())
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        gen = torch.Generator(device="cuda").manual_seed(5)
        w_full = pb.quantize_q4_0(torch.randn((n, k), generator=gen, device="cuda") * 0.02)
        x = torch.randn((m, k), generator=gen, device="cuda")
        row_bytes = k // 32 * pb.Q4_0_BYTES
        spans = [pb.shard_rows(n, world, r, granule) for r in range(world)]
        out = pb.GatheredC(m, n)
        c = out.tensor()
        c.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        b, e = spans[rank]
        if e > b:
            pb.compute_gather("q4_0", w_full[b * row_bytes: e * row_bytes], x, e - b, out.destinations(b), n,
                              path=path)
        torch.cuda.synchronize()
        dist.barrier()
        got = c.cpu()
        for r, (rb, re) in enumerate(spans):
            if re > rb:
                ref = pb.compute("q4_0", w_full[rb * row_bytes: re * row_bytes], x, re - rb, path=path).cpu()
                assert torch.equal(got[:, rb:re].view(torch.int32), ref.view(torch.int32)), f"rank {r} slice"
        pb.check_kernel_error()
        torch.cuda.synchronize()
        out.close()
    finally:
        dist.destroy_process_group()
