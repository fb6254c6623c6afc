"""The N > 1 host path on the CPU: two gloo ranks each compute their row
shard of a small matvecQ8 stack with the oracle (standing in for the GPU
kernel), all-gather the slices, and must reproduce the single-process
result exactly; each rank generates only its shard of the seeded weights."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from xpuops.dist import gathered_to_rows, shard_bytes, shard_rows
from xpuops.synth import fill_normal, tensor_seed


def test_shard_rows_cover_every_row_once():
    for N in (1, 7, 28672, 32001):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                first, count, per = shard_rows(N, world, r)
                assert count <= per
                seen.extend(range(first, first + count))
            assert seen == list(range(N))


def test_fill_normal_start_offset_gives_identical_shards():
    full = fill_normal(4 * 37, 9)
    parts = [fill_normal(37, 9, start=37 * r) for r in range(4)]
    np.testing.assert_array_equal(np.concatenate(parts), full)


def test_shard_bytes_sum():
    tot = sum(shard_bytes(28672, 8192, 8, r, 80) for r in range(8))
    assert tot == 80 * 28672 * (4 * 2048 + 8) + 8 * 4 * 8192


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, M, N, K, out_path):
    import torch
    import torch.distributed as dist

    import oracle.oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    first, rows, per = shard_rows(N, world, rank)
    y = np.zeros((M, per), np.float32)
    x = fill_normal(K, tensor_seed(1, 0))
    for m in range(M):
        wf = fill_normal(rows * K, tensor_seed(0, m), 0.0, 0.02, start=first * K)
        codes, scales = orc.quantize(wf, rows, K)
        y[m, :rows] = orc.matvec_q8(orc.pack_q8(codes, rows, K), scales, x, rows, K)
    parts = [torch.zeros(M * per) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(y.ravel()))
    if rank == 0:
        np.save(out_path, gathered_to_rows(torch.cat(parts).numpy(), world, M, N))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 10), (2, 9)])
def test_two_rank_sharded_stack_matches_single_process(tmp_path, world, N):
    import oracle.oracle as orc

    M, K = 3, 37
    out = tmp_path / "y.npy"
    mp.start_processes(_rank_main, args=(world, _free_port(), M, N, K, str(out)), nprocs=world,
                       start_method="spawn", join=True)
    got = np.load(out)
    x = fill_normal(K, tensor_seed(1, 0))
    for m in range(M):
        wf = fill_normal(N * K, tensor_seed(0, m), 0.0, 0.02)
        codes, scales = orc.quantize(wf, N, K)
        want = orc.matvec_q8(orc.pack_q8(codes, N, K), scales, x, N, K)
        np.testing.assert_array_equal(got[m], want)


def test_single_process_group_rejects_bad_arguments_before_device_work():
    """xpu_dist_create / xpu_dist_matvec_q8_rowshard validate their
    arguments on the host (no device needed for these paths)."""
    import ctypes as C

    from xpuops._lib import XPU_EINVAL, lib

    L = lib()
    h = C.c_void_p()
    assert L.xpu_dist_create(0, None, C.byref(h)) == XPU_EINVAL
    assert L.xpu_dist_create(1, None, C.byref(h)) == XPU_EINVAL
    assert L.xpu_dist_create(1, (C.c_int32 * 1)(0), None) == XPU_EINVAL
    assert L.xpu_dist_matvec_q8_rowshard(None, None, 0, None, None, 1, 8, 8, None) == XPU_EINVAL
    assert L.xpu_dist_destroy(None) == 0
