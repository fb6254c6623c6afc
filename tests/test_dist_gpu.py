"""The row-sharded matvecQ8 stack on 2 GPUs: one process per GPU over NCCL,
each computes its row shard (generated on its own GPU from the seeded
stream's offset), the slices are all-gathered, and the result must equal
the unsharded GEMV on one GPU bit for bit, on both matvecQ8 paths (a row's
CUDA-core summation order depends on K only; the tensor-core sums are exact
integers, whichever CTAs and GPU compute them).  Skipped with fewer than 2
GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

M, N, K = 3, 1024, 8192


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard(rank_rows, first_row):
    """Rows [first_row, first_row + rank_rows) of every matrix and x, on the
    current device."""
    from xpuops import ops
    from xpuops.synth import tensor_seed

    W = K // 4
    w = torch.empty(M * rank_rows * W, dtype=torch.int32, device="cuda")
    s = torch.empty(M * rank_rows, dtype=torch.float32, device="cuda")
    tmp = torch.empty(rank_rows * K, dtype=torch.float32, device="cuda")
    for m in range(M):
        ops.fill_normal_dev(tmp, rank_rows * K, tensor_seed(7, m), 0.0, 0.02, start=first_row * K)
        ops.quantizePackQ8_dev(tmp, rank_rows, K, w.data_ptr() + 4 * m * rank_rows * W, s.data_ptr() + 4 * m * rank_rows)
    x = torch.empty(K, dtype=torch.float32, device="cuda")
    ops.fill_normal_dev(x, K, tensor_seed(8, 0))
    torch.cuda.synchronize()
    return w, s, x


def _stack(rank_rows, first_row):
    from xpuops import ops

    W = K // 4
    w, s, x = _shard(rank_rows, first_row)
    y = torch.empty(M * rank_rows, dtype=torch.float32, device="cuda")
    ops.matvecQ8Stack_dev(w, rank_rows * W, s, x, M, rank_rows, K, y)
    torch.cuda.synchronize()
    return y


def _rank(rank, world, port, out, path):
    from datetime import timedelta

    import torch.distributed as dist

    from xpuops import ops
    from xpuops.dist import gathered_to_rows, shard_rows

    ops.setMatvecPath(path)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    first, rows, per = shard_rows(N, world, rank)
    y = _stack(rows, first)
    full = torch.empty(world * M * per, dtype=torch.float32, device="cuda")
    dist.all_gather_into_tensor(full, y)
    if rank == 0:
        np.save(out, gathered_to_rows(full.cpu().numpy(), world, M, N))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("path", ["cuda_cores", "tensor_cores"])
def test_two_gpu_row_shard_equals_one_gpu(tmp_path, path):
    from xpuops import ops

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    code = {"cuda_cores": ops.MATVEC_CUDA_CORES, "tensor_cores": ops.MATVEC_TENSOR_CORES}[path]
    out = tmp_path / "y.npy"
    mp.start_processes(_rank, args=(2, _port(), str(out), code), nprocs=2, start_method="spawn", join=True)
    torch.cuda.set_device(0)
    ops.setMatvecPath(code)
    try:
        single = _stack(N, 0).cpu().numpy().reshape(M, N)
    finally:
        ops.setMatvecPath(ops.MATVEC_AUTO)
    np.testing.assert_array_equal(np.load(out), single)


@pytest.mark.parametrize("path", ["cuda_cores", "tensor_cores"])
def test_single_process_group_equals_one_gpu(path):
    """xpu_dist_matvec_q8_rowshard: one process, two GPUs, each with its row
    shard; every device ends with the whole stack's output, bit-identical to
    the unsharded stack on one GPU."""
    from xpuops import ops
    from xpuops.dist import RowShardGroup

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    code = {"cuda_cores": ops.MATVEC_CUDA_CORES, "tensor_cores": ops.MATVEC_TENSOR_CORES}[path]
    G, W = 2, K // 4
    R = N // G
    shards, outs = [], []
    for g in range(G):
        torch.cuda.set_device(g)
        shards.append(_shard(R, g * R))
        outs.append(torch.full((M * N,), float("nan"), dtype=torch.float32, device="cuda"))
    ops.setMatvecPath(code)
    try:
        with RowShardGroup(range(G)) as grp:
            grp.matvecQ8StackRowShard([sh[0] for sh in shards], R * W, [sh[1] for sh in shards],
                                      [sh[2] for sh in shards], M, N, K, outs)
        torch.cuda.set_device(0)
        single = _stack(N, 0).cpu().numpy()
    finally:
        ops.setMatvecPath(ops.MATVEC_AUTO)
    for g in range(G):
        np.testing.assert_array_equal(outs[g].cpu().numpy(), single)


def _fused_rank(rank, world, port, out):
    """One process per GPU: this rank's shard through
    xpu_matvec_q8_stack_allgather_dev, every rank's output mapped over CUDA
    IPC; three calls (epochs 1-3, two output buffers in turn)."""
    from datetime import timedelta

    import torch.distributed as dist

    from xpuops import ops
    from xpuops.dist import shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    first, rows, per = shard_rows(N, world, rank)
    assert rows == per  # N divides
    w, s, x = _shard(rows, first)
    W = K // 4
    outs = [ops.DeviceBuffer(4 * M * N) for _ in range(2)]
    flags = ops.DeviceBuffer(4 * world)
    flags.upload(np.zeros(world, np.uint32))
    mine = [ops.ipcHandle(o) for o in outs] + [ops.ipcHandle(flags)]
    every = [None] * world
    dist.all_gather_object(every, mine)
    peer = [[ops.ipcOpen(h) if r != rank else None for h in every[r]] for r in range(world)]
    ptr = lambda r, i: (outs[i].ptr if i < 2 else flags.ptr) if r == rank else peer[r][i]
    results = []
    for epoch in (1, 2, 3):
        b = epoch % 2
        ops.matvecQ8StackAllGather_dev(w, rows * W, s, x, M, rows, K, rank, world, [ptr(r, b) for r in range(world)],
                                       [ptr(r, 2) for r in range(world)], epoch)
        ops.stream_sync()
        results.append(outs[b].download(np.float32, M * N))
    got_flags = flags.download(np.uint32, world)
    dist.barrier()  # every rank's kernels are done before any mapping closes
    for r in range(world):
        for p_ in peer[r]:
            if p_:
                ops.ipcClose(p_)
    dist.barrier()
    if rank == 0:
        np.save(out, np.stack(results))
        np.save(str(out) + ".flags.npy", got_flags)
    dist.destroy_process_group()


def test_fused_allgather_two_processes_equals_one_gpu(tmp_path):
    """xpu_matvec_q8_stack_allgather_dev on 2 GPUs, one process each: the
    GEMV epilogue writes every row into both GPUs' outputs over NVLink, and
    each call returns with the whole stack's output in place, bit-identical
    to the unsharded tensor-core stack on one GPU, on three calls in a row."""
    from xpuops import ops

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "fused.npy"
    mp.start_processes(_fused_rank, args=(2, _port(), str(out)), nprocs=2, start_method="spawn", join=True)
    torch.cuda.set_device(0)
    ops.setMatvecPath(ops.MATVEC_TENSOR_CORES)
    try:
        single = _stack(N, 0).cpu().numpy()
    finally:
        ops.setMatvecPath(ops.MATVEC_AUTO)
    got = np.load(out)
    for i in range(3):
        np.testing.assert_array_equal(got[i], single)
    assert np.load(str(out) + ".flags.npy").tolist() == [3, 3]


def test_fused_allgather_contract_errors():
    """Argument checks happen before any device work."""
    import xpuops
    from xpuops import ops

    z = ops.DeviceBuffer(4096)
    with pytest.raises(xpuops.XpuInvalidArgument, match="rank 2 of 2"):
        ops.matvecQ8StackAllGather_dev(z, 512, z, z, 1, 8, 2048, 2, 2, [z, z], [z, z], 1)
    with pytest.raises(xpuops.XpuInvalidArgument, match="epoch 0"):
        ops.matvecQ8StackAllGather_dev(z, 512, z, z, 1, 8, 2048, 0, 1, [z], [z], 0)
    with pytest.raises(xpuops.XpuInvalidArgument, match="tensor-core path"):
        ops.matvecQ8StackAllGather_dev(z, 513, z, z, 1, 8, 2050, 0, 1, [z], [z], 1)
