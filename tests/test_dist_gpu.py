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
