"""GPU tier (2+ GPUs): the row-split GEMM with B broadcast by NCCL, one process per GPU.

Each rank computes its rows of C = alpha*A*B + beta*C with B arriving from rank 0 in K
panels (matrixflash_pro_b200.distributed.RowSplitGemm); the parent compares the
assembled C with the oracle. Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

M, N, K, LDA, LDB, LDC = 1000, 700, 2080, 2084, 704, 708
ALPHA, BETA = 0.5, 1.0


def _inputs():
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (M, LDA)).astype(np.float32)
    b = rng.standard_normal((K, LDB)).astype(np.float32)
    c = rng.standard_normal((M, LDC)).astype(np.float32)
    return a, b, c


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir, precision):
    import datetime
    import torch.distributed as dist
    import matrixflash_pro_b200 as mf
    from matrixflash_pro_b200.distributed import RowSplitGemm, row_partition
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        a, b, c = _inputs()
        r0, r1 = row_partition(M, world, rank)
        A = torch.from_numpy(a[r0:r1]).cuda()
        B = torch.from_numpy(b).cuda() if rank == 0 else torch.full((K, LDB), float("nan"), device="cuda")
        C = torch.from_numpy(c[r0:r1]).cuda()
        op = RowSplitGemm(r1 - r0, N, K, LDA, LDB, LDC, mf.GemmPrecision(precision))
        op(A[:, :K], B[:, :N], C[:, :N], ALPHA, BETA)
        torch.cuda.synchronize()
        mf.sync()
        np.save(os.path.join(out_dir, f"c{rank}.npy"), C.cpu().numpy())
        assert len(op.sched.panels) == (2 if world > 1 else 1)
        op.close()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("precision", [0, 1])
def test_row_split_broadcast_two_gpus(tmp_path, precision):
    import torch.multiprocessing as mp
    import oracle
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), precision), nprocs=world,
                       start_method="spawn")
    got = np.concatenate([np.load(tmp_path / f"c{r}.npy") for r in range(world)])
    a, b, c = _inputs()
    assert np.array_equal(got[:, N:], c[:, N:])
    ref32 = c.copy()
    oracle.gemm_f32(M, N, K, a, LDA, b, LDB, ref32, LDC, ALPHA, BETA)
    ref32 = ref32[:, :N]
    if precision == 0:
        ref64 = oracle.gemm_f64(M, N, K, a, LDA, b, LDB, c, LDC, ALPHA, BETA)
        assert oracle.normwise_rel(got[:, :N], ref64) <= max(1e-6, oracle.normwise_rel(ref32, ref64))
    else:
        assert oracle.normwise_rel(got[:, :N], ref32) <= 5e-3
