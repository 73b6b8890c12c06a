"""CPU tier: the multi-GPU row split on 2 gloo ranks (no GPU).

Checks the host logic of matrixflash_pro_b200.distributed: row partition, column panels,
the packing and broadcast of B's column panels from rank 0, and that each panel's GEMM
writes its own columns of C. The per-panel GEMM is the oracle here (test
infrastructure), standing in for the tcgen05 plan that runs on the GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from matrixflash_pro_b200.distributed import col_panels, row_partition, run_schedule, schedule


def test_row_partition_covers_rows_once():
    for m in (1, 7, 8192, 32768, 1000):
        for world in (1, 2, 3, 4, 8):
            spans = [row_partition(m, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == m
            for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
                assert e0 == b1 and b0 <= e0
    with pytest.raises(Exception):
        row_partition(10, 2, 2)


def test_col_panels():
    assert col_panels(11008, 1) == [(0, 11008)]
    assert col_panels(11008, 8, 4096) == [(0, 1024), (1024, 11008)]  # the linear layer: a 163 MB rest
    # a 4.3 GB B: a 128 MB first panel, then panels doubling while the rest is > 4x the last
    assert col_panels(32768, 8, 32768) == [(0, 1024), (1024, 3072), (3072, 7168), (7168, 15360), (15360, 32768)]
    assert col_panels(300, 4) == [(0, 300)]
    for n, k in ((600, 0), (4097, 100), (5000, 70000), (32768, 4096), (100000, 8192)):
        p = col_panels(n, 4, k)
        assert p[0][0] == 0 and p[-1][1] == n and all(a < b for a, b in p) and p[0][1] % 256 == 0
        assert all(x[1] == y[0] for x, y in zip(p, p[1:]))
        assert all(b1 - b0 <= 2 * (a1 - a0) for (a0, a1), (b0, b1) in zip(p[:-2], p[1:-1]))
        assert len(p) <= 2 or 4 * k * (p[-2][0] - p[-3][1] + (n - p[-2][0])) > 512 << 20
        if k:
            assert p[0][1] - p[0][0] == 256 or (p[0][1] - p[0][0]) * 4 * k <= 128 << 20


def test_schedule_sm_limits():
    s = schedule(11008, 4, 32, 148, 4096)
    assert s.sm_limits == [116, None] and len(s.panels) == 2
    s5 = schedule(32768, 8, 32, 148, 32768)
    assert s5.sm_limits == [116, 116, 116, 116, None] and len(s5.panels) == 5
    s1 = schedule(11008, 1, 16, 148)
    assert s1.panels == [(0, 11008)] and s1.sm_limits == [None]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_dir):
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, n, k, ldb = 37, 600, 70, 611
        alpha, beta = 0.5, 1.0
        rng = np.random.default_rng(0)
        A_full = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        B_full = rng.standard_normal((k, ldb)).astype(np.float32)
        C_full = rng.standard_normal((m, n)).astype(np.float32)
        r0, r1 = row_partition(m, world, rank)
        A = A_full[r0:r1].copy()
        C = C_full[r0:r1].copy()
        B = torch.from_numpy(B_full.copy()) if rank == 0 else torch.full((k, ldb), float("nan"))
        sched = schedule(n, world, 16, 148)
        assert len(sched.panels) == 2
        bufs = [torch.full((k, n1 - n0), float("nan")) for (n0, n1) in sched.panels]

        def pack(i, panel):
            n0, n1 = panel
            bufs[i].copy_(B[:, n0:n1])

        def panel_gemm(i, panel, sm_limit):
            n0, n1 = panel
            cp = np.ascontiguousarray(C[:, n0:n1])
            oracle.gemm_f32(r1 - r0, n1 - n0, k, A, k, bufs[i].numpy(), n1 - n0, cp, n1 - n0, alpha, beta)
            C[:, n0:n1] = cp

        run_schedule(sched, lambda i: bufs[i], pack, panel_gemm)
        np.save(os.path.join(result_dir, f"c{rank}.npy"), C)
        np.save(os.path.join(result_dir, f"b{rank}.npy"), np.concatenate([b.numpy() for b in bufs], axis=1))
    finally:
        dist.destroy_process_group()


def test_row_split_with_panel_broadcast_two_gloo_ranks(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    import oracle
    m, n, k, ldb = 37, 600, 70, 611
    rng = np.random.default_rng(0)
    A_full = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    B_full = rng.standard_normal((k, ldb)).astype(np.float32)
    C_full = rng.standard_normal((m, n)).astype(np.float32)
    got = np.concatenate([np.load(tmp_path / f"c{r}.npy") for r in range(world)])
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"b{r}.npy"), B_full[:, :n]), "B's panels reached every rank"
    ref64 = 0.5 * (A_full.astype(np.float64) @ B_full[:, :n].astype(np.float64)) + C_full
    ref32 = C_full.copy()
    oracle.gemm_f32(m, n, k, A_full, k, B_full, ldb, ref32, n, 0.5, 1.0)
    assert oracle.normwise_rel(got, ref64) <= max(1e-6, oracle.normwise_rel(ref32, ref64))
