"""GPU tier: tile and stream-K selection of GemmPlan.

When whole output tiles would leave workers idle (fewer tiles than SMs or SM pairs, or a
last wave mostly empty), the last tiles share their K blocks among all persistent workers
and a fix-up kernel adds the shares in K order. The reference gets the same kind of choice
from cuBLASLt's heuristic search (src/ops/gemm/plan/implementation.inc:13-60). Every
candidate a plan offers, split or not, is checked against the oracle (the reference's
gemm_f32 and an FP64 product) with the strict-FP32 and TF32 gates of the other GPU tests;
split results must also be bitwise repeatable."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import assert_strict, assert_tf32

pytestmark = pytest.mark.gpu

IMPL = "reference" if oracle.reference_available() else "restatement"
FP32, TF32 = mf.GemmPrecision.fp32, mf.GemmPrecision.tf32


def _ref(a, b, c0, alpha, beta, bias=None, epilogue=0):
    """gemm_f32 and FP64 of untransposed row-major a (m x k), b (k x n), c0 (m x n), plus the epilogue."""
    m, k = a.shape
    n = b.shape[1]
    ref32 = c0.copy()
    oracle.gemm_f32(m, n, k, a, k, b, n, ref32, n, alpha, beta, impl=IMPL)
    ref64 = alpha * (a.astype(np.float64) @ b.astype(np.float64)) + beta * c0.astype(np.float64)
    if epilogue:
        oracle.epilogue_f32(ref32, n, bias, m, n, epilogue - 1)
        ref64 = ref64 + bias.astype(np.float64)
        if epilogue == 2:
            ref64 = np.maximum(ref64, 0.0)
        elif epilogue == 3:
            ref64 = 0.5 * ref64 * (1.0 + np.tanh(0.7978845608 * (ref64 + 0.044715 * ref64 ** 3)))
    return ref32, ref64


def _gate(got, ref32, ref64, a, b, precision, what):
    if precision == FP32:
        return assert_strict(got, ref32, ref64, a.shape[1], float(np.abs(a).max()), float(np.abs(b).max()), what)
    return assert_tf32(got, ref32, what)


def _operands(m, n, k, seed, dist_b="uniform"):
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) if dist_b == "uniform" else rng.standard_normal((k, n))).astype(np.float32)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    return a, b, c0


def _run_plan(plan, A, B, C0, alpha, beta, bias=None):
    C = C0.clone()
    plan.execute(A, B, C, alpha, beta, bias)
    mf.sync()
    return C


@pytest.mark.parametrize("precision", [FP32, TF32])
def test_every_candidate_of_the_2048_cube(precision):
    """2048^3: 64 SM-pair tiles fill 86% of the 74 pairs, so the plan's first choice keeps
    whole tiles (measured faster than sharing K); the 128 x 128 single-CTA candidate (1.73
    waves) shares its last tiles. Every candidate, split or whole, gives the oracle's result."""
    m = n = k = 2048
    a, b, _ = _operands(m, n, k, 1)
    c0 = np.zeros((m, n), np.float32)
    A, B, C0 = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c0).cuda()
    plan = mf.GemmPlan(m, n, k, mf.GemmOptions(precision=precision))
    first = plan.info()
    assert first.stream_k_tiles == 0 and first.sm_pair == 1 and first.split_k == 1, (
        first.stream_k_tiles, first.sm_pair, first.split_k)
    ref32, ref64 = _ref(a, b, c0, 1.0, 0.0)
    kinds = set()
    for i in range(plan.candidate_count()):
        plan.select_candidate(i)
        info = plan.info()
        kinds.add((info.sm_pair, info.tile_n, info.stream_k_tiles > 0))
        got = _run_plan(plan, A, B, C0, 1.0, 0.0)
        _gate(got.cpu().numpy(), ref32, ref64, a, b, precision, f"candidate {i} {kinds}")
        if info.stream_k_tiles:
            again = _run_plan(plan, A, B, C0, 1.0, 0.0)
            assert torch.equal(got, again), "stream-K results must not depend on timing"
    assert (1, 256, False) in kinds and (0, 128, True) in kinds, kinds
    assert mf.device_status(0) == 0


def test_last_wave_shared_4096_cube():
    """4096^3 on SM pairs: 256 tiles are 3.46 waves; the last 108 tiles share their K."""
    m = n = k = 4096
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.rand((m, k), device="cuda", generator=g) * 2 - 1
    B = torch.rand((k, n), device="cuda", generator=g) * 2 - 1
    plan = mf.GemmPlan(m, n, k)
    info = plan.info()
    assert info.sm_pair == 1 and info.stream_k_tiles == 256 - 2 * info.workers, (info.stream_k_tiles, info.workers)
    C = torch.zeros((m, n), device="cuda")
    plan.execute(A, B, C)
    mf.sync()
    ref = A.double() @ B.double()
    err = float((C.double() - ref).norm() / ref.norm())
    assert err <= 1e-6, err
    # rows of the whole tiles and of the shared ones, against the oracle's gemm_f32 and FP64
    a, b = A.cpu().numpy(), B.cpu().numpy()
    rows = np.array([0, 1, 2047, 2048, 3000, 4095])
    cols = np.arange(0, n, 97)
    ref32 = oracle.gemm_f32_sampled(rows, cols, n, k, a, k, b, n)
    got = C.cpu().numpy()[np.ix_(rows, cols)]
    ref64 = (a[rows].astype(np.float64) @ b[:, cols].astype(np.float64))
    assert_strict(got, ref32, ref64, k, 1.0, 1.0, "4096^3 sampled")


def test_long_k_few_tiles_strict():
    """512 x 512 x 65536: 4 SM-pair tiles, K shared by ~18 pairs each."""
    m = n = 512
    k = 65536
    a, b, c0 = _operands(m, n, k, 2, "normal")
    plan = mf.GemmPlan(m, n, k)
    info = plan.info()
    assert info.stream_k_tiles > 0 and info.split_k >= 8, (info.stream_k_tiles, info.split_k)
    got = _run_plan(plan, torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c0).cuda(),
                    0.5, 1.0)
    ref32, ref64 = _ref(a, b, c0, 0.5, 1.0)
    _gate(got.cpu().numpy(), ref32, ref64, a, b, FP32, "512x512x65536")


def _stream_k_candidate(plan):
    for i in range(plan.candidate_count()):
        plan.select_candidate(i)
        if plan.info().stream_k_tiles > 0:
            return i
    return None


@pytest.mark.parametrize("precision", [FP32, TF32])
@pytest.mark.parametrize("m,n,k,ta,tb,ep", [(1000, 600, 3000, False, False, 2), (777, 1333, 2500, True, False, 0),
                                            (300, 2000, 4100, False, True, 3), (129, 520, 9000, True, True, 1)])
def test_stream_k_ragged_shapes_transposes_epilogues(m, n, k, ta, tb, ep, precision):
    a, b, c0 = _operands(m, n, k, m + n)
    bias = np.random.default_rng(k).standard_normal(n).astype(np.float32)
    A = torch.from_numpy(a.T.copy() if ta else a).cuda()
    B = torch.from_numpy(b.T.copy() if tb else b).cuda()
    o = mf.GemmOptions(precision=precision, transpose_left=ta, transpose_right=tb, epilogue=mf.GemmEpilogue(ep))
    plan = mf.GemmPlan(m, n, k, o)
    idx = _stream_k_candidate(plan)
    assert idx is not None, "no stream-K candidate"
    got = _run_plan(plan, A, B, torch.from_numpy(c0).cuda(), 0.75, -0.5,
                    torch.from_numpy(bias).cuda() if ep else None)
    ref32, ref64 = _ref(a, b, c0, 0.75, -0.5, bias if ep else None, ep)
    _gate(got.cpu().numpy(), ref32, ref64, a, b, precision, f"{m}x{n}x{k} ta={ta} tb={tb} ep={ep}")


def test_one_shot_and_batched_calls_take_the_split_path():
    """mfb_sgemm (per-stream scratch sized for the partial slots) and a strided batch."""
    m, n, k = 512, 384, 20000
    a, b, c0 = _operands(m, n, k, 9)
    C = torch.from_numpy(c0).cuda()
    mf.sgemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), C, 1.0, 1.0)
    mf.sync()
    ref32, ref64 = _ref(a, b, c0, 1.0, 1.0)
    _gate(C.cpu().numpy(), ref32, ref64, a, b, FP32, "sgemm 512x384x20000")

    nb, m, n, k = 3, 300, 500, 6000
    rng = np.random.default_rng(4)
    a = rng.uniform(-1, 1, (nb, m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (nb, k, n)).astype(np.float32)
    C = torch.zeros((nb, m, n), device="cuda")
    mf.sgemm_strided_batched(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), C, 1.0, 0.0)
    mf.sync()
    got = C.cpu().numpy()
    for i in range(nb):
        ref32, ref64 = _ref(a[i], b[i], np.zeros((m, n), np.float32), 1.0, 0.0)
        _gate(got[i], ref32, ref64, a[i], b[i], FP32, f"batch entry {i}")
    assert mf.device_status(0) == 0


def test_stream_k_plan_replays_in_a_cuda_graph():
    """A plan whose last tiles share K (GEMM + fix-up, both launched programmatically) captures into a
    CUDA graph; replays give the eager bits and read updated inputs."""
    m = n = 512
    k = 16384
    g = torch.Generator(device="cuda").manual_seed(21)
    A = torch.randn((m, k), device="cuda", generator=g)
    B = torch.randn((k, n), device="cuda", generator=g)
    C0 = torch.randn((m, n), device="cuda", generator=g)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        plan = mf.GemmPlan(m, n, k)
        assert plan.info().stream_k_tiles > 0
        eager = C0.clone()
        plan.execute(A, B, eager, 0.5, 1.0)
        C = C0.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            plan.execute(A, B, C, 0.5, 1.0)
        C.copy_(C0)
        graph.replay()
    side.synchronize()
    assert torch.equal(C, eager)
    with torch.cuda.stream(side):
        B.mul_(2.0)
        C.copy_(C0)
        graph.replay()
        want = C0.clone()
        plan.execute(A, B, want, 0.5, 1.0)
    side.synchronize()
    assert torch.equal(C, want)
    mf.sync()
