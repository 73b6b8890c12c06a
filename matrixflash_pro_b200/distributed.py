"""Row-split multi-GPU GEMM: C = alpha * A * B + beta * C over P ranks (one process per GPU).

Rank r owns rows [r*m/P, (r+1)*m/P) of A and C; B (k x n) lives on rank 0 and reaches
every rank by an NCCL broadcast over NVLink/NVSwitch. The broadcast is issued in K
panels (rows of B) on NCCL's stream; the GEMM runs panel by panel as
C = alpha * A[:, panel] * B[panel, :] + beta' * C (beta' = beta for the first panel,
1 afterwards), each panel waiting only for its own broadcast, so the transfer of
panel i+1 overlaps the GEMM of panel i. While later panels are still in flight the
GEMM runs on a capped grid so NCCL keeps SMs to run on. No output collective: C
stays row-sharded.

The reference's precedent is the CPU/GPU row split of HeterogeneousScheduler
(src/hw/scheduler.cpp:182-312), whose B transfer is host-staged
(src/hw/collectives.cpp:219-235); the reference never calls NCCL
(src/hw/cuda_backend.cu:252).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .errors import InvalidArgumentError
from .gemm import GemmPrecision, _stream_handle, make_desc


def row_partition(m: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [begin, end) of rank `rank`: ceil(m / world) per rank, the last rank takes the rest."""
    if world < 1 or not 0 <= rank < world:
        raise InvalidArgumentError("bad world/rank")
    per = -(-m // world)
    begin = min(m, rank * per)
    return begin, min(m, begin + per)


def k_panels(k: int, world: int, first_fraction: float = 0.125, align: int = 32) -> List[Tuple[int, int]]:
    """K panels for the broadcast/GEMM pipeline: one small leading panel (its broadcast is
    the only exposed transfer) and one panel for the rest. A single panel without peers."""
    if world <= 1 or k <= 2 * align:
        return [(0, k)]
    first = max(align, int(k * first_fraction) // align * align)
    if first >= k:
        return [(0, k)]
    return [(0, first), (first, k)]


PanelGemm = Callable[[int, Tuple[int, int], float, Optional[int]], None]


@dataclass
class PanelSchedule:
    """What one step does, in order: broadcast every panel, then per panel wait + GEMM."""
    panels: List[Tuple[int, int]]
    betas: List[float]
    sm_limits: List[Optional[int]]


def schedule(k: int, world: int, beta: float, comm_sms: int, total_sms: int) -> PanelSchedule:
    panels = k_panels(k, world)
    betas = [beta] + [1.0] * (len(panels) - 1)
    # While later panels are still broadcasting, leave comm_sms SMs to NCCL.
    limits = [max(1, total_sms - comm_sms) if i < len(panels) - 1 else None for i in range(len(panels))]
    return PanelSchedule(panels, betas, limits)


def run_schedule(sched: PanelSchedule, b_rows: Callable[[int, int], torch.Tensor], panel_gemm: PanelGemm,
                 group=None, src: int = 0,
                 before_wait: Optional[Callable[[int, Tuple[int, int]], None]] = None) -> None:
    """Issues the broadcasts (async, NCCL stream), then `before_wait(i, panel)` for every
    panel (work that does not read B, e.g. preparing A), then the per-panel GEMMs (current
    stream). `b_rows(k0, k1)` returns the contiguous row block of B's storage for a panel."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    works = []
    if world > 1:
        for (k0, k1) in sched.panels:
            works.append(dist.broadcast(b_rows(k0, k1), src=src, group=group, async_op=True))
    if before_wait is not None:
        for i, panel in enumerate(sched.panels):
            before_wait(i, panel)
    for i, panel in enumerate(sched.panels):
        if works:
            works[i].wait()  # current stream waits for this panel's broadcast only
        panel_gemm(i, panel, sched.betas[i], sched.sm_limits[i])


class _PointerPlan:
    """An mfb plan over explicit leading dimensions (panel views of padded operands)."""

    def __init__(self, device: int, m: int, n: int, k: int, lda: int, ldb: int, ldc: int, precision: int):
        self.desc = make_desc(m, n, k, lda, ldb, ldc, 1.0, 0.0, precision)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().mfb_plan_create(device, ctypes.byref(self.desc), ctypes.byref(h)), "panel plan")
        self.handle = h
        self.sm_limit = 0

    def set_sm_limit(self, sms: Optional[int]) -> None:
        sms = int(sms or 0)
        if sms != self.sm_limit:
            _lib.check(_lib.lib().mfb_plan_set_sm_limit(self.handle, sms), "panel plan sm limit")
            self.sm_limit = sms

    def prepare(self, stream: int, a: int, b: int) -> None:
        _lib.check(_lib.lib().mfb_plan_prepare(self.handle, stream, a, b), "panel prepare")

    def multiply(self, stream: int, a: int, b: int, c: int, alpha: float, beta: float) -> None:
        _lib.check(_lib.lib().mfb_plan_multiply(self.handle, stream, a, b, c, alpha, beta, 0), "panel multiply")

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            _lib.lib().mfb_plan_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RowSplitGemm:
    """This rank's share of a row-split strict-FP32 (or TF32) GEMM with B broadcast.

    A_local: (m_local x k) view of an (m_local x lda) buffer; B: (k x n) view of a
    (k x ldb) buffer, valid on `src` and overwritten by the broadcast elsewhere;
    C_local: (m_local x n) view of an (m_local x ldc) buffer."""

    def __init__(self, m_local: int, n: int, k: int, lda: int, ldb: int, ldc: int,
                 precision: GemmPrecision = GemmPrecision.fp32, group=None, src: int = 0, comm_sms: int = 16):
        self.device = torch.cuda.current_device()
        self.group, self.src = group, src
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.m, self.n, self.k = m_local, n, k
        self.lda, self.ldb, self.ldc = lda, ldb, ldc
        total_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.sched = schedule(k, self.world, 0.0, comm_sms, total_sms)
        self.plans = [_PointerPlan(self.device, m_local, n, k1 - k0, lda, ldb, ldc, int(precision))
                      for (k0, k1) in self.sched.panels]
        # Per-panel GEMM kernel time of the last step, when events are requested.
        self.kernel_events: List[Tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def __call__(self, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
                 time_kernels: bool = False) -> None:
        stream = _stream_handle()
        a0, b0, c0 = A.data_ptr(), B.data_ptr(), C.data_ptr()
        sched = PanelSchedule(self.sched.panels, [beta] + [1.0] * (len(self.sched.panels) - 1), self.sched.sm_limits)
        self.kernel_events = []

        split_a_early = self.world > 1

        def prepare_a(i, panel):
            # A's split/rounding prepass does not read B: it runs while B is in flight.
            self.plans[i].prepare(stream, a0 + 4 * panel[0], 0)

        def panel_gemm(i, panel, pbeta, sm_limit):
            k0, _ = panel
            plan = self.plans[i]
            a_ptr = a0 + 4 * k0
            b_ptr = b0 + 4 * k0 * self.ldb
            # one prepass launch for both operands unless A's was issued during the broadcast
            plan.prepare(stream, 0 if split_a_early else a_ptr, b_ptr)
            plan.set_sm_limit(sm_limit)
            if time_kernels:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            plan.multiply(stream, a_ptr, b_ptr, c0, alpha, pbeta)
            if time_kernels:
                e1.record()
                self.kernel_events.append((e0, e1))

        def b_rows(k0, k1):
            return B.as_strided((k1 - k0, self.ldb), (self.ldb, 1), B.storage_offset() + k0 * self.ldb)

        run_schedule(sched, b_rows, panel_gemm, self.group, self.src,
                     before_wait=prepare_a if split_a_early else None)

    def launches_per_step(self) -> int:
        """Kernels of this library per step, per panel: the operand prepass (hi/lo split, or TF32
        rounding; A's separately while B is broadcast) and the GEMM."""
        return (3 if self.world > 1 else 2) * len(self.plans)

    def kernel_ms(self) -> float:
        return sum(e0.elapsed_time(e1) for (e0, e1) in self.kernel_events)

    def panel_flops(self) -> List[float]:
        return [2.0 * self.m * self.n * (k1 - k0) for (k0, k1) in self.sched.panels]

    def close(self) -> None:
        for p in self.plans:
            p.close()
        self.plans = []
