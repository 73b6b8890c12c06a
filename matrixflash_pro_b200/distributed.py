"""Row-split multi-GPU GEMM: C = alpha * A * B + beta * C over P ranks (one process per GPU).

Rank r owns rows [r*m/P, (r+1)*m/P) of A and C; B (k x n) lives on rank 0 and reaches
every rank by NCCL broadcasts over NVLink/NVSwitch. B travels in column panels: rank 0
packs each panel B[:, n0:n1] into a contiguous k x (n1 - n0) buffer and broadcasts it on
NCCL's stream. Every rank splits A once per step while the panels are in flight, then per
panel waits for that panel only, splits it into the plan's B planes (its columns) and
computes C[:, n0:n1] = alpha * A * B[:, n0:n1] + beta * C[:, n0:n1] on the tcgen05 plan.
Each column of C is written once (a split along K would read and write all of C once per
panel), so the first panel, whose broadcast is the only exposed transfer, can be small.
While later panels are still in flight the GEMM runs on a capped grid so NCCL keeps SMs
to run on. No output collective: C stays row-sharded.

The reference's precedent is the CPU/GPU row split of HeterogeneousScheduler
(src/hw/scheduler.cpp:182-312), whose B transfer is host-staged
(src/hw/collectives.cpp:219-235); the reference never calls NCCL
(src/hw/cuda_backend.cu:252).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .errors import InvalidArgumentError
from .gemm import GemmPrecision, _stream_handle, make_desc


def sgemm_multi(a_blocks: List[torch.Tensor], b: torch.Tensor, c_blocks: List[torch.Tensor], alpha: float = 1.0,
                beta: float = 0.0, precision: GemmPrecision = GemmPrecision.fp32, root: int = 0,
                bias: Optional[torch.Tensor] = None, epilogue: int = 0) -> None:
    """The row split inside one process (mfb_sgemm_multi): block r of A (rows_r x k) and of C
    (rows_r x n) on its own GPU, B (k x n) and the bias on block `root`'s GPU; B reaches the other
    GPUs by NCCL broadcasts in column panels. Blocking. Row strides come from the tensors (padded
    rows allowed); all blocks share lda and ldc."""
    if len(a_blocks) != len(c_blocks) or not a_blocks:
        raise InvalidArgumentError("one A block and one C block per GPU")
    from .gemm import _ld
    k, n = int(b.shape[0]), int(b.shape[1])
    lda = max(_ld(t, "A") for t in a_blocks) if k else 1
    ldc = max(_ld(t, "C") for t in c_blocks)
    blocks = (_lib.RowBlock * len(a_blocks))()
    m = 0
    for i, (a, c) in enumerate(zip(a_blocks, c_blocks)):
        if int(a.shape[0]) != int(c.shape[0]) or int(c.shape[1]) != n or int(a.shape[1]) != k:
            raise InvalidArgumentError("A and C blocks must have matching rows, k and n")
        if int(c.shape[0]) > 1 and ((k and _ld(a, "A") != lda) or _ld(c, "C") != ldc):
            raise InvalidArgumentError("all A blocks share one row stride, and all C blocks another")
        blocks[i] = _lib.RowBlock(c.device.index, int(c.shape[0]), a.data_ptr() if a.numel() else 0, c.data_ptr())
        m += int(c.shape[0])
    desc = make_desc(m, n, k, lda, _ld(b, "B") if k else max(1, n), ldc, alpha, beta, int(precision), 0, 0, epilogue)
    _lib.check(_lib.lib().mfb_sgemm_multi(blocks, len(a_blocks), int(root), ctypes.byref(desc), b.data_ptr(),
                                          bias.data_ptr() if bias is not None else 0), "sgemm_multi")


def row_partition(m: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [begin, end) of rank `rank`: ceil(m / world) per rank, the last rank takes the rest."""
    if world < 1 or not 0 <= rank < world:
        raise InvalidArgumentError("bad world/rank")
    per = -(-m // world)
    begin = min(m, rank * per)
    return begin, min(m, begin + per)


def col_panels(n: int, world: int, k: int = 0, first_fraction: float = 0.1, tile: int = 256,
               max_first_bytes: int = 128 << 20, max_rest_bytes: int = 512 << 20,
               stop_ratio: int = 4) -> List[Tuple[int, int]]:
    """Column panels for the broadcast/GEMM pipeline. A single panel without peers.

    The first panel's broadcast is the only transfer nothing hides, so it is small: a tenth of
    the columns in whole 256-column tiles (measured best on 2 B200s for the linear layer,
    n = 11008: 1024 columns, then the rest), and at most max_first_bytes of B. Each later panel
    must arrive while the GEMM of the one before runs; a panel's GEMM takes 2 * m_local * k FLOP
    per column and its transfer 4 * k bytes per column, so with m_local in the thousands a panel
    twice as wide as the previous one arrives in time. While the rest of B is larger than
    max_rest_bytes and than stop_ratio times the last panel, the next panel is twice the last;
    the rest is the final panel. For n = 32768, k = 32768 (a 4.3 GB B): 1024, 2048, 4096, 8192,
    17408 columns, where a tenth plus the rest (3072 + 29696) would leave the GPUs waiting for a
    3.9 GB second panel. The linear layer (a 163 MB rest) keeps its two panels."""
    if world <= 1 or n <= 2 * tile:
        return [(0, n)]
    first = max(tile, int(n * first_fraction) // tile * tile)
    if k > 0:
        first = min(first, max(tile, max_first_bytes // (4 * k) // tile * tile))
    if first >= n:
        return [(0, n)]
    panels = [(0, first)]
    width, start = first, first
    while 4 * k * (n - start) > max_rest_bytes and n - start > stop_ratio * width:
        width *= 2
        panels.append((start, start + width))
        start += width
    panels.append((start, n))
    return panels


@dataclass
class PanelSchedule:
    """What one step does, in order: broadcast every panel, then per panel wait + GEMM."""
    panels: List[Tuple[int, int]]
    sm_limits: List[Optional[int]]


def schedule(n: int, world: int, comm_sms: int, total_sms: int, k: int = 0) -> PanelSchedule:
    panels = col_panels(n, world, k)
    # While later panels are still broadcasting, leave comm_sms SMs to NCCL.
    limits = [max(1, total_sms - comm_sms) if i < len(panels) - 1 else None for i in range(len(panels))]
    return PanelSchedule(panels, limits)


def run_schedule(sched: PanelSchedule, panel_buffer: Callable[[int], torch.Tensor],
                 pack_panel: Callable[[int, Tuple[int, int]], None],
                 panel_gemm: Callable[[int, Tuple[int, int], Optional[int]], None],
                 group=None, src: int = 0, before_wait: Optional[Callable[[], None]] = None,
                 prepare_panel: Optional[Callable[[int, Tuple[int, int]], None]] = None,
                 side: Optional["torch.cuda.Stream"] = None) -> None:
    """On `src`, `pack_panel(i, panel)` fills panel_buffer(i) before its broadcast; packs and
    broadcasts are issued from the `side` stream when one is given (NCCL's stream waits for
    it), so the current stream goes straight on to `before_wait()` (work that does not read
    B, e.g. preparing A). Then per panel the current stream waits for that panel's broadcast
    only and runs `panel_gemm(i, panel, sm_limit)`. With `prepare_panel`, panels after the
    first are prepared on `side` as soon as they arrive (overlapping the previous panel's
    GEMM) and panel_gemm waits for that instead."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    main = torch.cuda.current_stream() if side is not None else None
    if side is not None:
        side.wait_stream(main)  # B (and the panel buffers) as the caller's stream left them
    works = []
    with torch.cuda.stream(side) if side is not None else _nullcontext():
        for i, panel in enumerate(sched.panels):
            if rank == src:
                pack_panel(i, panel)
            if world > 1:
                works.append(dist.broadcast(panel_buffer(i), src=src, group=group, async_op=True))
    if before_wait is not None:
        before_wait()
    ready = [None] * len(sched.panels)
    if prepare_panel is not None and side is not None:
        with torch.cuda.stream(side):
            for i, panel in enumerate(sched.panels):
                if i == 0:
                    continue
                if works:
                    works[i].wait()  # side stream waits for this panel's broadcast
                prepare_panel(i, panel)
                ev = torch.cuda.Event()
                ev.record(side)
                ready[i] = ev
    for i, panel in enumerate(sched.panels):
        if ready[i] is not None:
            main.wait_event(ready[i])
        else:
            if works:
                works[i].wait()  # current stream waits for this panel's broadcast only
            if prepare_panel is not None:
                prepare_panel(i, panel)
        panel_gemm(i, panel, sched.sm_limits[i])
    if side is not None:
        main.wait_stream(side)  # nothing of the step is left behind on the side stream


class _nullcontext:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


class _PointerPlan:
    """An mfb plan over explicit leading dimensions."""

    def __init__(self, device: int, m: int, n: int, k: int, lda: int, ldb: int, ldc: int, precision: int):
        self.desc = make_desc(m, n, k, lda, ldb, ldc, 1.0, 0.0, precision)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().mfb_plan_create(device, ctypes.byref(self.desc), ctypes.byref(h)), "row-split plan")
        self.handle = h
        self.sm_limit = 0
        info = _lib.PlanInfo()
        _lib.check(_lib.lib().mfb_plan_info_get(h, ctypes.byref(info)), "row-split plan info")
        self.tcgen05 = info.path == 0
        self.stream_k = info.stream_k_tiles > 0  # whole-matrix multiplies add a fix-up launch

    def set_sm_limit(self, sms: Optional[int]) -> None:
        sms = int(sms or 0)
        if sms != self.sm_limit:
            _lib.check(_lib.lib().mfb_plan_set_sm_limit(self.handle, sms), "plan sm limit")
            self.sm_limit = sms

    def prepare(self, stream: int, a: int, b: int) -> None:
        _lib.check(_lib.lib().mfb_plan_prepare(self.handle, stream, a, b), "plan prepare")

    def prepare_cols(self, stream: int, b: int, ldb: int, n0: int, n1: int) -> None:
        _lib.check(_lib.lib().mfb_plan_prepare_cols(self.handle, stream, b, ldb, n0, n1), "plan prepare columns")

    def multiply(self, stream: int, a: int, b: int, c: int, alpha: float, beta: float) -> None:
        _lib.check(_lib.lib().mfb_plan_multiply(self.handle, stream, a, b, c, alpha, beta, 0), "plan multiply")

    def execute(self, stream: int, a: int, b: int, c: int, alpha: float, beta: float) -> None:
        _lib.check(_lib.lib().mfb_plan_execute(self.handle, stream, a, b, c, alpha, beta, 0), "plan execute")

    def multiply_cols(self, stream: int, a: int, c: int, alpha: float, beta: float, n0: int, n1: int) -> None:
        _lib.check(_lib.lib().mfb_plan_multiply_cols(self.handle, stream, a, c, alpha, beta, 0, n0, n1),
                   "plan multiply columns")

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
    (k x ldb) buffer, read on `src` (other ranks' B is not touched: the panels arrive in
    the object's own buffers); C_local: (m_local x n) view of an (m_local x ldc) buffer."""

    def __init__(self, m_local: int, n: int, k: int, lda: int, ldb: int, ldc: int,
                 precision: GemmPrecision = GemmPrecision.fp32, group=None, src: int = 0, comm_sms: int = 32):
        self.device = torch.cuda.current_device()
        self.group, self.src = group, src
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.m, self.n, self.k = m_local, n, k
        self.lda, self.ldb, self.ldc = lda, ldb, ldc
        total_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.plan = _PointerPlan(self.device, m_local, n, k, lda, ldb, ldc, int(precision))
        self.plans = [self.plan]
        self.sched = schedule(n, self.world if self.plan.tcgen05 else 1, comm_sms, total_sms, k)
        # Contiguous column panels of B, the broadcast buffers (several ranks only).
        self.panel_bufs: List[torch.Tensor] = []
        self.side = torch.cuda.Stream(self.device) if self.world > 1 else None
        if self.world > 1 and self.plan.tcgen05:
            self.panel_bufs = [torch.empty((k, n1 - n0), dtype=torch.float32, device=self.device)
                               for (n0, n1) in self.sched.panels]
        # GEMM kernel time of the last step per panel, when events are requested.
        self.kernel_events: List[Tuple[torch.cuda.Event, torch.cuda.Event]] = []
        # SMs are left to NCCL only while broadcasts run: a panel's GEMM is capped (sched.sm_limits)
        # until a step shows it started after the last panel had arrived (see _update_caps).
        self.capped = [lim is not None for lim in self.sched.sm_limits]
        self._gemm_start = [torch.cuda.Event(enable_timing=True) for _ in self.sched.panels]
        self._arrived_last = torch.cuda.Event(enable_timing=True)
        self._recorded = False

    def _update_caps(self) -> None:
        """From the previous step's events: a panel whose GEMM started after the last panel had
        arrived (all broadcasts done) runs on every SM from now on; one that started before stays
        capped. The first panel always overlaps the later broadcasts. Local to this rank (no
        collective), and only once the previous step's events have completed."""
        if not self._recorded or not self._arrived_last.query():
            return
        for i in range(len(self.sched.panels) - 1):
            start = self._gemm_start[i]
            # started at least 50 us after the last panel landed: no broadcast left to make room for
            if self.capped[i] and start.query() and start.elapsed_time(self._arrived_last) <= -0.05:
                self.capped[i] = False

    def __call__(self, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
                 time_kernels: bool = False) -> None:
        stream = _stream_handle()
        a0, b0, c0 = A.data_ptr(), B.data_ptr(), C.data_ptr()
        self.kernel_events = []
        plan = self.plan

        def timed(fn):
            if time_kernels:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                self.kernel_events.append((e0, e1))
            else:
                fn()

        if self.world == 1:
            plan.set_sm_limit(None)
            if time_kernels:
                # the two phases apart, so that events bracket the GEMM kernel alone
                plan.prepare(stream, a0, b0)
                timed(lambda: plan.multiply(stream, a0, b0, c0, alpha, beta))
            else:
                # one call: one prepass launch for both operands, then the GEMM, launched
                # programmatically so that it sets up while the prepass drains
                plan.execute(stream, a0, b0, c0, alpha, beta)
            return
        if not plan.tcgen05:
            # GEMV / scale plans: B's whole (k x ldb) storage is broadcast in place (it is
            # overwritten on the other ranks), then the plan runs as on one GPU.
            storage = B.as_strided((self.k, self.ldb), (self.ldb, 1), B.storage_offset())
            run_schedule(self.sched, lambda i: storage, lambda i, p: None,
                         lambda i, p, lim: timed(lambda: plan.multiply(stream, a0, b0, c0, alpha, beta)),
                         self.group, self.src)
            return

        def pack(i, panel):
            n0, n1 = panel
            self.panel_bufs[i].copy_(B[:, n0:n1])

        def prepare_a():
            # A's split/rounding prepass does not read B: it runs while B is in flight.
            plan.prepare(stream, a0, 0)

        def prepare_panel(i, panel):
            # the panel's B prepass, on whichever stream is current (the side stream for
            # panels after the first: it overlaps the previous panel's GEMM)
            n0, n1 = panel
            if i == len(self.sched.panels) - 1:
                self._arrived_last.record(torch.cuda.current_stream())  # every broadcast has landed
            plan.prepare_cols(_stream_handle(), self.panel_bufs[i].data_ptr(), n1 - n0, n0, n1)

        def panel_gemm(i, panel, sm_limit):
            n0, n1 = panel
            plan.set_sm_limit(sm_limit if self.capped[i] else None)
            self._gemm_start[i].record(torch.cuda.current_stream())
            timed(lambda: plan.multiply_cols(stream, a0, c0, alpha, beta, n0, n1))

        self._update_caps()
        run_schedule(self.sched, lambda i: self.panel_bufs[i], pack, panel_gemm, self.group, self.src,
                     before_wait=prepare_a, prepare_panel=prepare_panel, side=self.side)
        self._recorded = True

    def launches_per_step(self) -> int:
        """Kernels of this library per step: on one GPU the operand prepass (hi/lo split, or TF32
        rounding), the GEMM and, when its last tiles share K among the SMs (stream-K), their
        fix-up; with peers A's prepass, then per column panel its B prepass and its GEMM (column
        panels stay data parallel; the panel packing on rank 0 is a torch copy)."""
        if self.world == 1 or not self.plan.tcgen05:
            return 3 if self.plan.stream_k else 2
        return 1 + 2 * len(self.sched.panels)

    def gemm_launches_per_step(self) -> int:
        """GEMM kernels per step (one per column panel)."""
        return len(self.sched.panels)

    def kernel_ms(self) -> float:
        return sum(e0.elapsed_time(e1) for (e0, e1) in self.kernel_events)

    def panel_flops(self) -> List[float]:
        return [2.0 * self.m * (n1 - n0) * self.k for (n0, n1) in self.sched.panels]

    def close(self) -> None:
        self.plan.close()
        self.plans = []
