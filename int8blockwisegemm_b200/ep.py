"""Expert parallelism for the INT8 hybrid MoE forward over torch.distributed.

The experts are split contiguously: rank r owns experts
[r*E/P, (r+1)*E/P).  Each rank holds a contiguous shard of the tokens.  A
forward is one dispatch all-to-all, the unchanged single-GPU forward over the
rows that reached this rank (restricted to its local experts by an
``expert_map``, as the reference runner supports), and one combine
all-to-all:

* dispatch: every token row travels once to every rank that owns at least one
  of its top-k experts, together with its top-k ids and weights.  Segments
  are ordered by source rank and, within one, by token index, so the rows a
  rank receives are in global token order.  The stable per-expert sort of the
  local routing then puts every expert's rows in the same order as a
  single-GPU run.  With the tile_m of the single-GPU run (chosen from the
  global rows per expert) the INT8 activation tiles, scales, int32
  accumulators and mm1/mm2 rows of each expert are therefore bit-identical
  to the single-GPU forward.
* combine, two forms.  Top-k combine (the peer exchange's "topk" mode): the
  local forward stops after the w2 GEMM and each source rank performs the
  whole top-k weighted unpermute of its own tokens, reading every slot's
  mm2 row from the rank that owns the slot's expert -- fp32 in top-k order
  and one rounding, so the output equals a single-GPU forward bit for bit
  and no rank runs an unpermute pass.  Partial-row combine (NCCL, and the
  peer exchange's default "rows" mode): the local forward ends with the unpermute
  over this rank's experts (the reference's ``expert_map`` skip), the
  partial rows return to their source ranks, which add them in fp32 in rank
  order (one segment per rank, so the order is deterministic) and round
  once; this moves fewer bytes (one row per token and destination rank
  rather than one per top-k slot) but rounds each partial sum, so the output
  agrees with one GPU within the reference's tolerance, not bit for bit.

Two exchanges implement that on GPUs.  ``PeerExchange`` (the default of
``bench.py``) stores rows straight into the peers' receive buffers over NVLink
peer memory with device-side flags: no NCCL call and no host synchronisation
per step, so whole steps are CUDA-graph replays.  ``ExpertParallel`` uses
NCCL ``all_to_all_single`` calls; the bookkeeping around them runs in the
library's kernels (csrc/ep.cu): a plan kernel gives every token its slot in
each destination's segment, a pack kernel gathers the rows with their top-k
ids and weights, and a combine kernel sums the returned partial rows.  The
segment lengths of all ranks travel first (one all-gather) and their host copy
sizes the payload exchange: one host synchronisation per dispatch.  There is
no CPU path; the gloo tests run the same exchange order with a torch-only
stand-in kept under tests/.
"""

from __future__ import annotations

import ctypes

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass
class Dispatched:
    """Rows this rank received and what the combine needs to send them back."""
    hidden: torch.Tensor        # [n_recv, K]
    topk_ids: torch.Tensor      # [n_recv, k] int32, global expert ids
    topk_weights: torch.Tensor  # [n_recv, k] float32
    send_idx: torch.Tensor      # [n_send] int64 local token index of every sent row
    send_counts: list[int]      # rows sent to each rank
    recv_counts: list[int]      # rows received from each rank
    n_token: int                # local tokens
    pos: torch.Tensor | None = None  # [n_token, P] slot in each send segment or -1 (GPU path)


class ExpertParallel:
    """Dispatch / combine for ``num_experts`` experts over ``group``."""

    def __init__(self, num_experts: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if num_experts % self.world != 0:
            raise ValueError(f"num_experts={num_experts} is not divisible by the "
                             f"{self.world} ranks of the group")
        self.num_experts = num_experts
        self.n_local = num_experts // self.world
        self.first = self.rank * self.n_local

    def expert_map(self, device) -> torch.Tensor:
        """global expert id -> local id, -1 for experts of other ranks."""
        m = torch.full((self.num_experts,), -1, dtype=torch.int32)
        m[self.first:self.first + self.n_local] = torch.arange(self.n_local, dtype=torch.int32)
        return m.to(device)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits) -> None:
        dist.all_to_all_single(out, inp, output_split_sizes=list(out_splits),
                               input_split_sizes=list(in_splits), group=self.group)

    def dispatch(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                 topk_weights: torch.Tensor) -> Dispatched:
        if not hidden.is_cuda:
            raise RuntimeError("expert parallelism runs on CUDA tensors (sm_100a); "
                               "there is no CPU path")
        return self._dispatch_cuda(hidden, topk_ids, topk_weights)

    def _dispatch_cuda(self, hidden, topk_ids, topk_weights) -> Dispatched:
        from ._lib import call
        T, k = topk_ids.shape
        K = hidden.shape[1]
        dev, P = hidden.device, self.world
        stream = torch.cuda.current_stream(dev).cuda_stream
        hidden = hidden.contiguous()
        ids = topk_ids.to(torch.int32).contiguous()
        wts = topk_weights.to(torch.float32).contiguous()
        pos = torch.empty(T, P, dtype=torch.int32, device=dev)
        lst = torch.empty(P, max(T, 1), dtype=torch.int32, device=dev)
        counts = torch.empty(P, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            call("i8moe_ep_plan", ids.data_ptr(), T, k, self.n_local, P, pos.data_ptr(),
                 lst.data_ptr(), counts.data_ptr(), stream)
        allc = torch.empty(P * P, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(allc, counts.to(torch.int64), group=self.group)
        allc = allc.view(P, P).cpu()  # the one host synchronisation of the exchange
        send_counts = allc[self.rank].tolist()
        recv_counts = allc[:, self.rank].tolist()
        n_send, n_recv = sum(send_counts), sum(recv_counts)
        send_rows = torch.empty(n_send, K, dtype=hidden.dtype, device=dev)
        send_meta = torch.empty(n_send, 2 * k, dtype=torch.int32, device=dev)
        host_counts = (ctypes.c_int64 * P)(*send_counts)
        with torch.cuda.device(dev):
            call("i8moe_ep_pack", hidden.data_ptr(), K * hidden.element_size(), ids.data_ptr(),
                 wts.data_ptr(), k, lst.data_ptr(), T, P, ctypes.addressof(host_counts),
                 send_rows.data_ptr(), send_meta.data_ptr(), stream)
        r_hidden = torch.empty(n_recv, K, dtype=hidden.dtype, device=dev)
        r_meta = torch.empty(n_recv, 2 * k, dtype=torch.int32, device=dev)
        self._a2a(r_hidden, send_rows, recv_counts, send_counts)
        self._a2a(r_meta, send_meta, recv_counts, send_counts)
        r_ids = r_meta[:, :k].contiguous()
        r_w = r_meta[:, k:].contiguous().view(torch.float32)
        return Dispatched(r_hidden, r_ids, r_w, None, send_counts, recv_counts, T, pos)

    def combine(self, d: Dispatched, partial: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Return the partial rows to their sources and sum them per token."""
        if not (partial.is_cuda and d.pos is not None):
            raise RuntimeError("expert parallelism runs on CUDA tensors (sm_100a); "
                               "there is no CPU path")
        return self._combine_cuda(d, partial, out)

    def _combine_cuda(self, d: Dispatched, partial: torch.Tensor, out):
        from ._lib import BF16, FP16, call
        K = partial.shape[1]
        dev, P = partial.device, self.world
        back = torch.empty(sum(d.send_counts), K, dtype=partial.dtype, device=dev)
        self._a2a(back, partial.contiguous(), d.send_counts, d.recv_counts)
        if out is None:
            out = torch.empty(d.n_token, K, dtype=partial.dtype, device=dev)
        host_counts = (ctypes.c_int64 * P)(*d.send_counts)
        dt = {torch.bfloat16: BF16, torch.float16: FP16}[partial.dtype]
        with torch.cuda.device(dev):
            call("i8moe_ep_combine", back.data_ptr(), dt, d.pos.data_ptr(), d.n_token, P,
                 ctypes.addressof(host_counts), K, out.data_ptr(),
                 torch.cuda.current_stream(dev).cuda_stream)
        return out

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                local_forward: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                out: torch.Tensor | None = None) -> torch.Tensor:
        """dispatch -> ``local_forward(hidden, topk_ids, topk_weights)`` -> combine.

        ``local_forward`` returns the [n_recv, K] partial output of this
        rank's experts for the received rows."""
        d = self.dispatch(hidden, topk_ids, topk_weights)
        partial = local_forward(d.hidden, d.topk_ids, d.topk_weights)
        return self.combine(d, partial, out)


class _Layout(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in ("off_rows", "off_ids", "off_w", "off_out", "out_bytes",
                                              "off_inbox", "off_flags", "off_epoch", "off_mm2",
                                              "mm2_bytes", "off_inv", "inv_bytes", "bytes")]


COMBINE_ROWS, COMBINE_TOPK = 0, 1  # I8MOE_EP_COMBINE_ROWS / _TOPK of include/i8moe.h


class _P2PDesc(ctypes.Structure):
    """``i8moe_ep_p2p`` of include/i8moe.h."""
    _fields_ = [("bases", ctypes.c_void_p * 32), ("n_rank", ctypes.c_int64), ("rank", ctypes.c_int64),
                ("n_token", ctypes.c_int64), ("capacity", ctypes.c_int64), ("topk", ctypes.c_int64),
                ("n_hidden", ctypes.c_int64), ("elem_bytes", ctypes.c_int64),
                ("pad_expert", ctypes.c_int64), ("layout", _Layout)]


class _DeviceArray:
    """A borrowed device buffer seen through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3, "strides": None}


class PeerExchange:
    """Expert-parallel dispatch / combine over NVLink peer memory: no NCCL
    call and no host synchronisation in a step (csrc/ep.cu, ``ep_p2p_*``).

    Every rank allocates one region (receive rows, ids and weights for
    ``capacity = world * max_tokens`` rows, two output buffers, the
    segment-length inbox and the step flags) and maps the other ranks'
    regions through CUDA IPC handles exchanged once over the process group.
    A step runs ep_plan, the dispatch (rows stored straight into the
    destinations' receive buffers), a wait for every source's rows, the
    local forward over the ``capacity`` receive rows, the "output ready"
    signal and the combine.  Every shape is static, so whole steps can be
    captured in CUDA graphs.

    ``combine="rows"`` (the default): the local forward ends with the
    unpermute over this rank's experts into the output buffer and the
    combine adds the returned partial rows in rank order.
    ``combine="topk"``: the local forward stops after the w2 GEMM, writing
    its mm2 rows and the routing's inverse map into this step's region
    buffers, and the combine performs the whole top-k weighted unpermute of
    this rank's tokens from the peers' mm2 rows -- one fp32 fma chain in
    top-k order and one rounding, so the output equals a single-GPU forward
    bit for bit, and no rank runs an unpermute pass.  It reads one row per
    top-k slot over NVLink instead of one per destination rank (8 against
    about 2 at two ranks, 8 against about 5.25 at eight), which at two
    ranks costs more than the unpermute it removes (0.955 against 0.892 ms
    per step at the default shape)."""

    def __init__(self, ep: ExpertParallel, max_tokens: int, n_hidden: int, topk: int,
                 dtype: torch.dtype, device, combine: str = "rows"):
        from ._lib import call
        assert dtype in (torch.bfloat16, torch.float16) and ep.world >= 2
        if combine not in ("topk", "rows"):
            raise ValueError(f"combine must be 'topk' or 'rows', not {combine!r}")
        self.ep, self.device, self.dtype = ep, torch.device(device), dtype
        P, r = ep.world, ep.rank
        self.P, self.k, self.K, self.T = P, topk, n_hidden, max_tokens
        self.C = P * max_tokens
        self.combine = combine
        lay = _Layout()
        call("i8moe_ep_p2p_region_bytes", P, self.C, topk, n_hidden, 2,
             COMBINE_TOPK if combine == "topk" else COMBINE_ROWS, ctypes.addressof(lay))
        ptr, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
        with torch.cuda.device(self.device):
            call("i8moe_ep_ipc_alloc", lay.bytes, ctypes.addressof(ptr), ctypes.addressof(handle))
        self._own = ptr.value
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        every = torch.empty(P * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=ep.group)
        every = every.view(P, 64).cpu()
        self._opened = []
        desc = _P2PDesc()
        for d in range(P):
            if d == r:
                desc.bases[d] = self._own
                continue
            h = (ctypes.c_uint8 * 64)(*every[d].tolist())
            p = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                call("i8moe_ep_ipc_open", ctypes.addressof(h), ctypes.addressof(p))
            self._opened.append(p.value)
            desc.bases[d] = p.value
        desc.n_rank, desc.rank, desc.n_token, desc.capacity = P, r, max_tokens, self.C
        desc.topk, desc.n_hidden, desc.elem_bytes = topk, n_hidden, 2
        # an expert of the next rank: the local routing skips padding rows
        desc.pad_expert = ((r + 1) % P) * ep.n_local
        desc.layout = lay
        self._desc = desc
        base, C, k, K = self._own, self.C, topk, n_hidden
        as_t = lambda off, shape, ts: torch.as_tensor(_DeviceArray(base + off, shape, ts),
                                                      device=self.device)
        self.recv_rows = as_t(lay.off_rows, (C, K), "<i2").view(dtype)
        self.recv_ids = as_t(lay.off_ids, (C, k), "<i4")
        self.recv_w = as_t(lay.off_w, (C, k), "<f4")
        if combine == "rows":
            self.out_buf = [as_t(lay.off_out + i * lay.out_bytes, (C, K), "<i2").view(dtype)
                            for i in range(2)]
        else:
            self.mm2_buf = [as_t(lay.off_mm2 + i * lay.mm2_bytes, (C * k, K), "<i2").view(dtype)
                            for i in range(2)]
            self.inv_buf = [as_t(lay.off_inv + i * lay.inv_bytes, (C * k,), "<i4")
                            for i in range(2)]
        self.pos = torch.empty(max_tokens, P, dtype=torch.int32, device=self.device)
        self.lst = torch.empty(P, max_tokens, dtype=torch.int32, device=self.device)
        self.counts = torch.empty(P, dtype=torch.int32, device=self.device)
        self.step = 0
        dist.barrier(group=ep.group)  # every region is mapped before any rank writes into one

    def forward(self, hidden, topk_ids, topk_weights, local_forward, out=None):
        """One expert-parallel step.  ``local_forward(rows, ids, weights, out)``
        runs the local experts over the ``capacity`` receive rows into out
        (combine="rows"); with combine="topk" it is called as
        ``local_forward(rows, ids, weights, None, mm2=..., inv=...)`` and
        must leave the w2 GEMM rows in ``mm2`` and the inverse map in
        ``inv`` instead."""
        from ._lib import BF16, FP16, call
        T, k = topk_ids.shape
        assert T <= self.T and k == self.k and hidden.shape[1] == self.K
        assert hidden.dtype == self.dtype and hidden.is_contiguous()
        par = self.step & 1
        self.step += 1
        self._desc.n_token = T
        st = torch.cuda.current_stream(self.device).cuda_stream
        ids = topk_ids.to(torch.int32).contiguous()
        wts = topk_weights.to(torch.float32).contiguous()
        if out is None:
            out = torch.empty(T, self.K, dtype=self.dtype, device=self.device)
        d = ctypes.addressof(self._desc)
        with torch.cuda.device(self.device):
            call("i8moe_ep_plan", ids.data_ptr(), T, k, self.ep.n_local, self.P,
                 self.pos.data_ptr(), self.lst.data_ptr(), self.counts.data_ptr(), st)
            call("i8moe_ep_p2p_dispatch", d, par, hidden.data_ptr(), ids.data_ptr(),
                 wts.data_ptr(), self.lst.data_ptr(), self.counts.data_ptr(), st)
            call("i8moe_ep_p2p_wait", d, par, st)
        dt = {torch.bfloat16: BF16, torch.float16: FP16}[self.dtype]
        if self.combine == "rows":
            local_forward(self.recv_rows, self.recv_ids, self.recv_w, self.out_buf[par])
            with torch.cuda.device(self.device):
                call("i8moe_ep_p2p_ready", d, par, st)
                call("i8moe_ep_p2p_combine", d, par, dt, self.pos.data_ptr(), out.data_ptr(), st)
            return out
        local_forward(self.recv_rows, self.recv_ids, self.recv_w, None,
                      mm2=self.mm2_buf[par], inv=self.inv_buf[par])
        with torch.cuda.device(self.device):
            call("i8moe_ep_p2p_ready", d, par, st)
            call("i8moe_ep_p2p_combine_topk", d, par, dt, self.pos.data_ptr(), ids.data_ptr(),
                 wts.data_ptr(), self.ep.n_local, out.data_ptr(), st)
        return out

    def close(self):
        """Unmap the peers' regions and free this rank's (collective)."""
        from ._lib import call
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.ep.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                call("i8moe_ep_ipc_close", p)
            dist.barrier(group=self.ep.group)
            call("i8moe_ep_ipc_free", self._own)
        self._own = None


def global_tile_m(n_token_global: int, topk: int, num_experts: int) -> int:
    """tile_m of the single-GPU run (cutlass_runner.py:43-50 on the global
    rows per expert), which keeps the EP quant tiles identical to it."""
    from .cutlass_runner import _variant_tile_m, pick_grouped_hybrid_variant
    return _variant_tile_m(pick_grouped_hybrid_variant(n_token_global * topk, num_experts))


class EPMoE:
    """Expert-parallel INT8 hybrid MoE forward on the sm_100a kernels.

    Holds this rank's slice of the expert weights (experts
    [rank*E/P, (rank+1)*E/P)) and runs ``cutlass_runner`` on the rows the
    dispatch delivers."""

    def __init__(self, ep: ExpertParallel, w1, w2, w1_qscale, w1_fscale, w2_qscale, w2_fscale,
                 *, quant_block_size: int, super_group_size: int, q_max: int, tile_m: int):
        lo, n = ep.first, ep.n_local
        self.ep = ep
        self.w1, self.w2 = w1[lo:lo + n].contiguous(), w2[lo:lo + n].contiguous()
        self.w1_q, self.w1_f = w1_qscale[lo:lo + n].contiguous(), w1_fscale[lo:lo + n].contiguous()
        self.w2_q, self.w2_f = w2_qscale[lo:lo + n].contiguous(), w2_fscale[lo:lo + n].contiguous()
        self.qbs, self.sg, self.q_max, self.tile_m = quant_block_size, super_group_size, q_max, tile_m
        self.emap = ep.expert_map(w1.device)
        self._ws = None

    def _workspaces(self, rows: int, K: int, N: int, dtype, device, with_ws2: bool = True):
        need13, need2 = rows * max(2 * N, K), rows * max(N, K) if with_ws2 else 0
        if (self._ws is None or self._ws[0].numel() < need13 or self._ws[1].numel() < need2
                or self._ws[0].dtype != dtype):
            self._ws = (torch.empty(need13, dtype=dtype, device=device),
                        torch.empty(need2, dtype=dtype, device=device))
        ws2 = self._ws[1][:need2].view(rows, -1) if with_ws2 else None
        return self._ws[0][:need13].view(rows, -1), ws2

    def local_forward(self, hidden, topk_ids, topk_weights, trace: dict | None = None, out=None,
                      mm2=None, inv=None):
        """The runner over the received rows with this rank's experts.  With
        ``mm2`` / ``inv`` (the top-k combine) the w2 GEMM rows go to ``mm2``
        ([rows * topk, K]), the inverse map to ``inv`` and no unpermute
        runs."""
        from .activation import MoEActivation
        from .cutlass_runner import _run_cutlass_int8_hybrid_grouped_moe
        T, k = topk_ids.shape
        K, N = hidden.shape[1], self.w2.shape[2]
        topk_combine = mm2 is not None
        if out is None and not topk_combine:
            out = torch.empty(T, K, dtype=hidden.dtype, device=hidden.device)
        if T == 0:
            return out
        ws13, ws2 = self._workspaces(T * k, K, N, hidden.dtype, hidden.device,
                                     with_ws2=not topk_combine)
        if topk_combine:
            # mm2 is [rows*k, K]: it holds every view the runner takes of
            # workspace2 ([rows*k, N] and [rows*k, K])
            assert mm2.shape == (T * k, K) and mm2.dtype == hidden.dtype and N <= K
            assert inv is not None and inv.numel() == T * k
            ws2 = mm2
        _run_cutlass_int8_hybrid_grouped_moe(
            out, hidden, self.w1, self.w2, topk_ids, topk_weights, MoEActivation.SILU,
            self.ep.num_experts, self.emap, self.w1_q, self.w1_f, self.w2_q, self.w2_f,
            ws13, ws2, self.qbs, self.sg, self.q_max, _trace=trace, _tile_m=self.tile_m,
            _inv_out=inv, _unpermute=not topk_combine)
        return out

    def enable_peer_exchange(self, max_tokens: int, n_hidden: int, topk: int, dtype,
                             combine: str = "rows"):
        """Use the NVLink peer-memory exchange (no NCCL, no host
        synchronisation) for steps of up to ``max_tokens`` tokens per rank."""
        self.p2p = PeerExchange(self.ep, max_tokens, n_hidden, topk, dtype, self.w1.device,
                                combine=combine)
        return self.p2p

    def forward(self, hidden, topk_ids, topk_weights, out=None, trace: dict | None = None):
        p2p = getattr(self, "p2p", None)
        if p2p is not None and hidden.is_cuda:
            return p2p.forward(
                hidden, topk_ids, topk_weights,
                lambda h, i, w, o, mm2=None, inv=None: self.local_forward(
                    h, i, w, trace, out=o, mm2=mm2, inv=inv), out)
        return self.ep.forward(
            hidden, topk_ids, topk_weights,
            lambda h, i, w: self.local_forward(h, i, w, trace), out)
