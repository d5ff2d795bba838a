"""Torch-only stand-in for the expert-parallel exchange, for the gloo tests.

The product exchange (int8blockwisegemm_b200.ep) runs on CUDA tensors only.
This subclass gives CPU tensors the same dispatch / combine semantics with
plain torch ops and ``all_to_all_single`` over gloo: every token row travels
once to each rank owning one of its experts, segments ordered by source rank
and by token within one, and the partial rows come back to be summed in fp32
in rank order.  Test infrastructure only."""

from __future__ import annotations

import torch

from int8blockwisegemm_b200.ep import Dispatched, ExpertParallel


class CPUExchange(ExpertParallel):
    def dispatch(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                 topk_weights: torch.Tensor) -> Dispatched:
        T, k = topk_ids.shape
        dev = hidden.device
        dest = topk_ids.long() // self.n_local                       # [T, k]
        member = torch.zeros(T, self.world, dtype=torch.bool, device=dev)
        member.scatter_(1, dest.clamp(0, self.world - 1), True)
        # rows for rank d: the tokens with an expert on d, in token order
        order = member.t().nonzero()                                 # [n_send, 2] (rank, token)
        send_idx = order[:, 1]
        counts = member.sum(0).to(torch.int64)                       # [P]
        recv = torch.empty_like(counts)
        self._a2a(recv, counts, [1] * self.world, [1] * self.world)
        send_counts = counts.tolist()
        recv_counts = recv.tolist()
        n_recv = sum(recv_counts)
        r_hidden = torch.empty(n_recv, hidden.shape[1], dtype=hidden.dtype, device=dev)
        r_ids = torch.empty(n_recv, k, dtype=torch.int32, device=dev)
        r_w = torch.empty(n_recv, k, dtype=torch.float32, device=dev)
        self._a2a(r_hidden, hidden.index_select(0, send_idx).contiguous(), recv_counts,
                  send_counts)
        self._a2a(r_ids, topk_ids.to(torch.int32).index_select(0, send_idx).contiguous(),
                  recv_counts, send_counts)
        self._a2a(r_w, topk_weights.to(torch.float32).index_select(0, send_idx).contiguous(),
                  recv_counts, send_counts)
        return Dispatched(r_hidden, r_ids, r_w, send_idx, send_counts, recv_counts, T)

    def combine(self, d: Dispatched, partial: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        K = partial.shape[1]
        back = torch.empty(sum(d.send_counts), K, dtype=partial.dtype, device=partial.device)
        self._a2a(back, partial.contiguous(), d.send_counts, d.recv_counts)
        acc = torch.zeros(d.n_token, K, dtype=torch.float32, device=partial.device)
        start = 0
        for n in d.send_counts:  # each segment holds distinct tokens: a deterministic order
            if n:
                acc.index_add_(0, d.send_idx[start:start + n], back[start:start + n].float())
            start += n
        if out is None:
            return acc.to(partial.dtype)
        out.copy_(acc)
        return out
