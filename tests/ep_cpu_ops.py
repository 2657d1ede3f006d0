"""CPU stand-in for the device steps of d3moe.ep (test infrastructure only).

It lets the expert-parallel exchange (row plan, FP8 row packing, all_to_all
dispatch, expert compute on the owner, return, combine) run on gloo CPU
ranks. The arithmetic
is the oracle's, so an EP run can be compared with the single-process oracle
layer.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as O


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(O.bf16_to_bits(np.asarray(a, np.float32)).view(np.int16)).view(torch.bfloat16)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


class CpuExperts:
    """Expert container whose w13_weight has the [E, 2I, H] shape of the real one."""

    def __init__(self, ex: "O.Experts", E: int, I: int, H: int):
        self.ex = ex
        self.w13_weight = torch.empty((E, 2 * I, H), dtype=torch.uint8)


class CpuEPOps:
    def router_logits(self, x, router_weight, bias=None):
        if bias is None:
            return _bf16(O.router_logits(_np(x), _np(router_weight)))
        return _bf16(O.router_logits(_np(x), _np(router_weight), bias.numpy(), nbias=bias.numel()))

    def route(self, logits, k, bias=None):
        w, ids = O.route(_np(logits), k, None if bias is None else bias.numpy())
        return _bf16(O.bf16_round(w)), torch.from_numpy(ids)

    def plan_rows(self, ids, experts_per_rank, ranks):
        """d3_ep_plan_rows: one row per (token, rank owning >= 1 of its
        experts), ordered by rank then token."""
        idn = ids.numpy()
        T = idn.shape[0]
        owned = experts_per_rank * ranks
        need = np.zeros((T, ranks), bool)
        for t in range(T):
            for e in idn[t]:
                if 0 <= e < owned:
                    need[t, e // experts_per_rank] = True
        counts = need.sum(axis=0).astype(np.int32)
        starts = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
        slot = np.full((T, ranks), -1, np.int32)
        for d in range(ranks):
            rows = np.nonzero(need[:, d])[0]
            slot[rows, d] = starts[d] + np.arange(rows.size, dtype=np.int32)
        return torch.from_numpy(counts), torch.from_numpy(slot)

    def dispatch_meta(self, ids, weights, experts_per_rank, ranks):
        T, k = ids.shape
        idn = ids.numpy()
        wn = weights
        meta_ids = np.full((ranks, T, k), -1, np.int64)
        meta_w = torch.zeros((ranks, T, k), dtype=torch.bfloat16)
        for d in range(ranks):
            mine = (idn // experts_per_rank) == d
            meta_ids[d][mine] = idn[mine] - d * experts_per_rank
            meta_w[d][torch.from_numpy(mine)] = wn[torch.from_numpy(mine)]
        return torch.from_numpy(meta_ids), meta_w

    def pack_fp8(self, x, ids, weights, experts_per_rank, ranks, slot=None, rows=None):
        """The FP8 packed dispatch rows of d3_ep_pack_fp8: the oracle's 1x128
        quantiser bytes, group scales, then dispatch_meta's ids and weights,
        at row d*T + t, or at slot[t, d] with a plan_rows slot map."""
        from d3moe.ep import ep_row_bytes_fp8
        T, H = x.shape
        k = ids.shape[1]
        rb = ep_row_bytes_fp8(H, k)
        G = H // 128
        q, sx = O.quant_act_fp8(_np(x))
        qb = torch.from_numpy(np.ascontiguousarray(q, np.uint8))
        sb = torch.from_numpy(np.ascontiguousarray(sx, np.float32)).view(torch.uint8)
        meta_ids, meta_w = self.dispatch_meta(ids, weights, experts_per_rank, ranks)
        n = ranks * T if slot is None else rows
        send = torch.zeros((n, rb), dtype=torch.uint8)
        off = H + 4 * G
        for d in range(ranks):
            for t in range(T):
                r = d * T + t if slot is None else int(slot[t, d])
                if r < 0:
                    continue
                send[r, :H] = qb[t]
                send[r, H: off] = sb[t]
                send[r, off: off + 8 * k] = meta_ids[d, t].contiguous().view(torch.uint8)
                send[r, off + 8 * k: off + 10 * k] = meta_w[d, t].contiguous().view(torch.uint8)
        return send.reshape(ranks, T * rb) if slot is None else send

    def unpack_fp8(self, recv, rows, k, H):
        from d3moe.ep import ep_row_bytes_fp8
        rb = ep_row_bytes_fp8(H, k)
        G = H // 128
        r = recv.reshape(rows, rb)
        q = r[:, :H].contiguous()
        scales = r[:, H: H + 4 * G].contiguous().view(torch.float32)
        off = H + 4 * G
        ids = r[:, off: off + 8 * k].contiguous().view(torch.int64)
        w = r[:, off + 8 * k: off + 10 * k].contiguous().view(torch.bfloat16)
        return q, scales, ids, w

    def local_experts_fp8(self, q, scales, ids, weights, experts):
        """Oracle expert sum over each row's valid ids, on the received bytes."""
        qn = q.numpy()
        sx = scales.numpy()
        idn = ids.numpy()
        w = _np(weights)
        M, k = idn.shape
        ex = experts.ex
        acc = np.zeros((M, qn.shape[1]), np.float32)
        for j in range(k):
            valid = idn[:, j] >= 0
            if not valid.any():
                continue
            sel = np.nonzero(valid)[0]
            e_ids = idn[sel, j].reshape(-1, 1)
            gu = O.expert_gate_up(qn[sel], sx[sel], ex.w13, ex.s13, e_ids)
            a, sa = O.silu_mul_quant(gu)
            d = O.expert_down_rows(a, sa, ex.w2, ex.s2, e_ids)
            acc[sel] = (acc[sel] + d * w[sel, j: j + 1]).astype(np.float32)
        return _bf16(O.bf16_round(acc))

    def shared_expert(self, x, shared):
        T = x.shape[0]
        out, _ = O.moe_experts(_np(x), np.zeros((T, 1), np.int64), np.ones((T, 1), np.float32), shared.ex)
        return _bf16(out)

    def combine(self, rows, inv, weights, shared, gate):
        T, k = weights.shape
        r = _np(rows)
        w = _np(weights)
        acc = np.zeros((T, r.shape[1]), np.float32)
        invn = inv.numpy().reshape(T, k)
        for j in range(k):
            idx = invn[:, j]
            term = np.where((idx >= 0)[:, None], r[np.maximum(idx, 0)] * w[:, j: j + 1], 0.0)
            acc = np.where((idx >= 0)[:, None], acc + term, acc).astype(np.float32)
        routed = O.bf16_round(acc)
        return _bf16(O.combine_experts(routed, _np(shared), _np(gate).reshape(-1)))
